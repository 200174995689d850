"""Eager numpy versions of the ``jax.lax`` control-flow and slicing helpers.

Test infrastructure only.  Start indices are clamped the way XLA clamps them
(the slice is shifted to fit inside the operand).
"""

from __future__ import annotations

import numpy as _np

from .numpy import Array as _Array

_MISSING = object()


class Precision:
    HIGHEST = "highest"
    DEFAULT = "default"


def cond(pred, true_fun, false_fun, *operands, operand=_MISSING):
    if operand is not _MISSING:
        operands = (operand,)
    return true_fun(*operands) if bool(pred) else false_fun(*operands)


def fori_loop(lower, upper, body_fun, init_val):
    val = init_val
    for i in range(int(lower), int(upper)):
        val = body_fun(i, val)
    return val


def _clamp_starts(shape, starts, sizes):
    out = []
    for dim, s, n in zip(shape, starts, sizes):
        s = int(s)
        s = max(0, min(s, dim - n))
        out.append(s)
    return out


def dynamic_slice(operand, start_indices, slice_sizes):
    x = _np.asarray(operand)
    starts = _clamp_starts(x.shape, start_indices, slice_sizes)
    idx = tuple(slice(s, s + n) for s, n in zip(starts, slice_sizes))
    return _np.array(x[idx], copy=True).view(_Array)


def dynamic_update_slice(operand, update, start_indices):
    x = _np.array(operand, copy=True)
    u = _np.asarray(update)
    starts = _clamp_starts(x.shape, start_indices, u.shape)
    idx = tuple(slice(s, s + n) for s, n in zip(starts, u.shape))
    x[idx] = u
    return x.view(_Array)


def dynamic_update_slice_in_dim(operand, update, start_index, axis):
    x = _np.asarray(operand)
    starts = [0] * x.ndim
    starts[axis] = start_index
    return dynamic_update_slice(x, update, starts)


def dynamic_index_in_dim(operand, index, axis=0, keepdims=True):
    x = _np.asarray(operand)
    i = int(index)
    i = max(0, min(i, x.shape[axis] - 1))
    out = _np.take(x, [i], axis=axis)
    if not keepdims:
        out = _np.squeeze(out, axis=axis)
    return _np.array(out, copy=True).view(_Array)
