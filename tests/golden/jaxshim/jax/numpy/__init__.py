"""A numpy-backed stand-in for the subset of ``jax.numpy`` that jax_gptq uses.

Test infrastructure only: ``tests/golden/make_golden.py`` puts this package on
``sys.path`` so that the reference's own, unmodified source files can run in a
container without JAX and produce golden vectors.  It follows JAX's default
(x64 disabled) conventions where they matter for the reference's arithmetic:

* float literals and float64 inputs become float32, int64 becomes int32;
* ``argsort`` is stable (``jnp.argsort`` is stable by default);
* arrays are immutable values updated through ``x.at[idx].set(v)``, which
  returns a fresh copy.
"""

from __future__ import annotations

import numpy as _np

float32 = _np.float32
float64 = _np.float64
float16 = _np.float16
int32 = _np.int32
int64 = _np.int64
uint8 = _np.uint8
bool_ = _np.bool_
inf = _np.inf
nan = _np.nan


class _AtIndexer:
    def __init__(self, arr, idx):
        self._arr = arr
        self._idx = idx

    def set(self, value):
        out = _np.array(self._arr, copy=True)
        out[self._idx] = _np.asarray(value)
        return out.view(Array)

    def add(self, value):
        out = _np.array(self._arr, copy=True)
        out[self._idx] += _np.asarray(value)
        return out.view(Array)


class _At:
    def __init__(self, arr):
        self._arr = arr

    def __getitem__(self, idx):
        return _AtIndexer(self._arr, idx)


def _clamp_gather(idx, shape):
    """JAX clamps out-of-range integer-array gathers into bounds (negative
    indices wrap first); numpy would raise.  Applied to every integer-array
    component of an index."""
    parts = idx if isinstance(idx, tuple) else (idx,)
    out, axis = [], 0
    for p in parts:
        if p is None:
            out.append(p)
            continue
        if p is Ellipsis:
            axis = len(shape) - (len(parts) - len(out) - 1)
            out.append(p)
            continue
        if isinstance(p, _np.ndarray) and p.dtype.kind in "iu" and axis < len(shape):
            dim = shape[axis]
            q = _np.where(p < 0, p + dim, p)
            out.append(_np.clip(q, 0, dim - 1))
        else:
            out.append(p)
        axis += 1
    return tuple(out) if isinstance(idx, tuple) else out[0]


class Array(_np.ndarray):
    """ndarray with JAX's functional update helpers."""

    @property
    def at(self):
        return _At(self)

    def block_until_ready(self):
        return self

    def __getitem__(self, idx):
        out = super().__getitem__(_clamp_gather(idx, self.shape))
        if isinstance(out, _np.generic):
            return _np.asarray(out).view(Array)
        return out

    def __bool__(self):
        return bool(_np.asarray(self))

    def __index__(self):
        return int(_np.asarray(self))


ndarray = Array


def _narrow(x):
    x = _np.asarray(x)
    if x.dtype == _np.float64:
        return x.astype(_np.float32)
    if x.dtype == _np.int64:
        return x.astype(_np.int32)
    return x


def _wrap(x):
    if isinstance(x, _np.ndarray):
        return x.view(Array)
    if isinstance(x, (_np.generic,)):
        return _np.asarray(x).view(Array)
    if isinstance(x, tuple):
        return tuple(_wrap(v) for v in x)
    return x


def asarray(x, dtype=None):
    if dtype is not None:
        return _np.asarray(x, dtype=dtype).view(Array)
    if isinstance(x, _np.ndarray):
        return x.view(Array)
    return _narrow(x).view(Array)


def array(x, dtype=None):
    if dtype is not None:
        return _np.array(x, dtype=dtype).view(Array)
    if isinstance(x, _np.ndarray):
        return _np.array(x, copy=True).view(Array)
    return _narrow(_np.array(x)).view(Array)


def zeros(shape, dtype=_np.float32):
    return _np.zeros(shape, dtype=dtype).view(Array)


def ones(shape, dtype=_np.float32):
    return _np.ones(shape, dtype=dtype).view(Array)


def eye(n, dtype=_np.float32):
    return _np.eye(n, dtype=dtype).view(Array)


def arange(*args, dtype=None):
    out = _np.arange(*args)
    if dtype is not None:
        out = out.astype(dtype)
    else:
        out = _narrow(out)
    return out.view(Array)


def argsort(x, axis=-1):
    return _narrow(_np.argsort(_np.asarray(x), axis=axis, kind="stable")).view(Array)


def argmax(x, axis=None):
    return _narrow(_np.argmax(_np.asarray(x), axis=axis)).view(Array)


def argmin(x, axis=None):
    return _narrow(_np.argmin(_np.asarray(x), axis=axis)).view(Array)


def linspace(start, stop, num, dtype=None):
    out = _np.linspace(start, stop, num)
    return out.astype(dtype if dtype is not None else _np.float32).view(Array)


def pad(x, pad_width, **kw):
    return _np.pad(_np.asarray(x), pad_width, **kw).view(Array)


def _passthrough(name):
    fn = getattr(_np, name)

    def wrapped(*args, **kwargs):
        return _wrap(fn(*args, **kwargs))

    wrapped.__name__ = name
    return wrapped


for _name in (
    "reshape", "max", "min", "abs", "maximum", "minimum", "clip", "round",
    "repeat", "where", "sum", "square", "sqrt", "dot", "outer", "diag", "mean",
    "any", "all", "concatenate", "tril", "triu", "cumsum", "ceil", "power",
    "zeros_like", "ones_like", "allclose", "array_equal", "isfinite", "matmul",
    "transpose", "stack", "exp", "log",
):
    globals()[_name] = _passthrough(_name)


class _Linalg:
    @staticmethod
    def norm(x, ord=None, axis=None):
        return _wrap(_np.linalg.norm(_np.asarray(x), ord=ord, axis=axis))

    @staticmethod
    def cholesky(x, upper=False):
        out = _np.linalg.cholesky(_np.asarray(x))
        return _wrap(out.T if upper else out)

    @staticmethod
    def qr(x, mode="reduced"):
        return _wrap(_np.linalg.qr(_np.asarray(x), mode=mode))

    @staticmethod
    def eigh(x):
        return _wrap(_np.linalg.eigh(_np.asarray(x)))


linalg = _Linalg()
