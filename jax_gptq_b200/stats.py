"""Hessian / cross-covariance accumulation -- drop-in for ``src/jax_gptq/stats.py:4-18``.

``h = x_quant^T x_quant`` and ``g = x_float^T x_quant`` for activations laid
out ``[tokens, in_features]``.  bf16 activations run on the tcgen05 tensor
cores (``gq_syrk_bf16`` / ``gq_gemm_tn_bf16``, fp32 accumulation in TMEM);
float32 activations run the fp32 CUDA-core GEMM.  Results are float32 (the
reference returns the input dtype; a bf16 Hessian would be useless for the
Cholesky that follows).

Differences from the reference, both deliberate: ``g`` is not recomputed
when ``x_float`` is None (the reference does the same product twice,
stats.py:10-11) -- the returned ``g`` is the same array as ``h``; and the
streaming ``HessianAccumulator`` adds batches into one buffer.
"""

from __future__ import annotations

import torch

from . import _arrays as A
from . import _lib


def _check(x_quant, x_float) -> None:
    """stats.py:8-13."""
    if len(tuple(x_quant.shape)) != 2:
        raise ValueError(f"x_quant must be 2D [tokens, in_features], got {tuple(x_quant.shape)}")
    if x_float is not None and tuple(x_float.shape) != tuple(x_quant.shape):
        raise ValueError(
            f"x_float shape must match x_quant, got {tuple(x_float.shape)} vs {tuple(x_quant.shape)}")


def _is_bf16(x) -> bool:
    return isinstance(x, torch.Tensor) and x.dtype == torch.bfloat16


# bf16 products are summed in tensor-memory chunks of this many tokens; calls
# split at multiples of it give the same bits as one call (see gq.h)
TOKEN_CHUNK_QUANTUM = 1024


def _token_slices(tokens: int, token_chunk):
    if not token_chunk or token_chunk >= tokens:
        return [(0, tokens)]
    if token_chunk % TOKEN_CHUNK_QUANTUM:
        raise ValueError(f"token_chunk must be a multiple of {TOKEN_CHUNK_QUANTUM}, got {token_chunk}")
    return [(t0, min(tokens, t0 + token_chunk)) for t0 in range(0, tokens, token_chunk)]


def syrk_into(h: torch.Tensor, x: torch.Tensor, accumulate: bool, token_chunk=None) -> None:
    """h (+)= x^T x on the device (h: [d, d] float32 contiguous).

    ``token_chunk`` splits the product into launches over that many tokens
    each (shorter kernels, so work on higher-priority streams is scheduled in
    between); for bf16 the result is bit-identical to a single launch."""
    d = x.shape[1]
    for i, (t0, t1) in enumerate(_token_slices(x.shape[0], token_chunk)):
        xs = x[t0:t1]
        acc = int(accumulate or i > 0)
        if x.dtype == torch.bfloat16:
            _lib.call("gq_syrk_bf16", A.ptr(xs), t1 - t0, d, x.stride(0), A.ptr(h), d, acc,
                      A.stream())
        else:
            _lib.call("gq_syrk_f32", A.ptr(xs), t1 - t0, d, x.stride(0), A.ptr(h), d, acc,
                      A.stream())


def gemm_tn_into(g: torch.Tensor, xa: torch.Tensor, xb: torch.Tensor, accumulate: bool,
                 token_chunk=None) -> None:
    """g (+)= xa^T xb on the device; ``token_chunk`` as for :func:`syrk_into`."""
    da = xa.shape[1]
    db = xb.shape[1]
    for i, (t0, t1) in enumerate(_token_slices(xa.shape[0], token_chunk)):
        sa, sb = xa[t0:t1], xb[t0:t1]
        acc = int(accumulate or i > 0)
        if xa.dtype == torch.bfloat16:
            _lib.call("gq_gemm_tn_bf16", A.ptr(sa), xa.stride(0), A.ptr(sb), xb.stride(0), t1 - t0,
                      da, db, A.ptr(g), db, acc, A.stream())
        else:
            _lib.call("gq_gemm_tn_f32", A.ptr(sa), xa.stride(0), A.ptr(sb), xb.stride(0), t1 - t0,
                      da, db, A.ptr(g), db, acc, A.stream())


def h_g_from_activations(x_quant, x_float=None):
    """stats.py:4 -- returns ``(h, g)`` in the container type of ``x_quant``."""
    _check(x_quant, x_float)
    dt = torch.bfloat16 if _is_bf16(x_quant) else torch.float32
    xq = A.to_device(x_quant, dt)
    d = xq.shape[1]
    h = A.empty((d, d))
    syrk_into(h, xq, accumulate=False)
    if x_float is None:
        g = h
    else:
        xf = A.to_device(x_float, dt)
        g = A.empty((d, d))
        gemm_tn_into(g, xf, xq, accumulate=False)
    h_out = A.like_input(h, x_quant)
    if g is h:
        return h_out, h_out
    return h_out, A.like_input(g, x_quant)


class HessianAccumulator:
    """Streamed ``H (+)= X_b^T X_b`` (and ``G (+)= Xf_b^T Xq_b``) over batches."""

    def __init__(self, d: int, with_cross: bool = False):
        A.require_cuda()
        self.d = d
        self.h = torch.zeros((d, d), dtype=torch.float32, device="cuda")
        self.g = torch.zeros((d, d), dtype=torch.float32, device="cuda") if with_cross else None
        self.tokens = 0

    def add(self, x_quant, x_float=None) -> None:
        _check(x_quant, x_float)
        dt = torch.bfloat16 if _is_bf16(x_quant) else torch.float32
        xq = A.to_device(x_quant, dt)
        syrk_into(self.h, xq, accumulate=True)
        if self.g is not None:
            xf = xq if x_float is None else A.to_device(x_float, dt)
            gemm_tn_into(self.g, xf, xq, accumulate=True)
        self.tokens += xq.shape[0]
