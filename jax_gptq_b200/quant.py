"""RTN quantize/dequantize -- drop-in for ``src/jax_gptq/quant.py:6-37``.

Runs ``gq_rtn`` (CUDA).  float32 arithmetic; bf16/fp16 inputs are upcast
exactly to float32 first (the reference would compute in the input dtype).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _arrays as A
from . import _lib
from .config import QuantConfig


def _check(w, cfg: QuantConfig) -> None:
    """quant.py:7-10."""
    if len(tuple(w.shape)) != 2:
        raise ValueError(f"Expected 2D weight matrix, got shape={tuple(w.shape)}")
    if cfg.group_size <= 0 or (w.shape[1] % cfg.group_size) != 0:
        raise ValueError("group_size must be positive and divide in_features exactly")


@dataclass
class RTNResult:
    dequant: torch.Tensor   # [m, n] float32, original column order
    codes: torch.Tensor     # [m, n] uint8 (q - qmin), original column order
    scales: torch.Tensor    # [m, n // group_size] float32, permuted group order
    zeros: torch.Tensor     # [m, n // group_size] float32


def rtn(w, cfg: QuantConfig, perm=None, want_codes: bool = True) -> RTNResult:
    """Device-side RTN with optional column permutation (groups in permuted order)."""
    _check(w, cfg)
    wt = A.to_device(w)
    m, n = wt.shape
    g = cfg.group_size
    out = A.empty((m, n))
    codes = A.empty((m, n), torch.uint8) if want_codes else None
    scales = A.empty((m, n // g)) if want_codes else None
    zeros = A.empty((m, n // g)) if want_codes else None
    p = None if perm is None else A.to_device(perm, torch.int32)
    _lib.call("gq_rtn", A.ptr(wt), m, n, n, A.ptr(p), cfg.w_bits, g, int(cfg.sym), A.ptr(out),
              A.ptr(codes), A.ptr(scales), A.ptr(zeros), A.stream())
    return RTNResult(out, codes, scales, zeros)


def quantize_dequantize(w, cfg: QuantConfig):
    """quant.py:6 -- dequantized weights, same container as ``w``."""
    res = rtn(w, cfg, want_codes=False)
    return A.like_input(res.dequant, w)
