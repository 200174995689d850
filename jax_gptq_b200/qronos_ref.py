"""Qronos single-layer update -- drop-in for ``src/jax_gptq/qronos_ref.py:7-25``.

``semantics="reference"`` returns RTN of ``weight_orig`` after the
reference's shape checks (qronos_ref.py:18-25).

``semantics="intended"`` runs Qronos (Zhang, Zhang & Saab 2025) with
``h = Xt^T Xt`` and ``g = X^T Xt`` as ``h_g_from_activations(x_quant=Xt,
x_float=X)`` produces them:

1. "correct the past" for the first column: ``v1 = ((g^T w_orig)_1 -
   h_{1,>1} w_{>1}) / h_11`` and ``q1 = Q(v1)`` (group-0 parameters from the
   starting weights);
2. "shape the future": ``w_{>1} = h_{>1,>1}^-1 ((g^T w_orig)_{>1} - h_{>1,1}
   q1)``, evaluated as ``b U2^T U2`` with ``U2 = U[1:, 1:]`` (the inverse
   Cholesky factor of the trailing block is the trailing block of ``U``);
3. the remaining columns follow the GPTQ error-feedback sweep, which is what
   both Qronos rules reduce to once the future is the least-squares optimum.

``h`` is damped like GPTQ's Hessian.  All of it runs on the device
(``gq_qronos``).
"""

from __future__ import annotations

import torch

from . import _arrays as A
from . import _lib
from .config import QuantConfig
from .gptq_ref import SWEEP_BLOCK, SweepResult, factor_hessian
from .quant import quantize_dequantize


def _check(weight, weight_orig, h, g) -> None:
    """qronos_ref.py:18-23."""
    if len(tuple(weight.shape)) != 2 or len(tuple(weight_orig.shape)) != 2:
        raise ValueError("weight and weight_orig must be 2D")
    if tuple(weight.shape) != tuple(weight_orig.shape):
        raise ValueError("weight and weight_orig shape mismatch")
    if h.shape[0] != h.shape[1] or tuple(g.shape) != tuple(h.shape):
        raise ValueError("h must be square and g must match h shape")


def qronos_quantize(weight, weight_orig, h, g, cfg: QuantConfig, factor=None) -> SweepResult:
    """Intended-semantics Qronos on the device; returns codes, scales, zeros, ..."""
    w = A.to_device(weight)
    wo = A.to_device(weight_orig)
    gd = A.to_device(g)
    m, n = w.shape
    if factor is None or factor.hd is None:
        factor = factor_hessian(h, cfg, want_hd=True)
    gs = cfg.group_size
    out = A.empty((m, n))
    codes = A.empty((m, n), torch.uint8)
    scales = A.empty((m, n // gs))
    zeros = A.empty((m, n // gs))
    g_idx = A.empty((n,), torch.int32)
    ws = A.workspace(_lib.lib().gq_qronos_workspace_size(m, n))
    _lib.call("gq_qronos", A.ptr(w), A.ptr(wo), m, n, A.ptr(factor.hd), A.ptr(factor.u),
              A.ptr(gd), A.ptr(factor.perm), cfg.w_bits, gs, int(cfg.sym), SWEEP_BLOCK,
              A.ptr(out), A.ptr(codes), A.ptr(scales), A.ptr(zeros), A.ptr(g_idx), A.ptr(ws),
              ws.numel(), A.stream())
    return SweepResult(out, codes, scales, zeros, g_idx, factor.perm)


def qronos_single_layer_update_ref(weight, weight_orig, h, g, cfg: QuantConfig):
    """qronos_ref.py:7 -- dequantized weights in the container type of ``weight_orig``."""
    _check(weight, weight_orig, h, g)
    if cfg.semantics == "reference":
        return quantize_dequantize(weight_orig, cfg)
    res = qronos_quantize(weight, weight_orig, h, g, cfg)
    return A.like_input(res.dequant, weight_orig)
