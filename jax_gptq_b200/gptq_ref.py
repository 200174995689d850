"""Hessian processing and the GPTQ step -- drop-in for ``src/jax_gptq/gptq_ref.py``.

``semantics="reference"`` (default) returns what the reference returns:
``process_hessian`` -> ``(eye(n), perm)`` (its Cholesky branch always falls
back, gptq_ref.py:85-92) and ``gptq_forward_step`` -> RTN of the permuted
weights, ignoring ``h_inv_sqrt`` (gptq_ref.py:150-155).

``semantics="intended"`` runs the algorithm: ``process_hessian`` factors the
damped, permuted Hessian on the GPU (``gq_hessian_factor``, with the 10x
damping retries of gptq_ref.py:80-83 driven by a device-side
positive-definiteness flag) and ``gptq_forward_step`` runs the GPTQ column
sweep honouring ``h_inv_sqrt`` (``gq_gptq_sweep``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _arrays as A
from . import _lib
from .config import QuantConfig
from .quant import rtn

SWEEP_BLOCK = 128


def _select_truncation_rank(eigvals_desc, cfg: QuantConfig) -> int:
    """gptq_ref.py:8-41 (host arithmetic on a small vector)."""
    ev = np.asarray(eigvals_desc.detach().cpu() if isinstance(eigvals_desc, torch.Tensor)
                    else eigvals_desc, dtype=np.float64)
    if ev.ndim != 1:
        raise ValueError(f"eigvals_desc must be 1D, got {ev.shape}")
    n = ev.shape[0]
    if n == 0:
        raise ValueError("eigvals_desc must be non-empty")
    mode, value = cfg.truncation_mode, float(cfg.truncation_value)
    if mode == "abs":
        rank = int(np.sum(ev > value))
    elif mode == "percent":
        rank = int(np.ceil((1.0 - min(max(value / 100.0, 0.0), 1.0)) * n))
    elif mode == "mean_top32":
        rank = int(np.sum(ev > value * np.mean(ev[: min(32, n)])))
    elif mode == "energy":
        rank = int(np.sum(np.cumsum(ev) <= (1.0 - value) * np.sum(ev)))
        if rank < n:
            rank += 1
    else:
        raise ValueError(f"unsupported truncation_mode={mode}")
    return max(1, min(rank, n))


def _check_hessian(h, cfg: QuantConfig) -> None:
    """gptq_ref.py:56-57, 62-65, 95-96."""
    shape = tuple(h.shape)
    if len(shape) != 2 or shape[0] != shape[1]:
        raise ValueError(f"h must be square 2D, got {shape}")
    if cfg.solver_mode == "chol":
        if cfg.ordering_mode not in {"none", "diag_h"}:
            raise ValueError(
                f"ordering_mode={cfg.ordering_mode} is not supported for solver_mode='chol'")
    elif cfg.solver_mode == "eigh":
        if cfg.ordering_mode not in {"none", "diag_h", "pivot_sqrt_h", "pivot_sqrt_hinv_smallest"}:
            raise ValueError(f"unsupported ordering_mode={cfg.ordering_mode}")
    else:
        raise ValueError(f"unsupported solver_mode={cfg.solver_mode}")


def act_order_perm(h_dev: torch.Tensor, ordering_mode: str) -> torch.Tensor:
    """gptq_ref.py:67-70 on the device."""
    d = h_dev.shape[0]
    perm = A.empty((d,), torch.int32)
    _lib.call("gq_act_order_perm", A.ptr(h_dev), d, d, 1 if ordering_mode == "diag_h" else 0,
              A.ptr(perm), A.stream())
    return perm


@dataclass
class HessianFactor:
    u: torch.Tensor            # [d, d] upper, u^T u = (H_perm + damp I)^-1
    perm: torch.Tensor         # [d] int32
    attempt: int               # damping exponent used
    hd: torch.Tensor | None    # damped, permuted Hessian (when requested)


def factor_hessian(h, cfg: QuantConfig, want_hd: bool = False) -> HessianFactor:
    """The working damped-Cholesky branch of gptq_ref.py:61-92 (device)."""
    _check_hessian(h, cfg)
    hd_dev = A.to_device(h)
    d = hd_dev.shape[0]
    perm = act_order_perm(hd_dev, cfg.ordering_mode)
    u = A.empty((d, d))
    hd = A.empty((d, d)) if want_hd else None
    ws = A.workspace(_lib.lib().gq_hessian_factor_workspace_size(d))
    attempt = _lib.ctypes.c_int(-1)
    status = _lib.lib().gq_hessian_factor(A.ptr(hd_dev), d, d, A.ptr(perm), float(cfg.damp_percent),
                                          A.ptr(u), d, A.ptr(hd), A.ptr(ws), ws.numel(),
                                          _lib.ctypes.byref(attempt), A.stream())
    if status == _lib.GQ_ENOTPD:
        # gptq_ref.py:91-92: fall back to the identity after five failed attempts
        u = torch.eye(d, dtype=torch.float32, device="cuda")
        return HessianFactor(u, perm, -1, hd)
    if status != _lib.GQ_OK:
        raise _lib.GQError(status, _lib.lib().gq_last_error().decode())
    return HessianFactor(u, perm, attempt.value, hd)


def factor_hessian_attempt0(h_dev: torch.Tensor, cfg: QuantConfig, want_hd: bool = False):
    """The first damping attempt of :func:`factor_hessian`, enqueued on the
    current stream with no host synchronization (``gq_hessian_factor_attempt``).

    Returns ``(factor, status)``: ``status`` is a 1-element int32 device tensor,
    0 when the factor is valid.  A caller that sees a non-zero status redoes
    the group with :func:`factor_hessian` (the later attempts and the identity
    fallback)."""
    _check_hessian(h_dev, cfg)
    d = h_dev.shape[0]
    perm = act_order_perm(h_dev, cfg.ordering_mode)
    u = A.empty((d, d))
    hd = A.empty((d, d)) if want_hd else None
    ws = A.workspace(_lib.lib().gq_hessian_factor_workspace_size(d))
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    _lib.call("gq_hessian_factor_attempt", A.ptr(h_dev), d, d, A.ptr(perm),
              float(cfg.damp_percent), 0, A.ptr(u), d, A.ptr(hd), A.ptr(ws), ws.numel(),
              A.ptr(status), A.stream())
    return HessianFactor(u, perm, 0, hd), status


def factor_from_activations_attempt0(x: torch.Tensor, cfg: QuantConfig,
                                     chain_stream: torch.cuda.Stream, reserve_sms: int):
    """Attempt 0 of :func:`factor_hessian` for ``h = x^T x`` formed from the
    bf16 activations ``x`` (``gq_factor_from_x_attempt``): the statistics run
    on the current stream, the factor on ``chain_stream``, whose first half
    starts while the rest of ``h`` is still accumulating.  Same factor, bit
    for bit, as ``factor_hessian_attempt0(x^T x)``.

    Returns ``(factor, status)`` like :func:`factor_hessian_attempt0`; the
    result tensors belong to ``chain_stream``."""
    if cfg.solver_mode != "chol" or cfg.ordering_mode not in {"none", "diag_h"}:
        raise ValueError("factor_from_activations_attempt0 supports solver_mode='chol' with "
                         "ordering_mode 'none' or 'diag_h'")
    tokens, d = x.shape
    main = torch.cuda.current_stream()
    lib = _lib.lib()
    ws = A.workspace(lib.gq_factor_from_x_workspace_size(tokens, d))
    with torch.cuda.stream(chain_stream):
        u = A.empty((d, d))
        perm = A.empty((d,), torch.int32)
        status = torch.empty((1,), dtype=torch.int32, device="cuda")
    # perm and status are written on the statistics stream first
    perm.record_stream(main)
    status.record_stream(main)
    ws.record_stream(chain_stream)
    _lib.call("gq_factor_from_x_attempt", A.ptr(x), tokens, d, x.stride(0),
              1 if cfg.ordering_mode == "diag_h" else 0, float(cfg.damp_percent), int(reserve_sms),
              A.ptr(u), d, A.ptr(perm), A.ptr(ws), ws.numel(), A.ptr(status),
              main.cuda_stream, chain_stream.cuda_stream)
    return HessianFactor(u, perm, 0, None), status


EIGH_MAX_SWEEPS = 30


def eigh(h) -> tuple[torch.Tensor, torch.Tensor]:
    """``jnp.linalg.eigh`` (gptq_ref.py:98) on the device with the library's
    Jacobi eigensolver (``gq_syevj``): eigenvalues ascending, eigenvectors as
    columns, ``h = v diag(w) v^T``."""
    hd = A.to_device(h)
    n = hd.shape[0]
    w = A.empty((n,))
    v = A.empty((n, n))
    ws = A.workspace(_lib.lib().gq_syevj_workspace_size(n))
    import ctypes
    sweeps = ctypes.c_int(0)
    _lib.call("gq_syevj", A.ptr(hd), n, hd.stride(0), A.ptr(w), A.ptr(v), n, EIGH_MAX_SWEEPS,
              ctypes.byref(sweeps), A.ptr(ws), ws.numel(), A.stream())
    return w, v


def _process_hessian_eigh(h, cfg: QuantConfig, panel_size: int):
    """gptq_ref.py:95-133 on the device.

    Every step runs on this library's kernels: the eigendecomposition by
    parallel Jacobi (:func:`eigh`, ``gq_syevj``), the unpivoted reduced QR by
    the Householder QR without pivoting (``gq_qrcp`` mode 2), the act-order
    ranking and the blocked pivoted QR of the pivot_* modes.
    ``sqrt_h = sqrt(lam) V^T`` and ``sqrt_hinv = lam^-1/2 V^T`` over the kept
    eigenpairs (descending, rank from the truncation rule).  For none / diag_h
    / pivot_sqrt_h the factor is R of ``sqrt_hinv.T[:, perm]``: in reference
    semantics the permutation indexes the eigen axis and, for rank < n, the
    gather past the kept columns is clamped to the last one (JAX's rule for
    out-of-range gathers), which leaves R diagonal in exact arithmetic; in
    intended semantics it acts on the feature axis, ``sqrt_hinv[:, perm]``,
    so ``R^T R`` is the permuted pseudo-inverse.  pivot_sqrt_hinv_smallest
    returns the pivoted QR of ``sqrt_hinv`` itself (rank x n)."""
    import importlib
    BQ = importlib.import_module("jax_gptq_b200.pallas.blocked_pivoted_qr")
    hd = A.to_device(h)
    n = hd.shape[0]
    evals, evecs = eigh(hd)
    evals, evecs = evals.flip(0), evecs.flip(1)
    rank = _select_truncation_rank(evals, cfg)
    lam, v = evals[:rank], evecs[:, :rank]
    sqrt_h = (torch.sqrt(lam)[:, None] * v.T).contiguous()
    sqrt_hinv = (torch.pow(lam, -0.5)[:, None] * v.T).contiguous()
    if cfg.ordering_mode == "pivot_sqrt_hinv_smallest":
        res = BQ.qrcp(sqrt_hinv, panel_size, "smallest", cfg.semantics)
        return res.work, res.perm
    if cfg.ordering_mode == "none":
        perm = torch.arange(n, dtype=torch.int32, device="cuda")
    elif cfg.ordering_mode == "diag_h":
        perm = act_order_perm(hd, "diag_h")
    else:
        perm = BQ.qrcp(sqrt_h, panel_size, "largest", cfg.semantics).perm
    idx = perm.long()
    if cfg.semantics == "reference":
        m = sqrt_hinv.T[:, idx.clamp(max=rank - 1)]
    else:
        m = sqrt_hinv[:, idx]
    r = BQ.householder_qr_r(m.contiguous())
    return r, perm


def process_hessian(h, cfg: QuantConfig, panel_size: int = 32):
    """gptq_ref.py:44 -- returns ``(h_inv_sqrt, perm)``."""
    _check_hessian(h, cfg)
    if cfg.solver_mode == "eigh":
        r, perm = _process_hessian_eigh(h, cfg, panel_size)
        return A.like_input(r, h), A.like_input(perm, h)
    if cfg.semantics == "reference":
        hd = A.to_device(h)
        perm = act_order_perm(hd, cfg.ordering_mode)
        eye = torch.eye(hd.shape[0], dtype=torch.float32, device="cuda")
        return A.like_input(eye, h), A.like_input(perm, h)
    f = factor_hessian(h, cfg)
    return A.like_input(f.u, h), A.like_input(f.perm, h)


@dataclass
class SweepResult:
    dequant: torch.Tensor   # [m, n] float32, original column order
    codes: torch.Tensor     # [m, n] uint8 = q - qmin, original column order
    scales: torch.Tensor    # [m, n // g] float32, permuted group order
    zeros: torch.Tensor     # [m, n // g]
    g_idx: torch.Tensor     # [n] int32 group of each original column
    perm: torch.Tensor      # [n] int32


def gptq_sweep(weight, u, perm, cfg: QuantConfig, start=None, group0=None,
               noprop_cols: int = 0) -> SweepResult:
    """GPTQ column sweep on the device (``gq_gptq_sweep``)."""
    w = A.to_device(weight)
    m, n = w.shape
    ud = A.to_device(u)
    pd = A.to_device(perm, torch.int32)
    g = cfg.group_size
    out = A.empty((m, n))
    codes = A.empty((m, n), torch.uint8)
    scales = A.empty((m, n // g))
    zeros = A.empty((m, n // g))
    g_idx = A.empty((n,), torch.int32)
    ws = A.workspace(_lib.lib().gq_gptq_sweep_workspace_size(m, n))
    st = None if start is None else A.to_device(start)
    g0s = g0z = None
    if group0 is not None:
        g0s, g0z = A.to_device(group0[0]), A.to_device(group0[1])
    _lib.call("gq_gptq_sweep", A.ptr(w), m, n, n, A.ptr(st), A.ptr(ud), n, A.ptr(pd), cfg.w_bits, g,
              int(cfg.sym), SWEEP_BLOCK, A.ptr(g0s), A.ptr(g0z), int(noprop_cols), A.ptr(out),
              A.ptr(codes), A.ptr(scales), A.ptr(zeros), A.ptr(g_idx), A.ptr(ws), ws.numel(),
              A.stream())
    return SweepResult(out, codes, scales, zeros, g_idx, pd)


def _check_step(weight, perm) -> None:
    """gptq_ref.py:146-149."""
    if len(tuple(weight.shape)) != 2:
        raise ValueError(f"weight must be 2D, got {tuple(weight.shape)}")
    if len(tuple(perm.shape)) != 1 or perm.shape[0] != weight.shape[1]:
        raise ValueError(f"perm must be shape ({weight.shape[1]},), got {tuple(perm.shape)}")


def gptq_forward_step(weight, h_inv_sqrt, perm, cfg: QuantConfig):
    """gptq_ref.py:136 -- dequantized weights in original column order."""
    _check_step(weight, perm)
    if cfg.semantics == "reference":
        res = rtn(weight, cfg, perm=perm, want_codes=False)
        return A.like_input(res.dequant, weight)
    res = gptq_sweep(weight, h_inv_sqrt, perm, cfg)
    return A.like_input(res.dequant, weight)


def gptq_quantize(weight, h, cfg: QuantConfig, factor: HessianFactor | None = None) -> SweepResult:
    """Whole GPTQ for one linear: perm, damped factor, sweep (intended semantics).

    ``factor`` lets linears that share an input (q/k/v, gate/up) reuse one
    factorization.
    """
    if factor is None:
        factor = factor_hessian(h, cfg)
    return gptq_sweep(weight, factor.u, factor.perm, cfg)
