"""Blocked column-pivoted Householder QR -- drop-in for
``src/jax_gptq/pallas/blocked_pivoted_qr.py``.

The factorization runs in ``libgq`` (``csrc/gq_qr.cu``): per pivot step a
kernel on a cluster of eight CTAs (pivot, swap, reflector, compact-WY
append, the exposed-row weights) and an all-SM kernel that exposes one row
of the deferred trailing block and downdates the column norms, launched as
programmatic dependents; per panel two fp32 tensor-core GEMMs around a small
T application apply the compact WY update, and one kernel refreshes the
norms.

``semantics="reference"`` (default) reproduces the reference's default
(jit-compiled) path bit for bit in control flow, including two index slips:
the reflector of step j in a panel starting at k is built from column j - k
(``householder_vector_panel_local_dynamic``, :359-366), and the norm
downdate exposes panel-local row j (:1106-1112).  For more than one panel
the result is therefore not a QR factorization (every later panel's
diagonal is zero), exactly as in the reference.  ``semantics="intended"``
is a correct blocked QRCP whose pivots and R equal unblocked Householder
QR with column pivoting up to rounding; it additionally returns the
reflectors so ``A[:, perm] = Q R`` can be checked.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import _arrays as A
from .. import _lib

ZERO_TOL = 1e-12
ZERO_TOL_SQ = ZERO_TOL * ZERO_TOL

_MODES = {"largest": 0, "smallest": 1}
_NO_PIVOTING = 2  # gq_qrcp pivot_mode for plain Householder QR (not a reference mode)
_SEMANTICS = {"reference": 0, "intended": 1}


@dataclass(frozen=True)
class CompactPanel:
    """:56-72 -- ``Q_panel = I - Y T Y^T``; ``y`` in panel-local rows."""
    panel_start: int
    panel_end: int
    y: object
    tau: object
    t: object


@dataclass(frozen=True)
class FactorPanelResult:
    """:99-116."""
    a: object
    perm: object
    norms: object
    reflectors: list
    panel: CompactPanel


@dataclass
class QRResult:
    work: torch.Tensor          # [m, n]: R in the upper triangle, zeros below
    perm: torch.Tensor          # [n] int32
    v: torch.Tensor             # [m, min(m, n)] Householder vectors (unit diagonal)
    tau: torch.Tensor           # [min(m, n)]
    panel_ends: list = field(default_factory=list)


def _mode(pivot_mode: str) -> int:
    if pivot_mode not in _MODES:
        raise ValueError(f"unsupported pivot_mode={pivot_mode}")
    return _MODES[pivot_mode]


def qrcp(a, panel_size: int, pivot_mode: str = "largest", semantics: str = "reference",
         _unpivoted: bool = False) -> QRResult:
    """Full factorization on the device; returns work, perm, reflectors.
    ``_unpivoted`` runs plain Householder QR instead (``pivot_mode`` ignored)."""
    if len(tuple(a.shape)) != 2:
        raise ValueError(f"a must be 2D, got {tuple(a.shape)}")
    if panel_size <= 0:
        raise ValueError(f"panel_size must be positive, got {panel_size}")
    mode = _NO_PIVOTING if _unpivoted else _mode(pivot_mode)
    if semantics not in _SEMANTICS:
        raise ValueError(f"unsupported semantics={semantics}")
    work = A.to_device(a).clone()
    m, n = work.shape
    r = min(m, n)
    perm = A.empty((n,), torch.int32)
    v = A.empty((m, r))
    tau = A.empty((r,))
    max_panels = r + 1
    ends = torch.zeros((max_panels,), dtype=torch.int32)
    npan = ctypes.c_int(0)
    ws = A.workspace(_lib.lib().gq_qrcp_workspace_size(m, n, min(panel_size, r)))
    _lib.call("gq_qrcp", A.ptr(work), m, n, n, int(panel_size), mode, _SEMANTICS[semantics],
              A.ptr(perm), A.ptr(v), r, A.ptr(tau), ctypes.c_void_p(ends.data_ptr()),
              ctypes.byref(npan), A.ptr(ws), ws.numel(), A.stream())
    return QRResult(work, perm, v, tau, ends[: npan.value].tolist())


def householder_qr_r(a, panel_size: int = 64) -> torch.Tensor:
    """R of the reduced QR of ``a`` [m, n] (``mode="r"``: min(m, n) x n, upper
    triangular) by the library's own Householder QR without pivoting."""
    res = qrcp(a, panel_size, semantics="intended", _unpivoted=True)
    return torch.triu(res.work[: min(res.work.shape)]).contiguous()


def blocked_pivoted_qr(a, panel_size: int, pivot_mode: str = "largest",
                       semantics: str = "reference"):
    """:1627 -- returns ``(work, perm)`` in the container type of ``a``."""
    res = qrcp(a, panel_size, pivot_mode, semantics)
    return A.like_input(res.work, a), A.like_input(res.perm, a)


def init_trailing_norm_metadata(a):
    """:971-988 -- squared column norms."""
    t = A.to_device(a)
    return A.like_input((t * t).sum(dim=0), a)


def factor_panel_pallas(a, perm, norms, k: int, panel_size: int, pivot_mode: str,
                        semantics: str = "reference") -> FactorPanelResult:
    """:1412-1476 -- one panel from column ``k`` (kernel-shaped entry point)."""
    mode = _mode(pivot_mode)
    at = A.to_device(a).clone()
    m, n = at.shape
    if len(tuple(perm.shape)) != 1 or perm.shape[0] != n:
        raise ValueError(f"perm must be shape ({n},), got {tuple(perm.shape)}")
    if len(tuple(norms.shape)) != 1 or norms.shape[0] != n:
        raise ValueError(f"norms must be shape ({n},), got {tuple(norms.shape)}")
    if panel_size <= 0:
        raise ValueError(f"panel_size must be positive, got {panel_size}")
    limit = min(m, n)
    if not 0 <= k < limit:
        raise ValueError(f"k must be in [0, {limit}), got {k}")
    pt = A.to_device(perm, torch.int32).clone()
    nt = A.to_device(norms).clone()
    P = min(panel_size, limit - k)
    y = A.empty((m - k, P))
    tau = A.empty((P,))
    t = A.empty((P, P))
    pend = ctypes.c_int(0)
    ws = A.workspace(_lib.lib().gq_qrcp_workspace_size(m, n, P))
    _lib.call("gq_qr_factor_panel", A.ptr(at), m, n, n, A.ptr(pt), A.ptr(nt), int(k), int(panel_size),
              mode, _SEMANTICS[semantics], A.ptr(y), A.ptr(tau), A.ptr(t), ctypes.byref(pend),
              A.ptr(ws), ws.numel(), A.stream())
    panel = CompactPanel(k, int(pend.value), A.like_input(y, a), A.like_input(tau, a),
                         A.like_input(t, a))
    refl = []
    width = int(pend.value) - k
    for i in range(width):
        refl.append((k + i, A.like_input(y[i:, i], a), A.like_input(tau[i], a)))
    return FactorPanelResult(A.like_input(at, a), A.like_input(pt, a), A.like_input(nt, a), refl,
                             panel)


def _apply_panel_dev(block: torch.Tensor, y: torch.Tensor, t: torch.Tensor) -> None:
    rows, cols = block.shape
    width = y.shape[1]
    scratch = A.empty((max(1, 2 * width * cols),))
    _lib.call("gq_qr_apply_panel", A.ptr(block), rows, cols, block.stride(0), A.ptr(y),
              y.stride(0), A.ptr(t), t.stride(0), width, A.ptr(scratch), A.stream())


def apply_compact_panel_to_block(panel: CompactPanel, block):
    """:818-862 -- ``B - Y (T^T (Y^T B))`` on panel-local or full-row blocks."""
    bt = A.to_device(block).clone()
    y = A.to_device(panel.y).contiguous()
    t = A.to_device(panel.t).contiguous()
    if bt.ndim != 2:
        raise ValueError(f"block must be 2D, got {tuple(bt.shape)}")
    if bt.shape[0] == y.shape[0]:
        tail = bt
    elif bt.shape[0] == panel.panel_start + y.shape[0]:
        tail = bt[panel.panel_start:]
    else:
        raise ValueError(
            f"block row dimension must match panel-local or full rows, got {bt.shape[0]}")
    tail_c = tail.contiguous()
    _apply_panel_dev(tail_c, y, t)
    tail.copy_(tail_c)
    return A.like_input(bt, block)


apply_compact_panel_to_block_pallas = apply_compact_panel_to_block


def apply_reflector_to_block(v, tau, block):
    """:369-396 -- ``B - v (tau v^T B)`` (a one-reflector compact panel)."""
    vt = A.to_device(v)
    bt = A.to_device(block).clone()
    if vt.ndim != 1:
        raise ValueError(f"v must be 1D, got {tuple(vt.shape)}")
    if bt.ndim != 2:
        raise ValueError(f"block must be 2D, got {tuple(bt.shape)}")
    if bt.shape[0] != vt.shape[0]:
        raise ValueError(
            f"block row dimension must match v length, got {bt.shape[0]} and {vt.shape[0]}")
    tt = A.to_device(tau).reshape(1, 1).contiguous()
    _apply_panel_dev(bt, vt.reshape(-1, 1).contiguous(), tt)
    return A.like_input(bt, block)


apply_reflector_to_block_pallas = apply_reflector_to_block


def apply_panel_to_trailing_pallas(a, panel: CompactPanel, panel_end: int):
    """:1592-1624 -- deferred update of ``a[panel_start:, panel_end:]``."""
    at = A.to_device(a).clone()
    if panel_end >= at.shape[1]:
        return A.like_input(at, a)
    y = A.to_device(panel.y).contiguous()
    t = A.to_device(panel.t).contiguous()
    blk = at[panel.panel_start:, panel_end:].contiguous()
    _apply_panel_dev(blk, y, t)
    at[panel.panel_start:, panel_end:] = blk
    return A.like_input(at, a)


apply_panel_to_trailing = apply_panel_to_trailing_pallas


def compute_exposed_trailing_row_from_compact_panel(panel: CompactPanel, trailing_block,
                                                    row_index: int):
    """:905-946 -- ``B[r] - (y_r T^T Y^T) B`` via three device GEMMs."""
    tb = A.to_device(trailing_block)
    y = A.to_device(panel.y).contiguous()
    t = A.to_device(panel.t).contiguous()
    if tb.shape[0] == y.shape[0]:
        local, tail = row_index, tb
    elif tb.shape[0] == panel.panel_start + y.shape[0]:
        local, tail = row_index - panel.panel_start, tb[panel.panel_start:]
    else:
        raise ValueError(
            "trailing_block row dimension must match panel-local or full rows, "
            f"got {tb.shape[0]}")
    local = max(0, min(int(local), y.shape[0] - 1))
    tail = tail.contiguous()
    L, w = y.shape
    cols = tail.shape[1]
    rw = A.empty((1, w))
    left = A.empty((1, L))
    out = tail[local:local + 1].clone()
    yr = y[local:local + 1].contiguous()
    _lib.call("gq_sgemm", 0, 1, 1, w, w, 1.0, A.ptr(yr), w, A.ptr(t), w, 0.0, A.ptr(rw), w, 0,
              A.stream())
    _lib.call("gq_sgemm", 0, 1, 1, L, w, 1.0, A.ptr(rw), w, A.ptr(y), w, 0.0, A.ptr(left), L, 0,
              A.stream())
    _lib.call("gq_sgemm", 0, 0, 1, cols, L, -1.0, A.ptr(left), L, A.ptr(tail), cols, 1.0,
              A.ptr(out), cols, 0, A.stream())
    return A.like_input(out[0], trailing_block)


def build_compact_panel(reflectors, panel_start: int, panel_end: int, n_rows: int) -> CompactPanel:
    """:545-599 -- pack reflectors into Y and build T column by column.

    Mirrors the reference exactly, including that column 1 of T is
    ``-tau_1 Y_0^T y_1`` without the ``T[0, 0]`` factor (the multiply by the
    leading block of T is only applied from column 2 on, :590-595).
    """
    if not 0 <= panel_start <= panel_end <= n_rows:
        raise ValueError(
            f"expected 0 <= panel_start <= panel_end <= n_rows, got "
            f"{panel_start}, {panel_end}, {n_rows}")
    width = panel_end - panel_start
    y = torch.zeros((n_rows - panel_start, width), dtype=torch.float32, device="cuda")
    tau = torch.zeros((width,), dtype=torch.float32, device="cuda")
    host = None
    for idx, (j, v, tau_j) in enumerate(reflectors):
        if not panel_start <= j < panel_end:
            raise ValueError(f"reflector row index {j} is outside panel [{panel_start}, {panel_end})")
        y[j - panel_start:, idx] = A.to_device(v)
        tau[idx] = A.to_device(tau_j).reshape(())
        host = v
    t = torch.zeros((width, width), dtype=torch.float32, device="cuda")
    yc = y.t().contiguous()  # width x L: reflector i in row i
    L = y.shape[0]
    for i in range(width):
        t[i, i] = tau[i]
        if i == 0:
            continue
        w = A.empty((1, i))
        _lib.call("gq_sgemm", 0, 1, 1, i, L, 1.0, A.ptr(yc[i:i + 1]), L, A.ptr(yc), L, 0.0,
                  A.ptr(w), i, 0, A.stream())
        w = -tau[i] * w
        if i > 1:
            w2 = A.empty((1, i))
            tl = t[:i, :i].contiguous()
            _lib.call("gq_sgemm", 0, 1, 1, i, i, 1.0, A.ptr(w.contiguous()), i, A.ptr(tl), i, 0.0,
                      A.ptr(w2), i, 0, A.stream())
            w = w2
        t[:i, i] = w[0]
    ref = host if host is not None else np.zeros(0, np.float32)
    return CompactPanel(panel_start, panel_end, A.like_input(y, ref), A.like_input(tau, ref),
                        A.like_input(t, ref))


def benchmark_matrix(n: int = 4096, seed: int = 1, rank_deficient: bool = False,
                     n_dependent: int = 256) -> np.ndarray:
    """The benchmark matrix ``A = G diag(s)``, ``G ~ N(0, 1)``, ``s_k =
    10^(-6k/n)`` in a shuffled column order; the rank-deficient variant
    replaces ``n_dependent`` columns by random combinations of the others
    (numpy PCG64, the same bytes as the test fixture's generator)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    g = rng.standard_normal((n, n)).astype(np.float32)
    s = (10.0 ** (-6.0 * np.arange(n) / n)).astype(np.float32)
    s = s[rng.permutation(n)]
    a = (g * s[None, :]).astype(np.float32)
    if rank_deficient:
        dep = rng.choice(n, size=min(n_dependent, n // 2), replace=False)
        indep = np.setdiff1d(np.arange(n), dep)
        coef = rng.standard_normal((indep.shape[0], dep.shape[0])).astype(np.float32)
        coef /= np.sqrt(np.float32(indep.shape[0]))
        a[:, dep] = (a[:, indep] @ coef).astype(np.float32)
    return a


def benchmark(n: int = 4096, panel: int = 64, reps: int = 2, seed: int = 1,
              variants: str | None = None) -> dict:
    """Time the 4096 x 4096 fp32 benchmark matrix (:func:`benchmark_matrix`)
    in both semantics, and the rank-deficient variant in ``smallest`` mode
    (the pivot order the reference's rank-deficient QRCP case uses) and
    ``largest`` mode (rank revealing: its numerical rank is the 3840 of the
    construction).  GFLOP/s counts (4/3) n^3."""
    a = torch.from_numpy(benchmark_matrix(n, seed)).cuda()
    a_def = torch.from_numpy(benchmark_matrix(n, seed, rank_deficient=True)).cuda()
    flops = 4.0 / 3.0 * n ** 3
    out = {"n": n, "panel": panel, "flop_count": "(4/3) n^3"}
    for label, mat, mode, sem in [("intended_largest", a, "largest", "intended"),
                                  ("reference_largest", a, "largest", "reference"),
                                  ("intended_rankdef_smallest", a_def, "smallest", "intended"),
                                  ("intended_rankdef_largest", a_def, "largest", "intended")]:
        if variants and label not in variants.split(","):
            continue
        qrcp(mat, panel, mode, sem)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            res = qrcp(mat, panel, mode, sem)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        entry = {"ms": ms, "gflops": flops / (ms / 1e3) / 1e9, "panels": len(res.panel_ends)}
        if sem == "intended":
            q_err = _residual_dev(mat, res)
            entry["residual"] = q_err
            entry.update(numerical_rank(res.work))
            # smallest-norm-first pivoting moves dependent columns to the
            # front while their residual norms are still large, so R's
            # diagonal does not reveal the rank in that mode
            entry["rank_revealing"] = mode == "largest"
        out[label] = entry
    return out


# Relative to max |R_jj|: about two float32 epsilons.  The factorization's own
# rounding noise bounds what the diagonal can resolve: on the rank-deficient
# 4096 benchmark matrix its 256 dependent columns end at |R_jj| / max up to
# 1.1e-7 (3xTF32 trailing updates), while the smallest independent one is
# 2.3e-7.
RANK_RCOND = 2e-7


def numerical_rank(work: torch.Tensor, rcond: float = RANK_RCOND) -> dict:
    """Numerical rank from the diagonal of R: the number of ``|R_jj|`` above
    ``rcond * max_j |R_jj|`` (the largest, not the first: in ``smallest`` mode
    the first pivot is the smallest column), plus the position of the largest
    drop between consecutive ``|R_jj|`` of the sorted diagonal."""
    d = work.diagonal().abs().double()
    top = float(d.max().item()) if d.numel() else 0.0
    rank = int((d > rcond * top).sum().item()) if top > 0 else 0
    ds = torch.sort(d, descending=True).values
    gap_at, gap = 0, 1.0
    if ds.numel() > 1:
        ratios = ds[:-1] / torch.clamp(ds[1:], min=1e-300)
        j = int(torch.argmax(ratios).item())
        gap_at, gap = j + 1, float(ratios[j].item())
    return {"numerical_rank": rank, "rank_rcond": rcond, "largest_gap_at": gap_at,
            "largest_gap_ratio": gap}


def _residual_dev(a: torch.Tensor, res: QRResult) -> float:
    """``||A[:, perm] - Q R||_F / ||A||_F`` in float64 on the device."""
    a64 = a.double()
    x = torch.triu(res.work.double())
    v = res.v.double()
    tau = res.tau.double()
    # Q R = H_1 ... H_r R, applied right to left
    for i in reversed(range(v.shape[1])):
        vi = v[:, i:i + 1]
        x = x - vi @ (tau[i] * (vi.T @ x))
    pa = a64[:, res.perm.long()]
    return float(torch.linalg.norm(pa - x) / torch.linalg.norm(a64))
