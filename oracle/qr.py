"""Blocked column-pivoted Householder QR -- restates
``src/jax_gptq/pallas/blocked_pivoted_qr.py`` (compiled-path semantics).

Test infrastructure (see ``oracle/__init__.py``).  Everything is float32 and
follows the reference's op order:

* driver ``blocked_pivoted_qr`` (:1627-1722): ``perm = arange``, squared
  column norms (:971-988); per panel of ``panel_size`` columns: factor the
  panel, apply the deferred compact-WY update to ``a[k:, panel_end:]``
  (:1592-1624, :818-862), recompute the norms from rows ``>= panel_end``
  (:991-1011);
* panel factorization ``_factor_panel_compiled`` (:1479-1589): per step j,
  ``smallest`` early stop when no norm ``> ZERO_TOL**2`` (:1562-1570); pivot
  = first argmax / argmin (:202-219) over *all* columns ``>= j`` -- including
  deferred (stale) trailing columns; full-column swap (:264-283); Householder
  vector from rows ``>= j`` (:327-356, ``alpha = +|x|`` when ``x0 <= 0``);
  incremental T column (:674-726); reflector applied to the panel columns
  ``>= j`` and the pivot column overwritten with ``alpha`` / zeros
  (:786-815); norm metadata: panel columns downdated by the new row and
  recomputed exactly every 8 completed steps (:1014-1104), trailing columns
  downdated by the exposed row ``B[r] - (y_r T^T Y^T) B`` of the stale
  trailing block ``B = a[k:, panel_end:]`` (:1106-1119, :905-946), where the
  reference passes the global step index as the panel-local row ``r = j``
  (clamped to the block), so for ``k > 0`` it is not the pivot row.

With ``panel_size >= min(m, n)`` (one panel) this is Householder QR with
column pivoting.  With more than one panel it is not a factorization: the
compiled path builds every later panel's reflectors from the wrong column
(see ``factor_panel``), and mid-panel pivots may come from the stale
trailing block (the reference's docstrings list that fix as future work,
:18-25).  ``exact_pivoted_qr`` -- the eager path at ``panel_size = 1`` -- is
the exact algorithm the blocked code is meant to reproduce.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

ZERO_TOL = 1e-12
ZERO_TOL_SQ = ZERO_TOL * ZERO_TOL
F32 = np.float32


@dataclass
class Panel:
    panel_start: int
    panel_end: int
    y: np.ndarray
    tau: np.ndarray
    t: np.ndarray


def householder(x: np.ndarray):
    """:286-324 -- returns ``(v, tau, alpha)`` for a 1-D float32 vector."""
    x = np.asarray(x, F32)
    x0 = x[0]
    x_tail = x[1:]
    sigma = np.dot(x_tail, x_tail)
    if sigma == 0:
        v = np.zeros_like(x)
        v[0] = 1
        return v, F32(0), x0
    norm_x = np.sqrt(x0 * x0 + sigma)
    alpha = norm_x if x0 <= 0 else -norm_x
    beta = x0 - alpha
    v = x / beta
    v[0] = 1
    return v.astype(F32), F32(-beta / alpha), F32(alpha)


def apply_reflector(v, tau, block):
    """:369-396 -- ``block - v (tau v^T block)``."""
    v = np.asarray(v)
    block = np.asarray(block)
    w = tau * (v @ block)
    return block - np.outer(v, w)


def build_compact_panel(reflectors, panel_start, panel_end, n_rows):
    """:545-599 -- Y (panel-local rows), tau and the LARFT-style forward T."""
    width = panel_end - panel_start
    y = np.zeros((n_rows - panel_start, width), F32)
    tau = np.zeros((width,), F32)
    for local_idx, (j, v, tau_j) in enumerate(reflectors):
        local_row = j - panel_start
        y[local_row:, local_idx] = v
        tau[local_idx] = tau_j
    t = np.zeros((width, width), F32)
    for i in range(width):
        t[i, i] = tau[i]
        if i == 0:
            continue
        w = -tau[i] * (y[:, :i].T @ y[:, i])
        if i > 1:
            w = t[:i, :i] @ w
        t[:i, i] = w
    return Panel(panel_start, panel_end, y, tau, t)


def apply_compact_panel(panel: Panel, block):
    """:818-862 -- ``Q_panel^T`` applied on the left: ``B - Y (T^T (Y^T B))``."""
    block = np.asarray(block, F32)
    if block.shape[0] == panel.y.shape[0]:
        tail, prefix = block, None
    elif block.shape[0] == panel.panel_start + panel.y.shape[0]:
        tail, prefix = block[panel.panel_start:], block[:panel.panel_start]
    else:
        raise ValueError(
            f"block row dimension must match panel-local or full rows, got {block.shape[0]}")
    w = panel.y.T @ tail
    w = panel.t.T @ w
    out = tail - panel.y @ w
    return out if prefix is None else np.concatenate([prefix, out], axis=0)


def exposed_row(panel: Panel, trailing_block, row_index: int):
    """:905-946 -- row ``row_index`` of the transformed trailing block.

    As in the reference, ``row_index`` is taken as panel-local when the block
    has panel-local rows and as global otherwise, and the row lookups clamp
    out-of-range indices like ``jax.lax.dynamic_index_in_dim``.
    """
    tb = np.asarray(trailing_block, F32)
    if tb.shape[0] == panel.y.shape[0]:
        local, tail = row_index, tb
    elif tb.shape[0] == panel.panel_start + panel.y.shape[0]:
        local, tail = row_index - panel.panel_start, tb[panel.panel_start:]
    else:
        raise ValueError(
            "trailing_block row dimension must match panel-local or full rows, "
            f"got {tb.shape[0]}")
    local = max(0, min(int(local), panel.y.shape[0] - 1))
    row_y = panel.y[local, :]
    left = (row_y @ panel.t.T) @ panel.y.T
    return tail[local, :] - left @ tail


def choose_pivot(norms, j: int, pivot_mode: str) -> int:
    """:202-219 -- first index of the max (``largest``) or of the smallest
    norm above ``ZERO_TOL**2`` (``smallest``), over columns ``>= j``."""
    idx = np.arange(norms.shape[0])
    trailing = idx >= j
    if pivot_mode == "largest":
        return int(np.argmax(np.where(trailing, norms, -np.inf)))
    if pivot_mode == "smallest":
        return int(np.argmin(np.where(trailing & (norms > ZERO_TOL_SQ), norms, np.inf)))
    raise ValueError(f"unsupported pivot_mode={pivot_mode}")


def factor_panel(a, perm, norms, k: int, panel_size: int, pivot_mode: str,
                 compiled: bool = True):
    """One panel; returns ``(a, perm, norms, Panel)``.

    ``compiled=True`` follows ``_factor_panel_compiled`` (:1479-1589), the
    path the reference takes by default.  Its Householder vector comes from
    ``householder_vector_panel_local_dynamic`` (:359-366), which passes the
    panel-local index ``j - k`` on as the *column* index into ``a[k:, :]``:
    for ``k > 0`` the reflector is built from column ``j - k`` (a finished
    column, zero below its diagonal), so every panel after the first yields
    trivial reflectors and a zero diagonal.  ``compiled=False`` follows the
    eager ``factor_panel`` (:1212-1383), which uses column ``j``
    (``householder_vector(a[j:, j])``, :1302) and, like the compiled path's
    incremental T (:674-726), is exact for one-column panels.
    """
    a = np.array(a, F32)
    perm = np.array(perm, np.int32)
    norms = np.array(norms, F32)
    m, n = a.shape
    limit = min(m, n)
    if not 0 <= k < limit:
        raise ValueError(f"k must be in [0, {limit}), got {k}")
    pe = min(k + panel_size, limit)
    width = pe - k
    y = np.zeros((m - k, width), F32)
    tau = np.zeros((width,), F32)
    t = np.zeros((width, width), F32)
    active = 0
    for j in range(k, pe):
        if pivot_mode == "smallest" and not np.any(norms[j:] > ZERO_TOL_SQ):
            break
        p = choose_pivot(norms, j, pivot_mode)
        if p != j:
            a[:, [j, p]] = a[:, [p, j]]
            perm[[j, p]] = perm[[p, j]]
            norms[[j, p]] = norms[[p, j]]
        lj = j - k
        col = a[k:, (j - k) if compiled else j].copy()
        x0 = col[lj]
        x_tail = np.where(np.arange(m - k) > lj, col, F32(0))
        sigma = np.dot(x_tail, x_tail)
        if sigma == 0:
            v = np.zeros((m - k,), F32)
            v[lj] = 1
            tau_j = F32(0)
            alpha = x0
        else:
            norm_x = np.sqrt(x0 * x0 + sigma)
            alpha = norm_x if x0 <= 0 else -norm_x
            beta = x0 - alpha
            v = np.where(np.arange(m - k) >= lj, col / beta, F32(0)).astype(F32)
            v[lj] = 1
            tau_j = F32(-beta / alpha)
        # append_reflector_to_panel_state_dynamic (:674-726)
        y[:, lj] = v
        tau[lj] = tau_j
        t[lj, lj] = tau_j
        prev = np.arange(width) < lj
        y_prev = np.where(prev[None, :], y, F32(0))
        w_full = -tau_j * (y_prev.T @ v)
        t_prev = np.where(prev[:, None] & prev[None, :], t, F32(0))
        w_full = t_prev @ w_full
        t[:, lj] = np.where(prev, w_full, t[:, lj])
        # apply_reflector_to_panel_block_dynamic (:786-815)
        blk = a[k:, k:pe]
        upd = apply_reflector(v, tau_j, blk)
        active_cols = np.arange(k, pe) >= j
        blk = np.where(active_cols[None, :], upd, blk)
        pc = blk[:, lj].copy()
        rows = np.arange(m - k)
        pc = np.where(rows > lj, F32(0), pc)
        pc = np.where(rows == lj, alpha, pc)
        blk[:, lj] = pc
        a[k:, k:pe] = blk
        # update_trailing_norm_metadata_in_panel (:1014-1124)
        nxt = j + 1
        if nxt < n:
            stop = min(pe, n)
            if nxt < stop:
                pblk = a[k:, k:stop]
                cur = norms[k:stop].copy()
                cmask = np.arange(k, stop) >= nxt
                row = pblk[lj, :]
                down = np.where(cmask, np.maximum(cur - np.square(row), F32(0)), cur)
                if (nxt - k) % 8 == 0:
                    masked = np.where(np.arange(m - k)[:, None] >= (nxt - k), pblk, F32(0))
                    exact = np.sum(np.square(masked), axis=0)
                    down = np.where(cmask, exact, down)
                norms[k:stop] = down
            if stop < n:
                # :1106-1112 passes the *global* row j with the panel-local
                # block a[k:, stop:], so the row used is local row j (clamped)
                panel = Panel(k, k + active + 1, y, tau, t)
                er = exposed_row(panel, a[k:, stop:], j)
                norms[stop:] = np.maximum(norms[stop:] - np.square(er), F32(0))
        active += 1
    return a, perm, norms, Panel(k, k + active, y, tau, t)


def apply_panel_to_trailing(a, panel: Panel, panel_end: int):
    """:1386-1409 / :1592-1624."""
    a = np.array(a, F32)
    if panel_end >= a.shape[1]:
        return a
    a[panel.panel_start:, panel_end:] = apply_compact_panel(panel, a[panel.panel_start:, panel_end:])
    return a


def refresh_norms(a, start_row: int):
    """:991-1011."""
    a = np.asarray(a, F32)
    if start_row >= a.shape[0]:
        return np.zeros((a.shape[1],), F32)
    return np.sum(np.square(a[start_row:, :]), axis=0)


def blocked_pivoted_qr(a, panel_size: int, pivot_mode: str = "largest", return_panels=False,
                       compiled: bool = True):
    """:1627-1722 -- returns ``(work, perm)`` (and the panels on request)."""
    a = np.array(a, F32)
    if a.ndim != 2:
        raise ValueError(f"a must be 2D, got {a.shape}")
    if panel_size <= 0:
        raise ValueError(f"panel_size must be positive, got {panel_size}")
    perm = np.arange(a.shape[1], dtype=np.int32)
    norms = np.sum(np.square(a), axis=0)
    limit = min(a.shape)
    panels = []
    for k in range(0, limit, panel_size):
        a, perm, norms, panel = factor_panel(a, perm, norms, k, panel_size, pivot_mode, compiled)
        panels.append(panel)
        a = apply_panel_to_trailing(a, panel, panel.panel_end)
        norms = refresh_norms(a, panel.panel_end)
    if return_panels:
        return a, perm, panels
    return a, perm


def exact_pivoted_qr(a, pivot_mode: str = "largest", return_panels=False):
    """Exact Householder QR with column pivoting: the reference driver at
    ``panel_size = 1`` on its eager panel path (``JAX_GPTQ_QR_TIMING=1``,
    :1443-1469), where every pivot sees exactly recomputed norms and every
    reflector is built from the pivot column."""
    return blocked_pivoted_qr(a, 1, pivot_mode, return_panels, compiled=False)


def form_q(m: int, panels) -> np.ndarray:
    """Q = H_1 H_2 ... H_r from the per-panel compact forms (float64)."""
    q = np.eye(m, dtype=np.float64)
    for p in reversed(panels):
        y = np.zeros((m, p.y.shape[1]), np.float64)
        y[p.panel_start:] = p.y
        width = p.panel_end - p.panel_start
        y = y[:, :width]
        t = np.asarray(p.t, np.float64)[:width, :width]
        q = q - y @ (t @ (y.T @ q))
    return q


def qr_residual(a, work, perm, panels) -> float:
    """``||A P - Q R||_F / ||A||_F`` with Q from the returned reflectors."""
    a = np.asarray(a, np.float64)
    m, n = a.shape
    q = form_q(m, panels)
    r = np.triu(np.asarray(work, np.float64))
    return float(np.linalg.norm(a[:, perm] - q @ r) / max(np.linalg.norm(a), 1e-300))
