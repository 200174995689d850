"""Hessian processing and the GPTQ step -- restates ``src/jax_gptq/gptq_ref.py``.

Test infrastructure (see ``oracle/__init__.py``).

Reference semantics (what the reference actually returns):

* ``process_hessian(solver_mode="chol")`` (gptq_ref.py:61-93) builds the
  permutation (``argsort(diag h)[::-1]`` with a stable sort, gptq_ref.py:67-68,
  else ``arange``, :70), and then *always* returns the identity as
  ``h_inv_sqrt``: line 85 calls ``jax.scipy`` in a module that only imported
  ``jax.numpy as jnp`` (gptq_ref.py:1), the NameError is swallowed by the bare
  ``except`` (:88-89) on all five damping attempts, and :91-92 falls back to
  ``eye(n)``.
* ``gptq_forward_step`` (gptq_ref.py:136-155) ignores ``h_inv_sqrt`` (:150):
  permute columns, RTN (quant.py), un-permute with ``argsort(perm)``.

Intended semantics (the algorithm the reference's docstrings describe; no
counterpart output exists in the reference): damped Cholesky with the
10x-damping retry loop of gptq_ref.py:79-83 actually working, the upper
factor ``U = chol(H^-1, upper)``, and the GPTQ column sweep of Frantar et
al. (2022) with lazy batch updates of ``block`` columns and groups whose
scale/zero are taken from the current (error-updated) weights at each group's
first column.  With ``U = I`` the sweep equals the reference exactly.
"""

from __future__ import annotations

import numpy as np

from . import quant as oq


def select_truncation_rank(eigvals_desc: np.ndarray, mode: str, value: float) -> int:
    """gptq_ref.py:8-41."""
    if eigvals_desc.ndim != 1:
        raise ValueError(f"eigvals_desc must be 1D, got {eigvals_desc.shape}")
    n = eigvals_desc.shape[0]
    if n == 0:
        raise ValueError("eigvals_desc must be non-empty")
    value = float(value)
    if mode == "abs":
        rank = int(np.sum(eigvals_desc > value))
    elif mode == "percent":
        drop_frac = min(max(value / 100.0, 0.0), 1.0)
        rank = int(np.ceil((1.0 - drop_frac) * n))
    elif mode == "mean_top32":
        ref_val = np.mean(eigvals_desc[: min(32, n)])
        rank = int(np.sum(eigvals_desc > value * ref_val))
    elif mode == "energy":
        total = np.sum(eigvals_desc)
        rank = int(np.sum(np.cumsum(eigvals_desc) <= (1.0 - value) * total))
        if rank < n:
            rank += 1
    else:
        raise ValueError(f"unsupported truncation_mode={mode}")
    return max(1, min(rank, n))


def act_order_perm(h: np.ndarray, ordering_mode: str) -> np.ndarray:
    """gptq_ref.py:67-70: descending diag(h); JAX's argsort is stable, so
    after the reversal equal diagonals come out highest-index-first."""
    n = h.shape[0]
    if ordering_mode == "diag_h":
        return np.argsort(np.diag(h), kind="stable")[::-1].astype(np.int32)
    return np.arange(n, dtype=np.int32)


def check_hessian_args(h: np.ndarray, solver_mode: str, ordering_mode: str) -> None:
    """gptq_ref.py:56-57, 62-65, 95-96."""
    if h.ndim != 2 or h.shape[0] != h.shape[1]:
        raise ValueError(f"h must be square 2D, got {h.shape}")
    if solver_mode == "chol":
        if ordering_mode not in {"none", "diag_h"}:
            raise ValueError(
                f"ordering_mode={ordering_mode} is not supported for solver_mode='chol'")
    elif solver_mode != "eigh":
        raise ValueError(f"unsupported solver_mode={solver_mode}")


def process_hessian_reference(h, ordering_mode: str = "none", solver_mode: str = "chol",
                              truncation_mode: str = "abs", truncation_value: float = 1e-5,
                              panel_size: int = 32):
    """Observed output of gptq_ref.py:44-133: ``(eye(n), perm)`` for the
    Cholesky branch (it always falls back, :85-92), the eigh branch as
    written otherwise (:95-133, see :func:`process_hessian_eigh`)."""
    h = np.asarray(h)
    check_hessian_args(h, solver_mode, ordering_mode)
    if solver_mode == "eigh":
        return process_hessian_eigh(h, ordering_mode, truncation_mode, truncation_value,
                                    panel_size, semantics="reference")
    perm = act_order_perm(h, ordering_mode)
    return np.eye(h.shape[0], dtype=h.dtype), perm


def process_hessian_eigh(h, ordering_mode: str = "none", truncation_mode: str = "abs",
                         truncation_value: float = 1e-5, panel_size: int = 32,
                         semantics: str = "reference", dtype=np.float32):
    """gptq_ref.py:95-133: eigendecomposition, truncation, and an upper factor.

    ``sqrt_h = sqrt(lam) V^T`` and ``sqrt_hinv = lam^-1/2 V^T`` (rank x n, the
    kept eigenpairs in descending order).  For none / diag_h / pivot_sqrt_h the
    factor is R of the QR of ``sqrt_hinv.T[:, perm]`` (:112, :117, :122): in
    ``reference`` semantics exactly that -- the permutation indexes the eigen
    axis, and for rank < n the gather runs past the kept columns and is
    clamped to the last one, as JAX clamps out-of-range gathers; in
    ``intended`` semantics the permutation acts on the feature axis,
    ``sqrt_hinv[:, perm]``, so that ``R^T R = H^+[perm][:, perm]``.  For
    pivot_sqrt_hinv_smallest the factor is the blocked pivoted QR of
    ``sqrt_hinv`` itself (:125-131).  The QR's own semantics follow
    ``semantics`` (compiled-path quirks for reference)."""
    from . import qr as oqr
    h = np.asarray(h, dtype)
    n = h.shape[0]
    evals, evecs = np.linalg.eigh(h)
    evals, evecs = evals[::-1], evecs[:, ::-1]
    rank = select_truncation_rank(np.asarray(evals, np.float64), truncation_mode,
                                  truncation_value)
    lam, v = evals[:rank], evecs[:, :rank]
    sqrt_h = (np.sqrt(lam)[:, None] * v.T).astype(dtype)
    sqrt_hinv = (np.power(lam, -0.5)[:, None] * v.T).astype(dtype)
    compiled = semantics == "reference"
    if ordering_mode == "pivot_sqrt_hinv_smallest":
        work, perm = oqr.blocked_pivoted_qr(sqrt_hinv, panel_size, "smallest", compiled=compiled)
        return np.asarray(work, dtype), np.asarray(perm, np.int32)
    if ordering_mode == "none":
        perm = np.arange(n, dtype=np.int32)
    elif ordering_mode == "diag_h":
        perm = act_order_perm(h, "diag_h")
    elif ordering_mode == "pivot_sqrt_h":
        _, perm = oqr.blocked_pivoted_qr(sqrt_h, panel_size, "largest", compiled=compiled)
        perm = np.asarray(perm, np.int32)
    else:
        raise ValueError(f"unsupported ordering_mode={ordering_mode}")
    if semantics == "reference":
        m = sqrt_hinv.T[:, np.clip(perm, 0, rank - 1)]
    else:
        m = sqrt_hinv[:, perm]
    return np.linalg.qr(m, mode="r").astype(dtype), perm


def damped_permuted(h: np.ndarray, perm: np.ndarray, damp: float, dtype=np.float64):
    """gptq_ref.py:72-83: ``h[perm][:, perm] + damp * mean(diag) * I`` (mean 0 -> 1)."""
    hp = np.asarray(h, dtype)[perm][:, perm]
    diag_mean = np.mean(np.diag(hp))
    if float(diag_mean) == 0.0:
        diag_mean = 1.0
    return hp + damp * diag_mean * np.eye(hp.shape[0], dtype=dtype)


def process_hessian_intended(h, ordering_mode: str = "none", damp_percent: float = 0.01,
                             dtype=np.float64):
    """Working version of gptq_ref.py:61-93.

    Returns ``(U, perm, attempt)`` with ``U`` upper triangular,
    ``U^T U = (H_perm + damp I)^-1``; ``attempt`` is the damping exponent that
    succeeded (-1 when all five failed and the identity is returned, as the
    reference's fallback does).
    """
    h = np.asarray(h)
    check_hessian_args(h, "chol", ordering_mode)
    perm = act_order_perm(h, ordering_mode)
    n = h.shape[0]
    for attempt in range(5):
        damp = (10 ** attempt) * damp_percent
        hd = damped_permuted(h, perm, damp, dtype)
        try:
            np.linalg.cholesky(hd)
            hinv = np.linalg.inv(hd)
            hinv = 0.5 * (hinv + hinv.T)
            u = np.linalg.cholesky(hinv).T
        except np.linalg.LinAlgError:
            continue
        if not np.all(np.isfinite(u)):
            continue
        return u.astype(dtype), perm, attempt
    return np.eye(n, dtype=dtype), perm, -1


def gptq_forward_step_reference(weight, perm, w_bits=4, group_size=128, sym=False):
    """gptq_ref.py:146-155 (``h_inv_sqrt`` ignored)."""
    weight = np.asarray(weight, np.float32)
    perm = np.asarray(perm)
    if weight.ndim != 2:
        raise ValueError(f"weight must be 2D, got {weight.shape}")
    if perm.ndim != 1 or perm.shape[0] != weight.shape[1]:
        raise ValueError(f"perm must be shape ({weight.shape[1]},), got {perm.shape}")
    w_q = oq.quantize_dequantize(weight[:, perm], w_bits, group_size, sym)
    inv_perm = np.argsort(perm, kind="stable")
    return w_q[:, inv_perm]


def gptq_sweep(weight, u, perm, w_bits=4, group_size=128, sym=False, block=128,
               dtype=np.float32, group0=None, noprop_cols=0, start=None, return_pre=False):
    """GPTQ column sweep with lazy block updates (Frantar et al., 2022).

    ``u`` is the upper factor in permuted coordinates.  Returns a dict with
    ``dequant`` (original column order), ``q`` (codes, original order),
    ``scales``/``zeros`` (``[m, n // group_size]``, permuted group order) and
    ``g_idx`` (group of each original column).

    ``start`` (permuted order) replaces ``weight[:, perm]`` as the initial
    estimate; ``group0`` = (scale, zero) presets group 0's parameters and
    ``noprop_cols`` columns at the front propagate no error (both used by the
    Qronos first step).  ``return_pre`` adds ``pre`` ([m, n], permuted
    order): the unrounded ``w / scale + zero`` each code was rounded from.
    """
    w = np.asarray(weight)
    m, n = w.shape
    perm = np.asarray(perm)
    g = group_size
    oq.check_rtn_args(w, g)
    wp = (np.asarray(start) if start is not None else w[:, perm]).astype(dtype).copy()
    u = np.asarray(u, dtype)
    q_out = np.zeros((m, n), dtype)
    dq_out = np.zeros((m, n), dtype)
    n_groups = n // g
    scales = np.zeros((m, n_groups), dtype)
    zeros = np.zeros((m, n_groups), dtype)
    qmin, qmax = oq.qrange(w_bits, sym)
    pre_out = np.zeros((m, n), dtype) if return_pre else None
    scale = zero = None
    for b0 in range(0, n, block):
        b1 = min(b0 + block, n)
        err_blk = np.zeros((m, b1 - b0), dtype)
        for i in range(b0, b1):
            if i % g == 0:
                gi = i // g
                if gi == 0 and group0 is not None:
                    scale = np.asarray(group0[0], dtype).reshape(m, 1)
                    zero = np.asarray(group0[1], dtype).reshape(m, 1)
                else:
                    scale, zero = oq.group_params(wp[:, i:i + g], w_bits, sym)
                    scale = scale.astype(dtype)
                    zero = zero.astype(dtype)
                scales[:, gi] = scale[:, 0]
                zeros[:, gi] = zero[:, 0]
            col = wp[:, i]
            pre = col / scale[:, 0] + zero[:, 0]
            if return_pre:
                pre_out[:, i] = pre
            qc = np.clip(np.round(pre), qmin, qmax).astype(dtype)
            dq = ((qc - zero[:, 0]) * scale[:, 0]).astype(dtype)
            q_out[:, i] = qc
            dq_out[:, i] = dq
            if i < noprop_cols:
                continue
            err = (col - dq) / u[i, i]
            wp[:, i + 1:b1] -= err[:, None] * u[i, i + 1:b1][None, :]
            err_blk[:, i - b0] = err
        if b1 < n:
            wp[:, b1:] -= err_blk @ u[b0:b1, b1:]
    inv_perm = np.argsort(perm, kind="stable")
    g_idx = (inv_perm // g).astype(np.int32)
    out = {
        "dequant": dq_out[:, inv_perm],
        "q": q_out[:, inv_perm],
        "scales": scales,
        "zeros": zeros,
        "g_idx": g_idx,
    }
    if return_pre:
        out["pre"] = pre_out
    return out


def reconstruction_error(w, w_hat, h) -> float:
    """``||W X^T - W_hat X^T||_F / ||W X^T||_F`` evaluated through ``H = X^T X``."""
    w = np.asarray(w, np.float64)
    d = w - np.asarray(w_hat, np.float64)
    h = np.asarray(h, np.float64)
    num = np.einsum("ij,jk,ik->", d, h, d)
    den = np.einsum("ij,jk,ik->", w, h, w)
    return float(np.sqrt(max(num, 0.0) / max(den, 1e-300)))
