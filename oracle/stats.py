"""Hessian / cross-covariance statistics -- restates ``src/jax_gptq/stats.py:4-18``.

Test infrastructure (see ``oracle/__init__.py``).  Layout is
``[tokens, in_features]`` (stats.py:15); ``h = x_q^T x_q`` (stats.py:16) and
``g = x_f^T x_q`` (stats.py:17), with ``x_f`` defaulting to ``x_q``
(stats.py:10-11).
"""

from __future__ import annotations

import numpy as np


def check_hg_args(x_quant: np.ndarray, x_float) -> None:
    """ValueError contract of stats.py:8-13."""
    if x_quant.ndim != 2:
        raise ValueError(f"x_quant must be 2D [tokens, in_features], got {x_quant.shape}")
    if x_float is not None and x_float.shape != x_quant.shape:
        raise ValueError(
            f"x_float shape must match x_quant, got {x_float.shape} vs {x_quant.shape}")


def h_g_from_activations(x_quant, x_float=None, dtype=np.float64):
    """Returns ``(h, g)`` computed in ``dtype`` (float64 for tolerance checks)."""
    xq = np.asarray(x_quant)
    xf = None if x_float is None else np.asarray(x_float)
    check_hg_args(xq, xf)
    xq = xq.astype(dtype)
    xf = xq if xf is None else xf.astype(dtype)
    h = xq.T @ xq
    g = xf.T @ xq
    return h, g


def h_tolerance_ok(h_test, h_ref, rel: float = 1e-5) -> tuple[bool, float, float]:
    """Frobenius-relative error and the elementwise bound
    ``|dH_ij| <= rel * sqrt(H_ii H_jj)`` used for H parity."""
    h_test = np.asarray(h_test, np.float64)
    h_ref = np.asarray(h_ref, np.float64)
    diff = h_test - h_ref
    fro = float(np.linalg.norm(diff) / max(np.linalg.norm(h_ref), 1e-300))
    d = np.sqrt(np.maximum(np.diag(h_ref), 0.0))
    bound = rel * np.outer(d, d)
    worst = float(np.max(np.abs(diff) / np.maximum(bound, 1e-300)))
    return (fro <= rel and worst <= 1.0), fro, worst
