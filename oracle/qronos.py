"""Qronos single-layer update -- restates ``src/jax_gptq/qronos_ref.py:7-25``.

Test infrastructure (see ``oracle/__init__.py``).

Reference semantics: shape checks (qronos_ref.py:18-23) and then
``quantize_dequantize(weight_orig, cfg)`` (qronos_ref.py:25); ``weight``,
``h`` and ``g`` are ignored (:24).

Intended semantics (Qronos, Zhang, Zhang & Saab 2025: "correct the past,
shape the future"), restated from its update rules.  With ``X`` the float
activations, ``Xt`` the quantized-model activations, ``h = Xt^T Xt`` and
``g = X^T Xt`` (the reference's ``h_g_from_activations(x_quant=Xt,
x_float=X)`` convention), each output row ``w`` minimises
``||X w_orig - Xt q||``:

1. first column: ``v1 = argmin_v ||X w_orig - Xt_1 v - Xt_{>1} w_{>1}||``
   ``= ((g^T w_orig)_1 - h_{1,>1} w_{>1}) / h_11`` and ``q1 = Q(v1)`` with
   group-0 parameters from the starting weights;
2. future: ``w_{>1} = h_{>1,>1}^-1 ((g^T w_orig)_{>1} - h_{>1,1} q1)``;
3. columns 2..n: because step 2 makes the remaining weights the joint
   least-squares optimum, "correcting the past" reduces to quantizing the
   current estimate, and "shaping the future" is the GPTQ error-feedback
   update with ``U = chol(h^-1, upper)`` -- so the GPTQ sweep runs on the
   corrected weights with column 1 fixed.

``h`` is damped exactly like GPTQ's Hessian.
"""

from __future__ import annotations

import numpy as np

from . import gptq as og
from . import quant as oq


def check_qronos_args(weight, weight_orig, h, g) -> None:
    """qronos_ref.py:18-23."""
    if weight.ndim != 2 or weight_orig.ndim != 2:
        raise ValueError("weight and weight_orig must be 2D")
    if weight.shape != weight_orig.shape:
        raise ValueError("weight and weight_orig shape mismatch")
    if h.shape[0] != h.shape[1] or g.shape != h.shape:
        raise ValueError("h must be square and g must match h shape")


def qronos_reference(weight, weight_orig, h, g, w_bits=4, group_size=128, sym=False):
    weight = np.asarray(weight)
    weight_orig = np.asarray(weight_orig, np.float32)
    h = np.asarray(h)
    g = np.asarray(g)
    check_qronos_args(weight, weight_orig, h, g)
    return oq.quantize_dequantize(weight_orig, w_bits, group_size, sym)


def qronos_intended(weight, weight_orig, h, g, w_bits=4, group_size=128, sym=False,
                    ordering_mode="none", damp_percent=0.01, block=128, dtype=np.float64,
                    factor=None, return_pre=False):
    """``factor = (u, perm, hd)`` replaces the oracle's own factor of ``h``
    (to compare the update and sweep arithmetic alone); ``return_pre`` adds
    the sweep's unrounded values (see :func:`oracle.gptq.gptq_sweep`)."""
    weight = np.asarray(weight)
    weight_orig = np.asarray(weight_orig)
    h = np.asarray(h)
    g = np.asarray(g)
    check_qronos_args(weight, weight_orig, h, g)
    m, n = weight.shape
    if factor is None:
        u, perm, attempt = og.process_hessian_intended(h, ordering_mode, damp_percent, dtype)
        damp = (10 ** max(attempt, 0)) * damp_percent
        hd = og.damped_permuted(h, perm, damp, dtype)
    else:
        u, perm, hd = (np.asarray(factor[0], dtype), np.asarray(factor[1]),
                       np.asarray(factor[2], dtype))
        attempt = 0
    gp = np.asarray(g, dtype)[perm][:, perm]
    wp = np.asarray(weight, dtype)[:, perm]
    wop = np.asarray(weight_orig, dtype)[:, perm]
    rhs = wop @ gp                       # row r: (g^T w_orig)_perm
    s0, z0 = oq.group_params(wp[:, :group_size], w_bits, sym)
    s0 = s0.astype(dtype)[:, 0]
    z0 = z0.astype(dtype)[:, 0]
    v1 = (rhs[:, 0] - wp[:, 1:] @ hd[0, 1:]) / hd[0, 0]
    qmin, qmax = oq.qrange(w_bits, sym)
    q1 = np.clip(np.round(v1 / s0 + z0), qmin, qmax)
    dq1 = (q1 - z0) * s0
    b = rhs[:, 1:] - dq1[:, None] * hd[0, 1:][None, :]
    future = np.linalg.solve(hd[1:, 1:], b.T).T if n > 1 else np.zeros((m, 0), dtype)
    start = np.concatenate([v1[:, None], future], axis=1)
    out = og.gptq_sweep(weight, u, perm, w_bits, group_size, sym, block, dtype,
                        group0=(s0, z0), noprop_cols=1, start=start, return_pre=return_pre)
    out["perm"] = perm
    out["attempt"] = attempt
    return out
