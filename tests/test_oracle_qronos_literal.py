"""The Qronos oracle against a literal, column-by-column reading of the
paper's two update rules (float64, CPU, tiny sizes).

The reference's ``qronos_single_layer_update_ref`` is a placeholder
(``qronos_ref.py:14-25``), so the intended-semantics oracle
(``oracle.qronos.qronos_intended``) is checked here against the rules of
Zhang, Zhang & Saab (2025) applied literally at every column t, with
``hd`` the damped Hessian of the quantized-model activations and
``g = X^T Xt`` (the reference's ``h_g_from_activations`` convention):

* correct the past -- the value to quantize at column t is the least-squares
  best v given the already quantized columns and the current estimate of the
  later ones:
  ``v_t = (r_t - sum_{j<t} hd_tj q_j - sum_{j>t} hd_tj w_j) / hd_tt``,
  ``r = w_orig g`` (the normal equations' right-hand side), ``q_t = Q(v_t)``;
* shape the future -- the later columns are re-solved exactly:
  ``w_{>t} = hd_{>t,>t}^-1 (r_{>t} - hd_{>t,<=t} q_{<=t})``.

The oracle instead solves once after the first column and then runs the GPTQ
sweep with ``U = chol(hd^-1, upper)``: it asserts that, once the later
columns are the least-squares optimum, the first rule returns the current
estimate and the second is the GPTQ (optimal brain surgeon) update.  These
tests check that equivalence numerically, including group parameters taken
at each group's first column (group 0 from the starting weights).
"""

import numpy as np
import pytest

from oracle import gptq as og
from oracle import qronos as oqn
from oracle import quant as oq


def _literal_qronos(w, w_orig, hd, gp, bits, gsize, sym=False):
    """Column-by-column Qronos in float64 (permuted coordinates)."""
    m, n = w.shape
    qmin, qmax = oq.qrange(bits, sym)
    r = w_orig @ gp
    cur = w.copy()
    q = np.zeros((m, n))
    dq = np.zeros((m, n))
    pre = np.zeros((m, n))
    scale = zero = None
    for t in range(n):
        v = (r[:, t] - dq[:, :t] @ hd[t, :t] - cur[:, t + 1:] @ hd[t, t + 1:]) / hd[t, t]
        if t % gsize == 0:
            # group 0 from the starting weights; later groups from the current
            # estimate of their columns, with column t at its corrected value
            blk = w[:, :gsize] if t == 0 else np.concatenate([v[:, None], cur[:, t + 1:t + gsize]], 1)
            s, z = oq.group_params(blk.astype(np.float64), bits, sym)
            scale, zero = s[:, 0].astype(np.float64), z[:, 0].astype(np.float64)
        pre[:, t] = v / scale + zero
        q[:, t] = np.clip(np.round(pre[:, t]), qmin, qmax)
        dq[:, t] = (q[:, t] - zero) * scale
        cur[:, t] = v
        if t + 1 < n:
            rhs = r[:, t + 1:] - dq[:, :t + 1] @ hd[t + 1:, :t + 1].T
            cur[:, t + 1:] = np.linalg.solve(hd[t + 1:, t + 1:], rhs.T).T
    return q, dq, pre


@pytest.mark.parametrize("m,n,bits,gsize,ordering,seed", [
    (6, 24, 3, 8, "diag_h", 0), (5, 32, 4, 16, "none", 1), (4, 40, 2, 8, "diag_h", 2)])
def test_qronos_oracle_equals_literal_update_rules(m, n, bits, gsize, ordering, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((8 * n, n)) * rng.lognormal(0, 0.7, n)
    xt = x + rng.standard_normal(x.shape) * 0.05 * x.std(0)
    h = xt.T @ xt
    g = x.T @ xt
    w_orig = rng.standard_normal((m, n)) * 0.02
    w = w_orig + rng.standard_normal((m, n)) * 0.002   # a starting estimate != w_orig
    ref = oqn.qronos_intended(w, w_orig, h, g, bits, gsize, False, ordering_mode=ordering,
                              dtype=np.float64, return_pre=True)
    perm = ref["perm"]
    u, perm2, att = og.process_hessian_intended(h, ordering, 0.01)
    assert np.array_equal(perm, perm2) and att == 0
    hd = og.damped_permuted(h, perm, 0.01)
    gp = g[perm][:, perm]
    q, dq, pre = _literal_qronos(w[:, perm], w_orig[:, perm], hd, gp, bits, gsize)
    # the oracle's unrounded values equal the literal "correct the past" values
    assert np.allclose(ref["pre"], pre, rtol=0, atol=1e-9 * np.abs(pre).max())
    # no value sits within 1e-6 of a half step, so the codes must agree exactly
    assert np.min(np.abs(pre - np.floor(pre) - 0.5)) > 1e-6
    assert np.array_equal(ref["q"][:, perm], q)
    assert np.allclose(ref["dequant"][:, perm], dq, rtol=1e-12, atol=1e-15)


def test_literal_rules_reduce_to_gptq_when_g_is_the_damped_h():
    """With g equal to the damped Hessian and the starting weights equal to
    w_orig, the first correction returns w_orig's own first column and the
    literal Qronos rules are exactly the GPTQ sweep."""
    rng = np.random.default_rng(7)
    n, m = 32, 5
    x = rng.standard_normal((8 * n, n)) * rng.lognormal(0, 0.7, n)
    h = x.T @ x
    w = rng.standard_normal((m, n)) * 0.02
    u, perm, _ = og.process_hessian_intended(h, "none", 0.01)
    hd = og.damped_permuted(h, perm, 0.01)
    q, dq, _ = _literal_qronos(w, w, hd, hd, 4, 8)
    ref = og.gptq_sweep(w, u, perm, 4, 8, False, dtype=np.float64)
    assert np.array_equal(ref["q"], q)
    assert np.allclose(ref["dequant"], dq, rtol=1e-12, atol=1e-15)
