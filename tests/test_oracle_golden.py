"""Pin the numpy oracle to golden vectors produced by the reference's own code.

``tests/golden/make_golden.py`` ran the reference's unmodified modules under a
numpy-backed ``jax`` stand-in; these tests check that the oracle restatement
reproduces those outputs (bit-exact codes, pivots and, where the op order is
the same, values).
"""

import os

import numpy as np
import pytest

from oracle import gptq as og
from oracle import qr as oqr
from oracle import qronos as oqn
from oracle import quant as oq
from oracle import stats as ost


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_rtn_matches_reference(golden_dir):
    d = _load(golden_dir, "rtn_golden.npz")
    names = [k[:-2] for k in d.files if k.startswith("rtn_") and k.endswith("_w")]
    assert len(names) >= 6
    for name in names:
        bits, gs, sym = (int(v) for v in d[name + "_cfg"])
        out = oq.quantize_dequantize(d[name + "_w"], bits, gs, bool(sym))
        assert np.array_equal(out, d[name + "_out"]), name


def test_reference_smoke_script_values(golden_dir):
    """scripts/smoke.py:8-16: arange weights, group 4, h passed as h_inv_sqrt."""
    d = _load(golden_dir, "rtn_golden.npz")
    h, g = ost.h_g_from_activations(d["smoke_xq"], d["smoke_xf"], dtype=np.float32)
    assert np.allclose(h, d["smoke_h"], rtol=1e-6)
    assert np.allclose(g, d["smoke_g"], rtol=1e-6)
    out = og.gptq_forward_step_reference(d["smoke_w"], np.arange(8), 4, 4, False)
    assert np.array_equal(out, d["smoke_out"])


@pytest.mark.parametrize("case", ["none", "diag", "diag_sym3"])
def test_gptq_and_qronos_match_reference(golden_dir, case):
    d = _load(golden_dir, "gptq_golden.npz")
    p = f"gptq_{case}"
    bits, gs, sym, diag = (int(v) for v in d[p + "_cfg"])
    x = d[p + "_x"]
    h = x.T @ x
    u, perm = og.process_hessian_reference(h, "diag_h" if diag else "none")
    assert bool(d[p + "_hinv_is_eye"]) and np.array_equal(u, np.eye(h.shape[0]))
    assert np.array_equal(perm, d[p + "_perm"])
    out = og.gptq_forward_step_reference(d[p + "_w"], perm, bits, gs, bool(sym))
    assert np.array_equal(out, d[p + "_out"])
    # the intended sweep reduces to the reference when U = I
    sw = og.gptq_sweep(d[p + "_w"], np.eye(h.shape[0], dtype=np.float32), perm, bits, gs,
                       bool(sym))
    assert np.array_equal(sw["dequant"], d[p + "_out"])
    qr_out = oqn.qronos_reference(d[p + "_w"], d[p + "_w"], h, h, bits, gs, bool(sym))
    assert np.array_equal(qr_out, d[p + "_qronos"])


def test_hg_matches_reference(golden_dir):
    d = _load(golden_dir, "gptq_golden.npz")
    h, g = ost.h_g_from_activations(d["gptq_none_x"])
    ok, fro, worst = ost.h_tolerance_ok(d["gptq_none_h"], h)
    assert ok, (fro, worst)
    assert np.array_equal(d["gptq_none_g"], d["gptq_none_h"])  # x_float=None -> g = h
    _, g2 = ost.h_g_from_activations(d["gptq_none_x"], d["gptq_none_xf"])
    assert ost.h_tolerance_ok(d["gptq_none_g2"], g2)[0]


def test_blocked_qr_compiled_path_matches_reference(golden_dir):
    d = _load(golden_dir, "qr_golden.npz")
    names = [k[:-2] for k in d.files if k.startswith("qr_") and k.endswith("_a")]
    assert len(names) >= 10
    for name in names:
        panel, sm = (int(v) for v in d[name + "_cfg"])
        work, perm = oqr.blocked_pivoted_qr(d[name + "_a"], panel,
                                            "smallest" if sm else "largest")
        assert np.array_equal(perm, d[name + "_perm"]), name
        assert np.array_equal(work, d[name + "_work"]), name


def test_exact_qrcp_matches_reference_eager_panel1(golden_dir):
    d = _load(golden_dir, "qr_golden.npz")
    names = [k[:-2] for k in d.files if k.startswith("exact_") and k.endswith("_a")]
    assert len(names) >= 4
    for name in names:
        _, sm = (int(v) for v in d[name + "_cfg"])
        a = d[name + "_a"]
        work, perm, panels = oqr.exact_pivoted_qr(a, "smallest" if sm else "largest",
                                                  return_panels=True)
        assert np.array_equal(perm, d[name + "_perm"]), name
        scale = np.abs(d[name + "_work"]).max()
        assert np.allclose(work, d[name + "_work"], atol=1e-5 * scale), name
        assert oqr.qr_residual(a, work, perm, panels) <= 1e-5


def test_factor_panel_state_matches_reference(golden_dir):
    d = _load(golden_dir, "qr_golden.npz")
    a = d["panel_a"]
    a_out, perm, norms, panel = oqr.factor_panel(a, np.arange(a.shape[1], dtype=np.int32),
                                                 d["panel_norms_in"], 8, 8, "largest")
    assert np.array_equal(a_out, d["panel_a_out"])
    assert np.array_equal(perm, d["panel_perm_out"])
    assert np.array_equal(norms, d["panel_norms_out"])
    assert np.array_equal(panel.y, d["panel_y"])
    assert np.array_equal(panel.t, d["panel_t"])
    assert np.array_equal(panel.tau, d["panel_tau"])
    assert panel.panel_end == int(d["panel_end"])


def test_reference_qr_known_answers():
    """Known-answer cases of the reference's tests/test_blocked_pivoted_qr.py."""
    ex = np.array([[3.0, 1.0, 0.0, 2.0], [4.0, 0.0, 2.0, 1.0],
                   [0.0, 5.0, 1.0, 0.0], [0.0, 0.0, 6.0, 1.0]], np.float32)
    # :263-282 reflector update
    v = np.array([1.0, 0.25, -0.5, 0.75], np.float32)
    blk = ex[:, :3]
    out = oqr.apply_reflector(v, np.float32(0.8), blk)
    w = np.float32(0.8) * (v @ blk)
    assert np.allclose(out, blk - np.outer(v, w), atol=1e-6)
    # :391-401 Y = I, T = 0.1 I  =>  0.9 * B
    y = np.eye(8, dtype=np.float32)
    panel = oqr.Panel(0, 8, y, np.full(8, 0.1, np.float32), np.diag(np.full(8, 0.1, np.float32)))
    b = np.arange(1024.0, dtype=np.float32).reshape(8, 128)
    assert np.allclose(oqr.apply_compact_panel(panel, b), 0.9 * b, atol=5e-4)
    # :101-132 triangularity and diagonal monotonicity
    work, _ = oqr.blocked_pivoted_qr(ex, 2, "largest")
    assert np.linalg.norm(np.tril(work, -1)) < 1e-5
    da = np.abs(np.diag(work))
    assert np.all(da[:-1] >= da[1:])
    work, _ = oqr.blocked_pivoted_qr(ex, 2, "smallest")
    assert np.linalg.norm(np.tril(work, -1)) < 1e-5
    # :135-142 single-panel reconstruction
    work, perm, panels = oqr.blocked_pivoted_qr(ex, 4, "largest", return_panels=True)
    assert oqr.qr_residual(ex, work, perm, panels) < 1e-6
    # :507-533 all-zero matrix, smallest mode: no reflector accepted
    _, _, _, pz = oqr.factor_panel(np.zeros((3, 3), np.float32), np.arange(3), np.zeros(3),
                                   0, 2, "smallest")
    assert pz.panel_end == 0


def test_intended_gptq_improves_on_rtn():
    from oracle import inputs
    w, x = inputs.single_linear(0, m=64, n=256, tokens=512)
    h = (x.astype(np.float64).T @ x) / x.shape[0]
    u, perm, attempt = og.process_hessian_intended(h, "diag_h", 0.01)
    assert attempt == 0
    out = og.gptq_sweep(w, u, perm, 4, 128, False, dtype=np.float64)
    rtn = oq.quantize_dequantize(w, 4, 128, False)
    e_gptq = og.reconstruction_error(w, out["dequant"], h)
    e_rtn = og.reconstruction_error(w, rtn, h)
    assert e_gptq < 0.8 * e_rtn


def test_intended_qronos_improves_on_rtn():
    from oracle import inputs
    w, x = inputs.single_linear(2, m=32, n=256, tokens=512)
    rng = np.random.default_rng(2)
    xt = x + rng.standard_normal(x.shape).astype(np.float32) * 0.05 * x.std(0)
    h, g = ost.h_g_from_activations(xt, x)
    out = oqn.qronos_intended(w, w, h, g, 3, 128, False)
    # target is X w; compare ||X w - Xt w_hat|| for Qronos and for RTN
    def err(w_hat):
        return np.linalg.norm(x.astype(np.float64) @ w.T - xt.astype(np.float64) @ w_hat.T)
    assert err(out["dequant"]) < 0.8 * err(oq.quantize_dequantize(w, 3, 128, False))


def test_eigh_branch_matches_reference_golden(golden_dir):
    """gptq_ref.py:95-133 run by the reference itself (numpy shim): every
    ordering mode, full-rank and truncated H."""
    g = _load(golden_dir, "eigh_golden.npz")
    for name in ("full", "deficient"):
        h = g[f"eigh_{name}_h"]
        for mode in ("none", "diag_h", "pivot_sqrt_h", "pivot_sqrt_hinv_smallest"):
            r, p = og.process_hessian_reference(h, mode, "eigh", panel_size=8)
            assert np.array_equal(p, g[f"eigh_{name}_{mode}_perm"]), (name, mode)
            assert np.array_equal(r, g[f"eigh_{name}_{mode}_r"]), (name, mode)
