"""Parity at the benchmark configurations' own sizes (through the C ABI).

* Single linear, full size (1024 x 1024 W ~ N(0, 0.02^2); 2048 x 1024 X ~
  N(0, 1) with 8 input channels x20; H = X^T X / n; damp 0.01; 4-bit asym,
  g128, block 128, no act-order; seed 0): H within 1e-5 of float64; codes
  equal to the float32 oracle sweep given the same factor except rows whose
  first differing code is a rounding tie (counted); dequantized values of the
  other rows within 1e-5 relative; the reconstruction error
  ||WX - W^X|| / ||WX|| within 1e-3 relative of the float64 oracle's (each
  with its own factor).  Reference semantics at full size: bit-exact.
* Llama-2-7B layer set, sampled: H and the Qronos cross term G of the
  d = 11008 input over 262,144 bf16 tokens (log-normal channel scales) on
  256 x 256 tiles against float64 sums of the same bf16 columns; the GPTQ
  sweep (4-bit, act-order) and the Qronos update (3-bit) of the 4096 x 11008
  down projection on sampled 32-row blocks against the float32 oracle with
  the same factor.
* Pivoted QR of the 4096 x 4096 benchmark matrices: pivots and |diag R|
  against the oracle's fixture (``tests/golden/qr4096_fixture.npz``), and
  ||AP - QR|| / ||A|| <= 1e-5.

Measured tie counts go to ``GQ_PARITY_REPORT`` when it is set.
"""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import QuantConfig, gptq_forward_step, h_g_from_activations, process_hessian
from jax_gptq_b200 import gptq_ref as G
from jax_gptq_b200 import layerset as LS
from jax_gptq_b200 import qronos_ref as Q
from jax_gptq_b200 import stats
from oracle import gptq as og
from oracle import inputs
from oracle import qronos as oqn
from oracle import quant as oq
from oracle import stats as ost

from parity import TIE_TOL, code_diffs, report

RECON_REL = 1e-3    # reconstruction error, relative to the oracle's
DEQUANT_REL = 1e-5  # dequantized values of rows whose codes all agree
H_REL = 1e-5


def _ties_ok(name, got_codes, ref, perm, bits, sym=False):
    """Codes (uint8, original order) against an oracle sweep dict."""
    qmin = oq.qrange(bits, sym)[0]
    got_p = got_codes.astype(np.float32)[:, perm] + qmin
    ref_p = ref["q"][:, perm]
    cd = code_diffs(got_p, ref_p, ref["pre"])
    report(name, rows=cd["rows"], tie_rows=cd["tie_rows"], codes_differing=cd["codes_differing"],
           max_tie_dist=cd["max_tie_dist"], tie_tol=TIE_TOL)
    assert cd["max_tie_dist"] <= TIE_TOL, (name, cd["max_tie_dist"], cd["tie_rows"])
    return cd


def _dequant_rel(got, ref_dq, same_rows):
    g = got[same_rows].astype(np.float64)
    r = ref_dq[same_rows].astype(np.float64)
    err = np.abs(g - r) / np.maximum(np.abs(r), 1e-30)
    err[(g == 0) & (r == 0)] = 0.0
    return float(err.max()) if err.size else 0.0


# ----------------------------------------------------------------------------- single linear

def test_single_linear_full_size():
    w, x = inputs.single_linear(0)
    assert w.shape == (1024, 1024) and x.shape == (2048, 1024)
    n_tok = x.shape[0]
    hd, _ = h_g_from_activations(torch.from_numpy(x).cuda())
    h_dev = hd / n_tok
    h64 = x.astype(np.float64).T @ x.astype(np.float64) / n_tok
    ok, fro, worst = ost.h_tolerance_ok(h_dev.cpu().numpy(), h64, H_REL)
    assert ok, (fro, worst)

    cfg = QuantConfig(w_bits=4, group_size=128, sym=False, damp_percent=0.01,
                      ordering_mode="none", semantics="intended")
    f = G.factor_hessian(h_dev, cfg)
    assert f.attempt == 0
    res = G.gptq_sweep(torch.from_numpy(w).cuda(), f.u, f.perm, cfg)
    u = f.u.cpu().numpy()
    perm = f.perm.cpu().numpy()
    assert np.array_equal(perm, np.arange(1024))
    ref32 = og.gptq_sweep(w, u, perm, 4, 128, False, dtype=np.float32, return_pre=True)
    codes = res.codes.cpu().numpy()
    cd = _ties_ok("single_linear_codes_vs_f32_oracle", codes, ref32, perm, 4)
    qmin = oq.qrange(4, False)[0]
    same = ~(codes.astype(np.float32) + qmin != ref32["q"]).any(axis=1)
    dq_err = _dequant_rel(res.dequant.cpu().numpy(), ref32["dequant"], same)
    assert dq_err <= DEQUANT_REL, dq_err
    assert np.array_equal(res.g_idx.cpu().numpy(), ref32["g_idx"])

    # reconstruction error against the float64 oracle (its own float64 factor)
    u64, perm64, att = og.process_hessian_intended(h64, "none", 0.01)
    assert att == 0
    ref64 = og.gptq_sweep(w, u64, perm64, 4, 128, False, dtype=np.float64)
    e_gpu = og.reconstruction_error(w, res.dequant.cpu().numpy(), h64)
    e_ref = og.reconstruction_error(w, ref64["dequant"], h64)
    e_rtn = og.reconstruction_error(w, oq.quantize_dequantize(w, 4, 128), h64)
    report("single_linear_reconstruction", e_gpu=e_gpu, e_oracle64=e_ref, e_rtn=e_rtn,
           rel=abs(e_gpu - e_ref) / e_ref, dequant_rel=dq_err, h_fro=fro, h_worst=worst,
           tie_rows=cd["tie_rows"])
    assert abs(e_gpu - e_ref) <= RECON_REL * e_ref, (e_gpu, e_ref)
    assert e_gpu < e_rtn

    # reference semantics at full size: identity factor, RTN in permuted order, bit-exact
    rcfg = QuantConfig(w_bits=4, group_size=128, sym=False, ordering_mode="none")
    hinv, rperm = process_hessian(h_dev.cpu().numpy(), rcfg)
    assert np.array_equal(hinv, np.eye(1024, dtype=np.float32))
    out = gptq_forward_step(w, hinv, rperm, rcfg)
    assert np.array_equal(out, og.gptq_forward_step_reference(w, rperm, 4, 128, False))


# ----------------------------------------------------------------------------- 7B layer set

TOKENS = 128 * 2048
D_MLP = 11008


@pytest.fixture(scope="module")
def mlp_out_input():
    """The down projection's input: [262144, 11008] bf16 with log-normal
    channel scales (5.8 GB on the device), its channel stds and its H."""
    x, std = LS.synth_activations(TOKENS, D_MLP, 13)
    h = torch.empty((D_MLP, D_MLP), dtype=torch.float32, device="cuda")
    stats.syrk_into(h, x, accumulate=False)
    yield x, std, h
    del x, h
    torch.cuda.empty_cache()


TILES = [(0, 0), (10752, 10752), (2816, 7424), (5376, 10752)]


def _cols64(x, c0):
    return x[:, c0:c0 + 256].float().cpu().numpy().astype(np.float64)


def test_layer_set_h_tiles_at_full_size(mlp_out_input):
    x, _, h = mlp_out_input
    worst_all, fro_all = 0.0, 0.0
    for r0, c0 in TILES:
        xr = _cols64(x, r0)
        xc = xr if c0 == r0 else _cols64(x, c0)
        ref = xr.T @ xc
        got = h[r0:r0 + 256, c0:c0 + 256].cpu().numpy().astype(np.float64)
        bound = np.outer(np.sqrt(np.sum(xr * xr, axis=0)), np.sqrt(np.sum(xc * xc, axis=0)))
        worst = float(np.max(np.abs(got - ref) / bound))
        fro = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        worst_all, fro_all = max(worst_all, worst), max(fro_all, fro)
        assert worst <= H_REL and fro <= H_REL, ((r0, c0), worst, fro)
    # the lower triangle mirrors the upper one exactly
    assert torch.equal(h[10752:, :256], h[:256, 10752:].T)
    report("layer_set_h_tiles", tokens=TOKENS, d=D_MLP, worst_normalized=worst_all, fro=fro_all)


def test_layer_set_g_tiles_at_full_size(mlp_out_input):
    """Qronos cross term G = X^T Xt (the reference's g = x_float^T x_quant)
    with Xt = X + N(0, (0.05 sigma_c)^2)."""
    x, std, _ = mlp_out_input
    xt = LS.perturb_activations(x, std, 0.05, 63)
    g = torch.empty((D_MLP, D_MLP), dtype=torch.float32, device="cuda")
    stats.gemm_tn_into(g, x, xt, accumulate=False)
    worst_all = 0.0
    for r0, c0 in TILES[:3]:
        xr = _cols64(x, r0)
        xc = _cols64(xt, c0)
        ref = xr.T @ xc
        got = g[r0:r0 + 256, c0:c0 + 256].cpu().numpy().astype(np.float64)
        bound = np.outer(np.sqrt(np.sum(xr * xr, 0)), np.sqrt(np.sum(xc * xc, 0)))
        worst = float(np.max(np.abs(got - ref) / bound))
        worst_all = max(worst_all, worst)
        assert worst <= H_REL, ((r0, c0), worst)
    del xt, g
    report("layer_set_g_tiles", tokens=TOKENS, d=D_MLP, worst_normalized=worst_all)


ROW_BLOCKS = np.r_[0:32, 2048:2080, 4064:4096]


def test_layer_set_down_proj_sweep_sampled(mlp_out_input):
    _, _, h = mlp_out_input
    cfg = QuantConfig(w_bits=4, group_size=128, sym=False, damp_percent=0.01,
                      ordering_mode="diag_h", semantics="intended")
    f = G.factor_hessian(h, cfg)
    assert f.attempt == 0
    w = LS.synth_weights([("down", 4096, D_MLP, "mlp_out")], 0.02, 5)["down"]
    res = G.gptq_sweep(w, f.u, f.perm, cfg)
    u = f.u.cpu().numpy()
    perm = f.perm.cpu().numpy()
    rows = torch.from_numpy(ROW_BLOCKS).cuda()
    ref = og.gptq_sweep(w[rows].cpu().numpy(), u, perm, 4, 128, False, dtype=np.float32,
                        return_pre=True)
    codes = res.codes[rows].cpu().numpy()
    cd = _ties_ok("down_proj_sweep_sampled", codes, ref, perm, 4)
    qmin = oq.qrange(4, False)[0]
    same = ~(codes.astype(np.float32) + qmin != ref["q"]).any(axis=1)
    dq_err = _dequant_rel(res.dequant[rows].cpu().numpy(), ref["dequant"], same)
    report("down_proj_sweep_dequant", dequant_rel=dq_err, rows=len(ROW_BLOCKS),
           tie_rows=cd["tie_rows"])
    assert dq_err <= DEQUANT_REL, dq_err
    assert np.array_equal(res.g_idx.cpu().numpy(), ref["g_idx"])


def _recon(w, w_hat, h64):
    """||(W - W^) X^T|| / ||W X^T|| through H = X^T X (BLAS products)."""
    w = np.asarray(w, np.float64)
    d = w - np.asarray(w_hat, np.float64)
    return float(np.sqrt(np.sum((d @ h64) * d) / np.sum((w @ h64) * w)))


def test_layer_set_down_proj_reconstruction_vs_float64(mlp_out_input):
    """The GPU's GPTQ of the sampled down_proj rows against the float64
    oracle with its own float64 factor of the same H: the reconstruction
    errors agree within 1e-3 relative (H itself is checked to 1e-5 above)."""
    _, _, h = mlp_out_input
    cfg = QuantConfig(w_bits=4, group_size=128, sym=False, damp_percent=0.01,
                      ordering_mode="diag_h", semantics="intended")
    f = G.factor_hessian(h, cfg)
    w = LS.synth_weights([("down", 4096, D_MLP, "mlp_out")], 0.02, 5)["down"]
    res = G.gptq_sweep(w, f.u, f.perm, cfg)
    rows = torch.from_numpy(ROW_BLOCKS).cuda()
    ws = w[rows].cpu().numpy()
    h64 = h.cpu().numpy().astype(np.float64)
    u64, perm64, att = og.process_hessian_intended(h64, "diag_h", 0.01)
    assert att == 0
    assert np.array_equal(perm64, f.perm.cpu().numpy())
    ref64 = og.gptq_sweep(ws, u64, perm64, 4, 128, False, dtype=np.float64)
    e_gpu = _recon(ws, res.dequant[rows].cpu().numpy(), h64)
    e_ref = _recon(ws, ref64["dequant"], h64)
    e_rtn = _recon(ws, oq.quantize_dequantize(ws, 4, 128), h64)
    report("down_proj_reconstruction_vs_float64", e_gpu=e_gpu, e_oracle64=e_ref, e_rtn=e_rtn,
           rel=abs(e_gpu - e_ref) / e_ref, rows=len(ROW_BLOCKS))
    assert abs(e_gpu - e_ref) <= RECON_REL * e_ref, (e_gpu, e_ref)
    assert e_gpu < e_rtn


def test_layer_set_down_proj_qronos_sampled(mlp_out_input):
    """Qronos 3-bit: h = Xt^T Xt, g = X^T Xt, the GPU update against the
    float32 oracle given the same factor (U, permutation, damped H); then the
    layer's Qronos objective ||X w - Xt w^|| / ||X w|| on the sampled rows
    against the float64 oracle with its own float64 factor, within 1e-3
    relative."""
    x, std, hxx = mlp_out_input
    xt = LS.perturb_activations(x, std, 0.05, 63)
    hq = torch.empty((D_MLP, D_MLP), dtype=torch.float32, device="cuda")
    stats.syrk_into(hq, xt, accumulate=False)
    g = torch.empty((D_MLP, D_MLP), dtype=torch.float32, device="cuda")
    stats.gemm_tn_into(g, x, xt, accumulate=False)
    del xt
    cfg = QuantConfig(w_bits=3, group_size=128, sym=False, damp_percent=0.01,
                      ordering_mode="diag_h", semantics="intended")
    f = G.factor_hessian(hq, cfg, want_hd=True)
    hq64 = hq.cpu().numpy().astype(np.float64)
    del hq
    assert f.attempt == 0
    w = LS.synth_weights([("down", 4096, D_MLP, "mlp_out")], 0.02, 6)["down"]
    res = Q.qronos_quantize(w, w, None, g, cfg, factor=f)
    rows = torch.from_numpy(ROW_BLOCKS).cuda()
    ws = w[rows].cpu().numpy()
    perm = f.perm.cpu().numpy()
    gn = g.cpu().numpy()
    del g
    shape_only = np.broadcast_to(np.float32(0), gn.shape)  # h: only its shape is checked
    ref = oqn.qronos_intended(ws, ws, shape_only, gn, 3, 128, False, dtype=np.float32,
                              factor=(f.u.cpu().numpy(), perm, f.hd.cpu().numpy()),
                              return_pre=True)
    codes = res.codes[rows].cpu().numpy()
    cd = _ties_ok("down_proj_qronos_sampled", codes, ref, perm, 3)

    # the Qronos objective through the statistics: with d = w^ (Xt) and w (X),
    # ||X w - Xt w^||^2 = w Hxx w - 2 w G w^ + w^ Hq w^  (G = X^T Xt)
    g64 = gn.astype(np.float64)
    del gn, ref
    hxx64 = hxx.cpu().numpy().astype(np.float64)

    def objective(w_hat):
        w64, wh = ws.astype(np.float64), np.asarray(w_hat, np.float64)
        den = np.sum((w64 @ hxx64) * w64)
        num = den - 2.0 * np.sum((w64 @ g64) * wh) + np.sum((wh @ hq64) * wh)
        return float(np.sqrt(max(num, 0.0) / den))

    ref64 = oqn.qronos_intended(ws, ws, hq64, g64, 3, 128, False, ordering_mode="diag_h",
                                dtype=np.float64)
    assert np.array_equal(ref64["perm"], perm)
    e_gpu = objective(res.dequant[rows].cpu().numpy())
    e_ref = objective(ref64["dequant"])
    e_rtn = objective(oq.quantize_dequantize(ws, 3, 128))
    report("down_proj_qronos_rows", rows=len(ROW_BLOCKS), tie_rows=cd["tie_rows"],
           e_gpu=e_gpu, e_oracle64=e_ref, e_rtn=e_rtn, rel=abs(e_gpu - e_ref) / e_ref)
    assert abs(e_gpu - e_ref) <= RECON_REL * e_ref, (e_gpu, e_ref)
    assert e_gpu < e_rtn


# ----------------------------------------------------------------------------- pivoted QR 4096

QR_CASES = [("intended_largest", False, "largest", "intended"),
            ("reference_largest", False, "largest", "reference"),
            ("intended_rankdef_smallest", True, "smallest", "intended"),
            ("intended_rankdef_largest", True, "largest", "intended")]


@pytest.fixture(scope="module")
def qr_fixture(golden_dir):
    path = os.path.join(golden_dir, "qr4096_fixture.npz")
    if not os.path.exists(path):
        pytest.fail("qr4096_fixture.npz is missing: run tests/golden/make_qr4096.py")
    return np.load(path)


@pytest.mark.parametrize("name,rankdef,mode,sem", QR_CASES)
def test_qr_4096_pivots_match_oracle(qr_fixture, name, rankdef, mode, sem):
    """Pivots bit-exact against the oracle up to the first near-tie; the
    count of differing positions is reported.  The first differing position
    counts as a near-tie when the two |R_jj| there lie within 1e-4 relative
    of each other, or both at float32 noise level of the largest |R_jj| (the
    tail of the rank-deficient matrix, where every norm is rounding noise)."""
    import importlib
    BQ = importlib.import_module("jax_gptq_b200.pallas.blocked_pivoted_qr")
    n = int(qr_fixture["n"])
    a = inputs.qr_matrix(1, n, n, rank_deficient=rankdef)
    res = BQ.qrcp(torch.from_numpy(a).cuda(), int(qr_fixture["panel"]), mode, sem)
    perm = res.perm.cpu().numpy().astype(np.int64)
    ref_perm = qr_fixture[name + "_perm"].astype(np.int64)
    ref_d = qr_fixture[name + "_absdiag"].astype(np.float64)
    got_d = np.abs(np.diag(res.work.cpu().numpy())).astype(np.float64)
    mism = np.flatnonzero(perm != ref_perm)
    first = int(mism[0]) if mism.size else n
    noise = 2.0 ** -23 * ref_d.max() * 4
    # up to the first mismatch both follow the same pivots, so their
    # diagonals agree to float32 rounding of the updates; for the
    # rank-deficient matrix only the rank-revealing part is compared (its
    # last 256 steps factor rounding noise)
    upto = min(first, n - 256) if rankdef else first
    scale = np.maximum(ref_d[:upto], noise)
    d_rel = float(np.max(np.abs(got_d[:upto] - ref_d[:upto]) / scale)) if upto else 0.0
    near_tie = True
    if mism.size:
        a_j, b_j = ref_d[first], got_d[first]
        near_tie = bool(abs(a_j - b_j) <= 1e-4 * max(a_j, b_j) or max(a_j, b_j) <= 64 * noise
                        or (rankdef and first >= n - 256))
    srt = np.sort(got_d)[::-1]
    fields = {"n": n, "first_mismatch": first, "mismatches": int(mism.size),
              "diag_rel_before_first": d_rel, "near_tie_at_first": near_tie,
              "absdiag_sorted_3836_3844": [float(v) for v in srt[3836:3844]],
              "absdiag_sorted_last4": [float(v) for v in srt[-4:]],
              "oracle_absdiag_3836_3844": [float(v) for v in np.sort(ref_d)[::-1][3836:3844]]}
    if sem == "intended":
        resid = BQ._residual_dev(torch.from_numpy(a).cuda(), res)
        fields["residual"] = resid
        fields.update(BQ.numerical_rank(res.work))
        assert resid <= 1e-5, resid
    report("qr4096_" + name, **fields)
    assert near_tie, fields
    if mode == "largest":
        assert d_rel <= 1e-3, fields
    else:
        # smallest-first pivoting is not rank revealing: the later diagonal
        # entries carry amplified rounding, so only pivots and residual count
        assert first >= n - 256, fields
    if rankdef and mode == "largest":
        # rank-revealing order: the pivots agree with the oracle over all
        # 3840 independent columns; the 256 dependent ones come last
        assert first >= n - 256, fields
        assert fields["numerical_rank"] == n - 256, fields
