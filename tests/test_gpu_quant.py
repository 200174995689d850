"""GPU parity of the quantization path through the C ABI against the oracle.

Bit-exact: RTN codes / dequant (reference semantics), act-order permutation,
the sweep with U = I.  Tolerances (written per test): H within 1e-5
relative; the inverse-Cholesky factor within 2e-3 relative Frobenius of the
float64 oracle (float32 Cholesky of a damped Hessian); intended-semantics
reconstruction error within 1e-3 relative of the float64 oracle's.
"""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import QuantConfig, gptq_forward_step, h_g_from_activations
from jax_gptq_b200 import process_hessian, qronos_single_layer_update_ref, quantize_dequantize
from jax_gptq_b200 import gptq_ref as G
from jax_gptq_b200 import qronos_ref as Q
from jax_gptq_b200 import quant as RQ
from oracle import gptq as og
from oracle import inputs
from oracle import qronos as oqn
from oracle import quant as oq
from oracle import stats as ost

from parity import TIE_TOL, code_diffs, report


def _golden(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_rtn_bit_exact_vs_reference_vectors(golden_dir):
    d = _golden(golden_dir, "rtn_golden.npz")
    names = [k[:-2] for k in d.files if k.startswith("rtn_") and k.endswith("_w")]
    for name in names:
        bits, gs, sym = (int(v) for v in d[name + "_cfg"])
        cfg = QuantConfig(w_bits=bits, group_size=gs, sym=bool(sym))
        out = quantize_dequantize(d[name + "_w"], cfg)
        assert isinstance(out, np.ndarray)
        assert np.array_equal(out, d[name + "_out"]), name


@pytest.mark.parametrize("shape,bits,gs,sym", [
    ((256, 1024), 4, 128, False), ((64, 4096), 3, 128, False), ((128, 512), 4, 64, True),
    ((33, 384), 8, 32, False), ((7, 40), 2, 4, True), ((1, 11008), 4, 128, False)])
def test_rtn_codes_scales_zeros_match_oracle(shape, bits, gs, sym):
    rng = np.random.default_rng(sum(shape) + bits)
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    w[0, :gs] = 0.0  # constant group -> scale floor
    dq, q, s, z = oq.rtn(w, bits, gs, sym)
    res = RQ.rtn(w, QuantConfig(w_bits=bits, group_size=gs, sym=sym))
    qmin = oq.qrange(bits, sym)[0]
    assert np.array_equal(res.dequant.cpu().numpy(), dq)
    assert np.array_equal(res.codes.cpu().numpy().astype(np.float32) + qmin, q)
    assert np.array_equal(res.scales.cpu().numpy(), s)
    assert np.array_equal(res.zeros.cpu().numpy(), z)


@pytest.mark.parametrize("case", ["none", "diag", "diag_sym3"])
def test_gptq_reference_semantics_bit_exact(golden_dir, case):
    d = _golden(golden_dir, "gptq_golden.npz")
    p = f"gptq_{case}"
    bits, gs, sym, diag = (int(v) for v in d[p + "_cfg"])
    cfg = QuantConfig(w_bits=bits, group_size=gs, sym=bool(sym),
                      ordering_mode="diag_h" if diag else "none")
    x = d[p + "_x"]
    h, g = h_g_from_activations(x)
    hinv, perm = process_hessian(h, cfg)
    assert np.array_equal(hinv, np.eye(x.shape[1]))
    assert np.array_equal(perm, d[p + "_perm"])
    out = gptq_forward_step(d[p + "_w"], hinv, perm, cfg)
    assert np.array_equal(out, d[p + "_out"])
    # the sweep kernel with U = I gives the same bits
    sw = G.gptq_sweep(d[p + "_w"], hinv, perm, cfg)
    assert np.array_equal(sw.dequant.cpu().numpy(), d[p + "_out"])
    qr = qronos_single_layer_update_ref(d[p + "_w"], d[p + "_w"], h, g, cfg)
    assert np.array_equal(qr, d[p + "_qronos"])


def test_act_order_perm_matches_oracle_with_ties():
    rng = np.random.default_rng(5)
    for d in (7, 300, 4096):
        diag = rng.integers(0, 5, size=d).astype(np.float32)  # many ties
        h = np.diag(diag).astype(np.float32)
        dev = torch.from_numpy(h).cuda()
        perm = G.act_order_perm(dev, "diag_h").cpu().numpy()
        assert np.array_equal(perm, og.act_order_perm(h, "diag_h"))


def test_sgemm_matches_numpy():
    from jax_gptq_b200 import _arrays as A
    from jax_gptq_b200 import _lib
    rng = np.random.default_rng(1)
    for (M, N, K, ta, tb) in [(130, 70, 33, 0, 0), (64, 200, 129, 1, 0), (257, 129, 65, 0, 1),
                              (5, 3, 700, 1, 1)]:
        a = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
        b = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
        c = rng.standard_normal((M, N)).astype(np.float32)
        ref = 0.5 * ((a.T if ta else a).astype(np.float64) @ (b.T if tb else b)) + 2.0 * c
        at, bt, ct = (torch.from_numpy(v).cuda() for v in (a, b, c))
        _lib.call("gq_sgemm", ta, tb, M, N, K, 0.5, A.ptr(at), at.shape[1], A.ptr(bt), bt.shape[1],
                  2.0, A.ptr(ct), N, 0, A.stream())
        assert np.allclose(ct.cpu().numpy(), ref, rtol=1e-4, atol=1e-4)


def test_h_fp32_matches_oracle_within_1e5():
    w, x = inputs.single_linear(0, m=64, n=1024, tokens=2048)
    h, g = h_g_from_activations(x)
    h64, _ = ost.h_g_from_activations(x)
    ok, fro, worst = ost.h_tolerance_ok(h, h64, 1e-5)
    assert ok, (fro, worst)
    rng = np.random.default_rng(3)
    xf = x + rng.standard_normal(x.shape).astype(np.float32)
    h2, g2 = h_g_from_activations(x, xf)
    _, g64 = ost.h_g_from_activations(x, xf)
    assert np.linalg.norm(g2 - g64) / np.linalg.norm(g64) <= 1e-5


@pytest.mark.parametrize("ordering", ["none", "diag_h"])
def test_hessian_factor_matches_oracle(ordering):
    w, x = inputs.single_linear(0, m=64, n=512, tokens=2048)
    h = (x.astype(np.float64).T @ x / x.shape[0]).astype(np.float32)
    cfg = QuantConfig(ordering_mode=ordering, semantics="intended")
    f = G.factor_hessian(h, cfg, want_hd=True)
    u64, perm64, att = og.process_hessian_intended(h, ordering, 0.01)
    assert f.attempt == att == 0
    assert np.array_equal(f.perm.cpu().numpy(), perm64)
    u = f.u.cpu().numpy().astype(np.float64)
    assert np.allclose(np.tril(u, -1), 0.0)
    assert np.linalg.norm(u - u64) / np.linalg.norm(u64) < 2e-3
    hd = f.hd.cpu().numpy().astype(np.float64)
    ident = u @ hd @ u.T          # U Hd U^T = I  <=>  U^T U = Hd^-1
    assert np.abs(ident - np.eye(512)).max() < 5e-3


@pytest.mark.parametrize("d", [128, 200, 384, 1000, 1030])
def test_hessian_factor_sizes(d):
    """Recursive inverse Cholesky: partial last leaf (200, 1000, 1030) and a
    leading dimension that is not a multiple of 4 (1030: CUDA-core GEMMs)."""
    rng = np.random.default_rng(d)
    x = rng.standard_normal((2 * d, d)).astype(np.float32) * rng.uniform(0.2, 3.0, d).astype(np.float32)
    h = (x.astype(np.float64).T @ x / x.shape[0]).astype(np.float32)
    cfg = QuantConfig(ordering_mode="diag_h", semantics="intended")
    f = G.factor_hessian(h, cfg, want_hd=True)
    u64, perm64, att = og.process_hessian_intended(h, "diag_h", 0.01)
    assert f.attempt == att == 0
    u = f.u.cpu().numpy().astype(np.float64)
    assert np.array_equal(np.tril(u, -1), np.zeros_like(u))
    assert np.linalg.norm(u - u64) / np.linalg.norm(u64) < 2e-3
    hd = f.hd.cpu().numpy().astype(np.float64)
    assert np.abs(u @ hd @ u.T - np.eye(d)).max() < 5e-3


def test_hessian_factor_retries_damping_on_indefinite_input():
    # a negative-definite direction that 1% damping cannot fix but 100x can
    n = 128
    h = np.eye(n, dtype=np.float32)
    h[5, 5] = -0.5
    cfg = QuantConfig(semantics="intended", damp_percent=0.01)
    f = G.factor_hessian(h, cfg)
    _, _, att = og.process_hessian_intended(h, "none", 0.01)
    assert f.attempt == att and f.attempt >= 1


def test_gptq_intended_reconstruction_matches_oracle():
    w, x = inputs.single_linear(0, m=256, n=1024, tokens=2048)
    h = (x.astype(np.float64).T @ x / x.shape[0])
    cfg = QuantConfig(ordering_mode="diag_h", semantics="intended")
    res = G.gptq_quantize(w, h.astype(np.float32), cfg)
    u64, perm64, _ = og.process_hessian_intended(h, "diag_h", 0.01)
    ref = og.gptq_sweep(w, u64, perm64, 4, 128, False, dtype=np.float64)
    e_gpu = og.reconstruction_error(w, res.dequant.cpu().numpy(), h)
    e_ref = og.reconstruction_error(w, ref["dequant"], h)
    e_rtn = og.reconstruction_error(w, oq.quantize_dequantize(w, 4, 128), h)
    assert abs(e_gpu - e_ref) <= 1e-3 * e_ref, (e_gpu, e_ref)
    assert e_gpu < e_rtn
    codes = res.codes.cpu().numpy().astype(np.float32)
    agree = np.mean(codes == ref["q"])
    assert agree > 0.95, agree
    assert np.array_equal(res.g_idx.cpu().numpy(), ref["g_idx"])


def test_qronos_intended_matches_oracle():
    w, x = inputs.single_linear(2, m=128, n=512, tokens=2048)
    rng = np.random.default_rng(2)
    xt = (x + rng.standard_normal(x.shape).astype(np.float32) * 0.05 * x.std(0)).astype(np.float32)
    h, g = ost.h_g_from_activations(xt, x)
    cfg = QuantConfig(w_bits=3, semantics="intended")
    out = qronos_single_layer_update_ref(w, w, h.astype(np.float32), g.astype(np.float32), cfg)
    ref = oqn.qronos_intended(w, w, h, g, 3, 128, False)

    def err(w_hat):
        return np.linalg.norm(x.astype(np.float64) @ w.T - xt.astype(np.float64) @ w_hat.T)
    e_gpu, e_ref = err(out), err(ref["dequant"])
    assert abs(e_gpu - e_ref) <= 1e-3 * e_ref, (e_gpu, e_ref)
    assert e_gpu < err(oq.quantize_dequantize(w, 3, 128))


@pytest.mark.parametrize("m,n,bits,g,sym", [(512, 2048, 4, 128, False), (300, 1536, 3, 256, False),
                                            (256, 1536, 4, 384, False), (200, 1000, 4, 8, False),
                                            (384, 1536, 4, 128, True), (256, 1024, 3, 64, True),
                                            (256, 1024, 2, 128, False), (256, 1024, 8, 32, False)])
def test_sweep_codes_match_float32_oracle_up_to_rounding_ties(m, n, bits, g, sym):
    """The GPU sweep against the float32 oracle sweep on the same factor U and
    permutation: the two differ only in the order of float32 additions (lazy
    updates batched two-level on the GPU, BLAS in the oracle).  Rows are
    independent, so in every row the first code that differs must be a
    rounding tie: the oracle's unrounded value within TIE_TOL of a half step.
    Later codes of such a row follow from the flipped error and are counted,
    not checked.  g = 384 takes the 128-column fallback of the far update;
    symmetric grids and 2- and 8-bit codes are covered too."""
    rng = np.random.default_rng(m + n + g)
    w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    x = (rng.standard_normal((2 * n, n)) * rng.lognormal(0, 1, n)).astype(np.float32)
    h = x.T.astype(np.float64) @ x
    cfg = QuantConfig(w_bits=bits, group_size=g, sym=sym, ordering_mode="diag_h",
                      semantics="intended")
    f = G.factor_hessian(h.astype(np.float32), cfg)
    u = f.u.cpu().numpy()
    perm = f.perm.cpu().numpy()
    res = G.gptq_sweep(torch.from_numpy(w).cuda(), f.u, f.perm, cfg)
    ref = og.gptq_sweep(w, u, perm, bits, g, sym, dtype=np.float32, return_pre=True)
    codes_p = res.codes.cpu().numpy().astype(np.float32)[:, perm]   # permuted order
    qmin = oq.qrange(bits, sym)[0]
    ref_p = ref["q"][:, perm]
    cd = code_diffs(codes_p + qmin, ref_p, ref["pre"])
    report(f"sweep_ties_{m}x{n}_b{bits}_g{g}_s{int(sym)}", rows=m, tie_rows=cd["tie_rows"],
           codes_differing=cd["codes_differing"], max_tie_dist=cd["max_tie_dist"])
    # TIE_TOL is about ten float32 ulps of a 4-bit code; a finer grid divides
    # the same float32 differences of w by a proportionally smaller scale
    tol = TIE_TOL * max(1, 2 ** (bits - 4))
    assert cd["max_tie_dist"] <= tol, (cd["max_tie_dist"], cd["tie_rows"])
    # and the flips are rare
    assert cd["tie_rows"] <= 0.05 * m, (cd["tie_rows"], cd["codes_differing"])
    assert np.array_equal(res.g_idx.cpu().numpy(), ref["g_idx"])


@pytest.mark.parametrize("m,n,g", [(300, 1152, 128), (300, 1000, 8), (200, 1536, 256),
                                   (97, 640, 32), (640, 512, 64)])
def test_sweep_block_step_forms_agree(m, n, g):
    """The block step's forms (one warp per 32 rows; four warps per 32 rows
    with 1, 2 or 4 row groups sharing one CTA's staged U band) apply the same
    updates in the same order to every row, so they give the same bits, also
    for ragged row counts (a partly filled last CTA) and ragged blocks."""
    from jax_gptq_b200 import _lib
    rng = np.random.default_rng(m + n + g)
    x = (rng.standard_normal((2 * n, n)) * rng.lognormal(0, 1, n)).astype(np.float32)
    cfg = QuantConfig(w_bits=4, group_size=g, ordering_mode="diag_h", semantics="intended")
    f = G.factor_hessian((x.T @ x).astype(np.float32), cfg)
    w = torch.from_numpy((rng.standard_normal((m, n)) * 0.02).astype(np.float32)).cuda()
    lib = _lib.lib()
    outs = {}
    try:
        for r in (-1, 1, 2, 4):
            assert lib.gq_set_sweep_row_groups(r) == 0
            outs[r] = G.gptq_sweep(w, f.u, f.perm, cfg)
    finally:
        lib.gq_set_sweep_row_groups(0)
    for r in (1, 2, 4):
        for key in ("dequant", "codes", "scales", "zeros", "g_idx"):
            assert torch.equal(getattr(outs[-1], key), getattr(outs[r], key)), (r, key)


def test_sweep_single_warp_and_four_warp_block_steps_agree():
    """Grids larger than one wave of four-group CTAs take the single-warp
    block step; rows are independent, so sweeping halves of the rows (four
    warps per 32 rows, four row groups per CTA) must reproduce the whole
    sweep bit for bit."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    m, n = 32 * (4 * sms + 8), 512
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((2 * n, n)) * rng.lognormal(0, 1, n)).astype(np.float32)
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    f = G.factor_hessian((x.T @ x).astype(np.float32), cfg)
    w = torch.from_numpy((rng.standard_normal((m, n)) * 0.02).astype(np.float32)).cuda()
    whole = G.gptq_sweep(w, f.u, f.perm, cfg)
    h = m // 2
    top, bot = G.gptq_sweep(w[:h], f.u, f.perm, cfg), G.gptq_sweep(w[h:], f.u, f.perm, cfg)
    for key in ("dequant", "codes", "scales", "zeros"):
        both = torch.cat([getattr(top, key), getattr(bot, key)])
        assert torch.equal(getattr(whole, key), both), key


@pytest.mark.parametrize("bits,g,sym", [(3, 128, False), (4, 64, True)])
def test_qronos_codes_match_float32_oracle_up_to_rounding_ties(bits, g, sym):
    """Qronos on the GPU against the float32 oracle given the same factor
    (U, permutation, damped H): the first code that differs in a row must be
    a rounding tie of the oracle's unrounded value (within TIE_TOL of a half
    step); later codes of that row follow from the flip."""
    m, n = 256, 1024
    rng = np.random.default_rng(21)
    x = (rng.standard_normal((2 * n, n)) * rng.lognormal(0, 1, n)).astype(np.float32)
    xt = (x + rng.standard_normal(x.shape).astype(np.float32) * 0.05 * x.std(0)).astype(np.float32)
    h, gm = ost.h_g_from_activations(xt, x)
    h, gm = h.astype(np.float32), gm.astype(np.float32)
    w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    cfg = QuantConfig(w_bits=bits, group_size=g, sym=sym, ordering_mode="diag_h",
                      semantics="intended")
    f = G.factor_hessian(h, cfg, want_hd=True)
    res = Q.qronos_quantize(torch.from_numpy(w).cuda(), torch.from_numpy(w).cuda(), None,
                            torch.from_numpy(gm).cuda(), cfg, factor=f)
    perm = f.perm.cpu().numpy()
    ref = oqn.qronos_intended(w, w, h, gm, bits, g, sym, dtype=np.float32,
                              factor=(f.u.cpu().numpy(), perm, f.hd.cpu().numpy()),
                              return_pre=True)
    qmin = oq.qrange(bits, sym)[0]
    got_p = res.codes.cpu().numpy().astype(np.float32)[:, perm] + qmin
    ref_p = ref["q"][:, perm]
    cd = code_diffs(got_p, ref_p, ref["pre"])
    report(f"qronos_ties_256x1024_b{bits}_g{g}_s{int(sym)}", rows=m, tie_rows=cd["tie_rows"],
           codes_differing=cd["codes_differing"], max_tie_dist=cd["max_tie_dist"])
    # Qronos' first step solves with the damped H, which amplifies the float32
    # ordering differences of its inputs beyond the plain sweep's: measured
    # first differences up to 2.8e-5 of a half step (symmetric 4-bit)
    assert cd["max_tie_dist"] <= 4 * TIE_TOL, (cd["max_tie_dist"], cd["tie_rows"])
    assert cd["tie_rows"] <= 0.1 * m, (cd["tie_rows"], cd["codes_differing"])
    # the objective ||X w - Xt w^|| / ||X w|| within 1e-3 of the float64 oracle's
    ref64 = oqn.qronos_intended(w, w, h.astype(np.float64), gm.astype(np.float64), bits, g, sym,
                                ordering_mode="diag_h", dtype=np.float64)
    x64, xt64 = x.astype(np.float64), xt.astype(np.float64)
    target = x64 @ w.astype(np.float64).T

    def objective(w_hat):
        out = xt64 @ np.asarray(w_hat, np.float64).T
        return float(np.linalg.norm(target - out) / np.linalg.norm(target))

    e_gpu, e_ref = objective(res.dequant.cpu().numpy()), objective(ref64["dequant"])
    report(f"qronos_objective_256x1024_b{bits}_g{g}_s{int(sym)}", e_gpu=e_gpu, e_oracle64=e_ref,
           rel=abs(e_gpu - e_ref) / e_ref)
    assert abs(e_gpu - e_ref) <= 1e-3 * e_ref, (e_gpu, e_ref)


def test_factor_attempt_replays_from_a_cuda_graph():
    """The factor's side-stream fork joins a stream capture through its events:
    after one call on the capture stream (which creates that stream's side
    stream), the attempt captured in a CUDA graph and replayed gives the eager
    factor bit for bit."""
    rng = np.random.default_rng(21)
    d = 1152
    x = torch.from_numpy(rng.standard_normal((2 * d, d)).astype(np.float32)).cuda()
    h = x.T @ x
    cfg = QuantConfig(ordering_mode="diag_h", semantics="intended")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        eager, st = G.factor_hessian_attempt0(h, cfg)
        eager_u = eager.u.clone()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    assert st.item() == 0
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        cap, cst = G.factor_hessian_attempt0(h, cfg)
    cap.u.zero_()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    assert cst.item() == 0
    assert torch.equal(cap.u, eager_u)
    assert torch.equal(cap.perm, eager.perm)
