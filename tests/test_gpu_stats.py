"""GPU parity of H / G accumulation (tcgen05 bf16 path and fp32 path).

Tolerance (from the hot-path contract): ``||dH||_F / ||H||_F <= 1e-5`` and
``|dH_ij| <= 1e-5 sqrt(H_ii H_jj)`` against a float64 oracle on the same
bf16-representable inputs (bf16 x bf16 products are exact in fp32, so only
the accumulation order differs).
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import _arrays as A
from jax_gptq_b200 import _lib
from jax_gptq_b200 import h_g_from_activations
from jax_gptq_b200.stats import HessianAccumulator
from oracle import stats as ost


def _bf16(rng, shape, scale=None):
    x = rng.standard_normal(shape).astype(np.float32)
    if scale is not None:
        x *= scale
    t = torch.from_numpy(x).to(torch.bfloat16)
    return t, t.float().numpy()


def _status():
    v = ctypes.c_int(-1)
    _lib.call("gq_device_status", ctypes.byref(v), 1, A.stream())
    return v.value


@pytest.mark.parametrize("tokens,d", [(64, 128), (1000, 296), (2048, 1024), (777, 520),
                                      (4096, 2048)])
def test_syrk_bf16_matches_oracle(tokens, d):
    rng = np.random.default_rng(tokens + d)
    scale = rng.lognormal(0, 1, d).astype(np.float32)
    xt, xn = _bf16(rng, (tokens, d), scale)
    h, _ = h_g_from_activations(xt.cuda())
    assert _status() == 0
    h64, _ = ost.h_g_from_activations(xn)
    ok, fro, worst = ost.h_tolerance_ok(h.cpu().numpy(), h64, 1e-5)
    assert ok, (fro, worst)
    hn = h.cpu().numpy()
    assert np.array_equal(hn, hn.T)


@pytest.mark.parametrize("tokens,da,db", [(512, 256, 640), (1000, 392, 136), (2048, 1024, 1024)])
def test_gemm_tn_bf16_matches_oracle(tokens, da, db):
    rng = np.random.default_rng(7 + tokens)
    xa, xa_n = _bf16(rng, (tokens, da))
    xb, xb_n = _bf16(rng, (tokens, db))
    g = torch.empty((da, db), dtype=torch.float32, device="cuda")
    xa_d, xb_d = xa.cuda(), xb.cuda()  # keep both alive across the call
    _lib.call("gq_gemm_tn_bf16", A.ptr(xa_d), da, A.ptr(xb_d), db, tokens, da, db,
              A.ptr(g), db, 0, A.stream())
    assert _status() == 0
    ref = xa_n.astype(np.float64).T @ xb_n.astype(np.float64)
    rel = np.linalg.norm(g.cpu().numpy() - ref) / np.linalg.norm(ref)
    assert rel <= 1e-5, rel


def test_streamed_accumulation_equals_one_shot():
    rng = np.random.default_rng(11)
    d = 384
    acc = HessianAccumulator(d, with_cross=True)
    parts, partsf = [], []
    for n in (300, 512, 64):
        xt, xn = _bf16(rng, (n, d))
        xf, xfn = _bf16(rng, (n, d))
        acc.add(xt.cuda(), xf.cuda())
        parts.append(xn)
        partsf.append(xfn)
    x = np.concatenate(parts)
    xf = np.concatenate(partsf)
    h64, g64 = ost.h_g_from_activations(x, xf)
    assert ost.h_tolerance_ok(acc.h.cpu().numpy(), h64, 1e-5)[0]
    assert np.linalg.norm(acc.g.cpu().numpy() - g64) / np.linalg.norm(g64) <= 1e-5
    assert acc.tokens == x.shape[0]


def test_cross_term_follows_reference_orientation():
    """stats.py:17: g = x_float^T x_quant."""
    rng = np.random.default_rng(12)
    xq, xqn = _bf16(rng, (256, 128))
    xf, xfn = _bf16(rng, (256, 128))
    h, g = h_g_from_activations(xq.cuda(), xf.cuda())
    ref = xfn.astype(np.float64).T @ xqn
    assert np.linalg.norm(g.cpu().numpy() - ref) / np.linalg.norm(ref) <= 1e-5


def test_zero_tokens_gives_zero_h():
    x = torch.zeros((0, 64), dtype=torch.bfloat16, device="cuda")
    h = torch.full((64, 64), 3.0, device="cuda")
    _lib.call("gq_syrk_bf16", A.ptr(x) if x.numel() else ctypes.c_void_p(256), 0, 64, 64, A.ptr(h),
              64, 0, A.stream())
    assert float(h.abs().max()) == 0.0


@pytest.mark.parametrize("tokens,d,chunk", [(4096, 520, 1024), (6144, 1024, 2048), (5000, 384, 1024)])
def test_token_chunked_launches_equal_one_launch(tokens, d, chunk):
    """Splitting the tokens at multiples of 1024 continues the same float32
    running sum: H and G are bit-identical to a single launch (the tail chunk
    may be ragged)."""
    from jax_gptq_b200 import stats
    rng = np.random.default_rng(tokens + chunk)
    xq = _bf16(rng, (tokens, d))[0].cuda()
    xf = _bf16(rng, (tokens, d))[0].cuda()
    h1 = torch.empty((d, d), device="cuda")
    h2 = torch.empty((d, d), device="cuda")
    g1 = torch.empty((d, d), device="cuda")
    g2 = torch.empty((d, d), device="cuda")
    stats.syrk_into(h1, xq, accumulate=False)
    stats.syrk_into(h2, xq, accumulate=False, token_chunk=chunk)
    stats.gemm_tn_into(g1, xf, xq, accumulate=False)
    stats.gemm_tn_into(g2, xf, xq, accumulate=False, token_chunk=chunk)
    assert _status() == 0
    assert torch.equal(h1, h2)
    assert torch.equal(g1, g2)
    # a streamed accumulator over 1024-multiple batches is the same sum again
    acc = HessianAccumulator(d, with_cross=True)
    for t0 in range(0, tokens, chunk):
        acc.add(xq[t0:t0 + chunk], xf[t0:t0 + chunk])
    assert torch.equal(acc.h, h1)
    assert torch.equal(acc.g, g1)


def test_token_chunk_must_be_a_multiple_of_1024():
    from jax_gptq_b200 import stats
    x = torch.zeros((4096, 64), dtype=torch.bfloat16, device="cuda")
    h = torch.empty((64, 64), device="cuda")
    for bad in (1000, 512):
        with pytest.raises(ValueError):
            stats.syrk_into(h, x, accumulate=False, token_chunk=bad)


@pytest.mark.parametrize("tokens,d,sym", [(4096, 1000, True), (2048, 520, True), (3000, 392, False)])
def test_pair_and_single_cta_statistics_agree(tokens, d, sym):
    """CTA-pair (cta_group::2, 256 x 256 tiles) and one-CTA (128 x 256) forms of
    the bf16 statistics kernels give the same bits."""
    from jax_gptq_b200 import stats
    rng = np.random.default_rng(tokens + d)
    xq = _bf16(rng, (tokens, d))[0].cuda()
    xf = _bf16(rng, (tokens, d))[0].cuda()
    out = []
    lib = _lib.lib()
    try:
        for pair in (1, 0):
            assert lib.gq_set_pair_kernels(pair) == 0
            c = torch.empty((d, d), device="cuda")
            if sym:
                stats.syrk_into(c, xq, accumulate=False)
            else:
                stats.gemm_tn_into(c, xf, xq, accumulate=False)
            out.append(c)
    finally:
        lib.gq_set_pair_kernels(1)
    assert _status() == 0
    assert torch.equal(out[0], out[1])
