"""Layer-set drivers on the GPU: the concurrent per-group schedule (each input
group's factor + sweep on its own stream, first damping attempt without a host
synchronization) must give exactly the sequential result, and a group whose
first attempt fails must be redone through the retrying path."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import layerset as LS
from jax_gptq_b200.config import QuantConfig
from jax_gptq_b200.gptq_ref import factor_hessian, factor_hessian_attempt0, gptq_sweep

SHAPES = [("q", 256, 512, "a"), ("k", 64, 512, "a"), ("o", 200, 384, "b"), ("d", 96, 640, "c")]


def _setup(seed=0, tokens=2048):
    weights = LS.synth_weights(SHAPES, 0.02, seed)
    dims = LS.group_dims(SHAPES)
    inputs = {g: LS.synth_activations(tokens, d, seed + 10 + i)[0] for i, (g, d) in enumerate(dims.items())}
    return weights, inputs


def _assert_same(a, b):
    for name, _m, _n, _g in SHAPES:
        for field in ("dequant", "codes", "scales", "zeros", "g_idx", "perm"):
            assert getattr(a[name], field).equal(getattr(b[name], field)), (name, field)


def test_concurrent_gptq_equals_sequential():
    weights, inputs = _setup()
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    seq, _ = LS.quantize_layer_gptq(weights, inputs, cfg, SHAPES, concurrent=False)
    for _ in range(2):
        con, _ = LS.quantize_layer_gptq(weights, inputs, cfg, SHAPES)
        torch.cuda.synchronize()
        _assert_same(con, seq)


def test_concurrent_qronos_equals_sequential():
    weights, inputs = _setup(1)
    xq = {g: LS.perturb_activations(x, LS.synth_activations(8, x.shape[1], 99)[1], 0.05, 5 + i)
          for i, (g, x) in enumerate(inputs.items())}
    cfg = QuantConfig(w_bits=3, group_size=128, ordering_mode="diag_h", semantics="intended")
    seq, _ = LS.quantize_layer_qronos(weights, inputs, xq, cfg, SHAPES, concurrent=False)
    con, _ = LS.quantize_layer_qronos(weights, inputs, xq, cfg, SHAPES)
    torch.cuda.synchronize()
    _assert_same(con, seq)


def test_failed_first_attempt_is_redone():
    n = 256
    h = np.eye(n, dtype=np.float32)
    h[5, 5] = -0.5  # 1% damping cannot fix this direction, 100x can
    h = torch.from_numpy(h).cuda()
    cfg = QuantConfig(semantics="intended", damp_percent=0.01)
    _, status = factor_hessian_attempt0(h, cfg)
    assert status.item() != 0
    w = torch.randn((64, n), device="cuda") * 0.02
    calls = []

    def work(grp, hh):
        f, st = factor_hessian_attempt0(hh, cfg)
        return st, gptq_sweep(w, f.u, f.perm, cfg)

    def redo(grp, hh):
        calls.append(grp)
        f = factor_hessian(hh, cfg)
        return gptq_sweep(w, f.u, f.perm, cfg)

    good = torch.eye(n, device="cuda")
    hs = {"bad": h, "good": good}
    out = LS._run_groups_concurrently({"bad": n, "good": n}, lambda g, _chunk: hs[g], work, redo)
    assert calls == ["bad"]
    f = factor_hessian(h, cfg)
    assert f.attempt >= 1
    ref = gptq_sweep(w, f.u, f.perm, cfg)
    assert out["bad"].dequant.equal(ref.dequant)
    fg = factor_hessian(good, cfg)
    assert out["good"].dequant.equal(gptq_sweep(w, fg.u, fg.perm, cfg).dequant)


def test_host_buffer_driver_equals_device_driver():
    """Host buffers in, host results out (chunked transfers, H accumulated per
    chunk, largest group first): the same bits as the device-resident path."""
    shapes = SHAPES
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    weights = LS.synth_weights(shapes, 0.02, 3)
    inputs = {g: LS.synth_activations(3000, d, 40 + i)[0]
              for i, (g, d) in enumerate(LS.group_dims(shapes).items())}
    old = LS.HOST_TOKEN_CHUNK
    LS.HOST_TOKEN_CHUNK = 1024
    try:
        w_host = {k: v.cpu().pin_memory() for k, v in weights.items()}
        x_host = {k: v.cpu().pin_memory() for k, v in inputs.items()}
        got, nbytes = LS.quantize_layer_gptq_host(w_host, x_host, cfg, shapes)
    finally:
        LS.HOST_TOKEN_CHUNK = old
    torch.cuda.synchronize()
    ref, _ = LS.quantize_layer_gptq(weights, inputs, cfg, shapes, concurrent=False)
    assert set(got) == set(ref)
    for name, (codes, scales, zeros, g_idx, perm) in got.items():
        r = ref[name]
        assert torch.equal(codes, r.codes.cpu()), name
        assert torch.equal(scales, r.scales.cpu()), name
        assert torch.equal(zeros, r.zeros.cpu()), name
        assert torch.equal(perm, r.perm.cpu()), name
    assert nbytes["h2d"] > 0 and nbytes["d2h"] > 0


def _two_step_and_fused(x, cfg):
    from jax_gptq_b200 import stats
    from jax_gptq_b200.gptq_ref import factor_from_activations_attempt0
    d = x.shape[1]
    h = torch.empty((d, d), device="cuda")
    stats.syrk_into(h, x, accumulate=False)
    f0, st0 = factor_hessian_attempt0(h, cfg)
    side = torch.cuda.Stream()
    f1, st1 = factor_from_activations_attempt0(x, cfg, side, LS.RESERVED_SMS)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    return (f0, st0.item()), (f1, st1.item())


@pytest.mark.parametrize("tokens,d,ordering", [
    (3000, 136, "diag_h"), (2048, 520, "diag_h"), (2048, 520, "none"), (4096, 1024, "diag_h"),
    (5000, 2304, "diag_h"), (1000, 64, "diag_h")])
def test_factor_from_activations_matches_two_step_path(tokens, d, ordering):
    """The factor formed straight from X (H in act-order blocks, leading block
    first, rec(A11) overlapping the rest) equals SYRK -> act order -> factor
    bit for bit: every element of the permuted H is the same tile arithmetic."""
    x = LS.synth_activations(tokens, d, tokens + d)[0]
    cfg = QuantConfig(ordering_mode=ordering, semantics="intended")
    (f0, st0), (f1, st1) = _two_step_and_fused(x, cfg)
    assert st0 == 0 and st1 == 0
    assert torch.equal(f0.perm, f1.perm)
    assert torch.equal(f0.u, f1.u)


def test_factor_from_activations_single_cta_statistics():
    from jax_gptq_b200 import _lib
    x = LS.synth_activations(2048, 776, 3)[0]
    cfg = QuantConfig(ordering_mode="diag_h", semantics="intended")
    lib = _lib.lib()
    try:
        assert lib.gq_set_pair_kernels(0) == 0
        (f0, st0), (f1, st1) = _two_step_and_fused(x, cfg)
    finally:
        lib.gq_set_pair_kernels(1)
    assert st0 == 0 and st1 == 0
    assert torch.equal(f0.u, f1.u) and torch.equal(f0.perm, f1.perm)


def test_factor_from_activations_reports_a_failed_attempt():
    x = LS.synth_activations(2048, 384, 4)[0]
    x[:, 17] = 0  # a dead feature: zero pivot without damping
    cfg = QuantConfig(ordering_mode="diag_h", semantics="intended", damp_percent=0.0)
    (_, st0), (_, st1) = _two_step_and_fused(x, cfg)
    assert st0 != 0 and st1 != 0


@pytest.fixture
def fused_first_group(monkeypatch):
    monkeypatch.setattr(LS, "FACTOR_FROM_ACTIVATIONS", True)


def test_concurrent_gptq_with_fused_first_group_equals_sequential(fused_first_group):
    weights, inputs = _setup(3)
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    seq, _ = LS.quantize_layer_gptq(weights, inputs, cfg, SHAPES, concurrent=False)
    con, _ = LS.quantize_layer_gptq(weights, inputs, cfg, SHAPES)
    torch.cuda.synchronize()
    _assert_same(con, seq)


def test_concurrent_gptq_redoes_a_failed_fused_group(fused_first_group):
    """The largest group (fused statistics + factor) fails its first attempt;
    the driver recomputes its H and takes the retrying path, as the sequential
    driver does."""
    weights, inputs = _setup(2)
    inputs["c"][:, 3] = 0
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended",
                      damp_percent=0.0)
    seq, _ = LS.quantize_layer_gptq(weights, inputs, cfg, SHAPES, concurrent=False)
    con, _ = LS.quantize_layer_gptq(weights, inputs, cfg, SHAPES)
    torch.cuda.synchronize()
    _assert_same(con, seq)
