"""Sharded execution of the quantization path on one GPU.

Ranks are emulated in one process (no process group): the partial Gram
matrices of token shards must add up to the whole-input H, and row shards
swept with the same factor must reproduce the unsharded sweep bit for bit
(rows are independent and every kernel's per-element arithmetic is
independent of where a row sits).  The single-rank driver must equal the
single-GPU layer-set path.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import distributed as D
from jax_gptq_b200 import layerset as LS
from jax_gptq_b200 import stats
from jax_gptq_b200.config import QuantConfig
from jax_gptq_b200.gptq_ref import factor_hessian, gptq_sweep

SHAPES = [("q", 256, 512, "a"), ("k", 64, 512, "a"), ("o", 200, 384, "b")]


def _inputs(tokens=3000):
    return {"a": LS.synth_activations(tokens, 512, 1)[0], "b": LS.synth_activations(tokens, 384, 2)[0]}


def test_token_shard_partials_sum_to_whole_h():
    x = _inputs()["a"]
    h_full = torch.empty((512, 512), dtype=torch.float32, device="cuda")
    stats.syrk_into(h_full, x, accumulate=False)
    parts = []
    for r in range(3):
        t0, t1 = D.shard_range(x.shape[0], r, 3)
        h = torch.empty_like(h_full)
        stats.syrk_into(h, x[t0:t1], accumulate=False)
        parts.append(h)
    h_sum = parts[0] + parts[1] + parts[2]
    rel = (torch.linalg.norm(h_sum - h_full) / torch.linalg.norm(h_full)).item()
    assert rel < 1e-6, rel
    assert D.hessians_token_sharded({"a": x})["a"].equal(h_full)  # one rank: no collective


@pytest.mark.parametrize("world", [2, 3, 8])
def test_row_shards_reproduce_the_whole_sweep(world):
    w = LS.synth_weights(SHAPES, 0.02, 3)["q"]
    x = _inputs()["a"]
    h = torch.empty((512, 512), dtype=torch.float32, device="cuda")
    stats.syrk_into(h, x, accumulate=False)
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    f = factor_hessian(h, cfg)
    whole = gptq_sweep(w, f.u, f.perm, cfg)
    pieces = []
    for r in range(world):
        r0, r1 = D.shard_range(w.shape[0], r, world, D.SWEEP_ROW_ALIGN)
        if r1 > r0:
            pieces.append(gptq_sweep(w[r0:r1], f.u, f.perm, cfg))
    assert torch.cat([p.dequant for p in pieces]).equal(whole.dequant)
    assert torch.cat([p.codes for p in pieces]).equal(whole.codes)
    assert torch.cat([p.scales for p in pieces]).equal(whole.scales)


def test_single_rank_driver_matches_layer_set_path():
    weights = LS.synth_weights(SHAPES, 0.02, 4)
    inputs = _inputs()
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    ref, _ = LS.quantize_layer_gptq(weights, inputs, cfg, SHAPES)
    got = D.quantize_layer_gptq_sharded(weights, inputs, cfg, SHAPES)
    for name, _m, _n, _g in SHAPES:
        assert got[name].dequant.equal(ref[name].dequant), name
        assert got[name].codes.equal(ref[name].codes), name


def test_empty_row_shard_still_writes_group_indices():
    """A rank whose row shard is empty (fewer rows than 32 * world) still
    returns the group index of every column: g_idx depends only on the
    permutation, and the sharded driver hands one rank's g_idx to every
    member linear.  The output buffer starts as garbage on purpose."""
    w = LS.synth_weights(SHAPES, 0.02, 3)["q"]
    x = _inputs()["a"]
    h = torch.empty((512, 512), dtype=torch.float32, device="cuda")
    stats.syrk_into(h, x, accumulate=False)
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    f = factor_hessian(h, cfg)
    whole = gptq_sweep(w, f.u, f.perm, cfg)
    r0, r1 = D.shard_range(w.shape[0], 8, 9, D.SWEEP_ROW_ALIGN)
    assert r0 == r1  # 256 rows, 9 ranks of 32: the last rank has none
    torch.cuda.empty_cache()
    junk = torch.full((1 << 20,), -7, dtype=torch.int32, device="cuda")  # dirty the allocator's blocks
    del junk
    empty = gptq_sweep(w[r0:r1], f.u, f.perm, cfg)
    assert empty.dequant.shape == (0, 512)
    assert empty.g_idx.equal(whole.g_idx)


@pytest.mark.parametrize("world,min_split", [(1, None), (2, None), (3, None), (8, None),
                                             (2, 1024), (3, 512), (8, 512)])
def test_split_factor_matches_the_whole_factor(world, min_split):
    """The factor with its split products divided by rows over `world`
    ranks (emulated on one GPU: every slice computed in turn) equals the
    unsplit factor to float32 rounding: same permutation, U upper
    triangular, within 1e-5 relative.  With `min_split` the diagonal blocks
    at least that wide are split again (2560 -> 1280 -> 640 -> 320 at 512:
    three levels of split products)."""
    x = LS.synth_activations(8192, 2560, 21)[0]
    h = torch.empty((2560, 2560), dtype=torch.float32, device="cuda")
    stats.syrk_into(h, x, accumulate=False)
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    whole = factor_hessian(h, cfg)
    split, status = D.factor_hessian_split_emulated(h, cfg, world, min_split)
    assert int(status.item()) == 0
    assert split.perm.equal(whole.perm)
    assert torch.equal(torch.tril(split.u, -1), torch.zeros_like(split.u))
    rel = (torch.linalg.norm(split.u - whole.u) / torch.linalg.norm(whole.u)).item()
    assert rel <= 1e-5, rel
