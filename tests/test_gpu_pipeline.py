"""The layer walk over a small random-init decoder stack: every linear ends on
its quantization grid (the packed checkpoint dequantizes to the model's
weights), GPTQ beats round-to-nearest on the stack's output, Qronos runs, and
a second run resumes from the checkpoints without re-quantizing."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import packing, pipeline
from jax_gptq_b200.config import QuantConfig
from jax_gptq_b200.quant import quantize_dequantize

CFG = pipeline.BlockConfig(hidden=256, intermediate=640, heads=4, kv_heads=2)


def _calib(seed=0, batches=4):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return [(torch.randn((4, 64, CFG.hidden), generator=gen, device="cuda")).to(torch.bfloat16)
            for _ in range(batches)]


def _rel(a, b):
    num = sum(((x.float() - y.float()) ** 2).sum() for x, y in zip(a, b))
    den = sum((y.float() ** 2).sum() for y in b)
    return (num / den).sqrt().item()


def test_gptq_stack_walk_and_resume(tmp_path):
    calib = _calib()
    ref = pipeline.stack_forward(pipeline.synth_stack(2, CFG, seed=1), calib)
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    blocks = pipeline.synth_stack(2, CFG, seed=1)
    reps = pipeline.quantize_stack(blocks, calib, cfg, checkpoint_dir=str(tmp_path))
    assert [r.resumed for r in reps] == [False, False]
    assert reps[0].tokens == 4 * 4 * 64
    for li, blk in enumerate(blocks):
        for name, p in packing.load_layer(str(tmp_path / f"layer{li}.pt"), "cuda").items():
            assert packing.dequantize(p).to(torch.bfloat16).equal(getattr(blk, name).weight)
    err_gptq = _rel(pipeline.stack_forward(blocks, calib), ref)
    rtn = pipeline.synth_stack(2, CFG, seed=1)
    for blk in rtn:
        for name in pipeline.GROUPS:
            lin = getattr(blk, name)
            lin.weight.data.copy_(quantize_dequantize(lin.weight.float(), QuantConfig(
                w_bits=4, group_size=128)).to(torch.bfloat16))
    err_rtn = _rel(pipeline.stack_forward(rtn, calib), ref)
    assert err_gptq < err_rtn, (err_gptq, err_rtn)
    # resume: both layers come from disk and give the same weights
    again = pipeline.synth_stack(2, CFG, seed=1)
    reps2 = pipeline.quantize_stack(again, calib, cfg, checkpoint_dir=str(tmp_path))
    assert [r.resumed for r in reps2] == [True, True]
    for a, b in zip(blocks, again):
        for name in pipeline.GROUPS:
            assert getattr(a, name).weight.equal(getattr(b, name).weight)


def test_qronos_stack_walk():
    calib = _calib(2, batches=2)
    blocks = pipeline.synth_stack(1, CFG, seed=3)
    ref = pipeline.stack_forward(pipeline.synth_stack(1, CFG, seed=3), calib)
    cfg = QuantConfig(w_bits=3, group_size=128, ordering_mode="diag_h", semantics="intended")
    reps = pipeline.quantize_stack(blocks, calib, cfg, method="qronos")
    assert not reps[0].resumed and set(reps[0].attempts) == {"attn_in", "attn_out", "mlp_in",
                                                            "mlp_out"}
    assert _rel(pipeline.stack_forward(blocks, calib), ref) < 0.5
    with pytest.raises(ValueError):
        pipeline.quantize_stack(blocks, calib, cfg, method="awq")


def test_walk_first_block_matches_the_oracle(tmp_path):
    """The layer walk's q/k/v (first block, group attn_in) against the oracle:
    the H the walk accumulates from the captured bf16 activations, factored
    the same way, gives codes equal to the float32 oracle sweep up to
    rounding ties (the walk's packed codes, unpacked), and the walk's
    reconstruction error is within 1e-3 relative of the float64 oracle's."""
    import numpy as np
    from jax_gptq_b200 import stats
    from jax_gptq_b200.gptq_ref import factor_hessian
    from oracle import gptq as og
    from oracle import quant as oq
    from parity import TIE_TOL, code_diffs, report

    calib = _calib(5)
    blocks = pipeline.synth_stack(1, CFG, seed=4)
    w_orig = torch.cat([getattr(blocks[0], n).weight.detach().float()
                        for n in ("q_proj", "k_proj", "v_proj")])
    with torch.no_grad():
        xs = [blocks[0].input_layernorm(b).reshape(-1, CFG.hidden) for b in calib]
    cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
    pipeline.quantize_stack(blocks, calib, cfg, checkpoint_dir=str(tmp_path))
    packed = packing.load_layer(str(tmp_path / "layer0.pt"), "cuda")
    codes = torch.cat([packing.unpack_codes(packed[n]) for n in ("q_proj", "k_proj", "v_proj")])
    deq = torch.cat([packing.dequantize(packed[n]) for n in ("q_proj", "k_proj", "v_proj")])

    acc = stats.HessianAccumulator(CFG.hidden)
    for x in xs:
        acc.add(x)
    f = factor_hessian(acc.h, cfg)
    u, perm = f.u.cpu().numpy(), f.perm.cpu().numpy()
    w = w_orig.cpu().numpy()
    ref32 = og.gptq_sweep(w, u, perm, 4, 128, False, dtype=np.float32, return_pre=True)
    got_p = codes.cpu().numpy().astype(np.float32)[:, perm] + oq.qrange(4, False)[0]
    cd = code_diffs(got_p, ref32["q"][:, perm], ref32["pre"])
    assert cd["max_tie_dist"] <= TIE_TOL, cd["max_tie_dist"]

    x64 = np.concatenate([x.float().cpu().numpy().astype(np.float64) for x in xs])
    h64 = x64.T @ x64
    u64, perm64, _ = og.process_hessian_intended(h64, "diag_h", 0.01)
    ref64 = og.gptq_sweep(w, u64, perm64, 4, 128, False, dtype=np.float64)
    e_walk = og.reconstruction_error(w, deq.cpu().numpy(), h64)
    e_ref = og.reconstruction_error(w, ref64["dequant"], h64)
    report("walk_first_block_attn_in", tie_rows=cd["tie_rows"], e_walk=e_walk, e_oracle64=e_ref)
    assert abs(e_walk - e_ref) <= 1e-3 * e_ref, (e_walk, e_ref)
