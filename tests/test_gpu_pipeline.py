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
