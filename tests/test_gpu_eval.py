"""Perplexity evaluation (eval.py's role) on the GPU.

* ``gq_masked_nll`` against the oracle's float64 restatement of
  ``_masked_nll_from_logits`` (eval.py:9-22): float32 and bf16 logits,
  a vocabulary that is not a multiple of 4, masked (-100) and out-of-range
  labels, single-token windows; relative error <= 1e-6, bit-identical reruns.
* The layer walk as a language model: a float TinyLM, the same model after
  GPTQ and after round-to-nearest, scored on held-out windows whose labels are
  the float model's own greedy predictions.  GPTQ's perplexity must lie
  closer to the float model's than round-to-nearest's does, and
  ``evaluate_perplexity`` must equal the oracle's NLL on the same logits.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import eval as E
from jax_gptq_b200 import pipeline
from jax_gptq_b200.config import QuantConfig
from jax_gptq_b200.quant import quantize_dequantize
from oracle import eval as oe

NLL_REL = 1e-6


@pytest.mark.parametrize("shape,dtype", [((3, 17, 1003), torch.float32),
                                         ((2, 33, 32000), torch.bfloat16),
                                         ((4, 1, 50), torch.float32),
                                         ((1, 9, 4096), torch.float32)])
def test_masked_nll_matches_oracle(shape, dtype):
    b, t, v = shape
    gen = torch.Generator(device="cuda").manual_seed(sum(shape))
    logits = (torch.randn(shape, generator=gen, device="cuda") * 3.0).to(dtype)
    rng = np.random.default_rng(sum(shape))
    labels = rng.integers(0, v, size=(b, t)).astype(np.int64)
    labels[rng.random((b, t)) < 0.2] = -100
    if t > 2:
        labels[0, 2] = v + 5  # clamped to v - 1, as JAX clamps gathers
    nll, cnt = E.masked_nll_from_logits(logits, labels)
    ref, rcnt = oe.masked_nll_from_logits(logits.float().cpu().numpy(), labels)
    assert cnt == rcnt
    if rcnt:
        assert abs(nll - ref) <= NLL_REL * abs(ref), (nll, ref)
    else:
        assert nll == 0.0
    again, _ = E.masked_nll_from_logits(logits, labels)
    assert again == nll  # fixed-order reduction


def test_masked_nll_rejects_bad_shapes():
    with pytest.raises(ValueError):
        E.masked_nll_from_logits(torch.zeros((2, 3), device="cuda"), np.zeros((2, 3), np.int64))


CFG = pipeline.BlockConfig(hidden=256, intermediate=640, heads=4, kv_heads=2)
VOCAB = 512


def _ids(seed, n, b=4, t=64):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, VOCAB, size=(b, t)).astype(np.int64) for _ in range(n)]


def _lm(blocks):
    return pipeline.TinyLM(blocks, VOCAB, CFG, seed=11)


def test_perplexity_of_quantized_stacks():
    float_lm = _lm(pipeline.synth_stack(2, CFG, seed=1))
    calib = [float_lm.hidden(torch.from_numpy(w).cuda()) for w in _ids(0, 4)]
    windows = [w[:1] for w in _ids(1, 6, b=1)]
    with torch.no_grad():
        labels = []
        for w in windows:
            pred = float_lm(torch.from_numpy(w).cuda()).float().argmax(-1).cpu().numpy()
            lab = np.full_like(w, -100)
            lab[:, 1:] = pred[:, :-1]   # the float model's greedy next-token choices
            labels.append(lab)
    ppl_float = E.evaluate_perplexity(float_lm, windows, labels, batch_size=2)

    gptq_lm = _lm(pipeline.synth_stack(2, CFG, seed=1))
    cfg = QuantConfig(w_bits=3, group_size=128, ordering_mode="diag_h", semantics="intended")
    pipeline.quantize_stack(list(gptq_lm.blocks), calib, cfg)
    ppl_gptq = E.evaluate_perplexity(gptq_lm, windows, labels, batch_size=2)

    rtn_lm = _lm(pipeline.synth_stack(2, CFG, seed=1))
    for blk in rtn_lm.blocks:
        for name in pipeline.GROUPS:
            lin = getattr(blk, name)
            lin.weight.data.copy_(quantize_dequantize(
                lin.weight.float(), QuantConfig(w_bits=3, group_size=128)).to(torch.bfloat16))
    ppl_rtn = E.evaluate_perplexity(rtn_lm, windows, labels, batch_size=2)
    # a quantized model can score the float model's greedy labels slightly
    # better than the float model itself (sharper peaks), so compare gaps
    assert abs(ppl_gptq - ppl_float) < abs(ppl_rtn - ppl_float), (ppl_float, ppl_gptq, ppl_rtn)

    # the loop's result equals the oracle's NLL over the same logits
    tot, cnt = 0.0, 0
    with torch.no_grad():
        for w, lab in zip(windows, labels):
            n, c = oe.masked_nll_from_logits(
                gptq_lm(torch.from_numpy(w).cuda()).float().cpu().numpy(), lab)
            tot, cnt = tot + n, cnt + c
    assert abs(np.log(ppl_gptq) - tot / cnt) <= NLL_REL * abs(tot / cnt)
