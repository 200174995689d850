"""Packed weights on the device: gq_pack_codes equals the oracle's layout bit
for bit, unpacking returns the codes, and dequantizing a packed GPTQ result
reproduces the sweep's dequantized weights exactly; save/load round trips."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import packing
from jax_gptq_b200.config import QuantConfig
from jax_gptq_b200.gptq_ref import gptq_quantize
from oracle import inputs
from oracle import pack as P


class _Codes:
    def __init__(self, codes, n_groups):
        m, n = codes.shape
        self.codes = codes
        self.scales = torch.ones((m, n_groups), device="cuda")
        self.zeros = torch.zeros((m, n_groups), device="cuda")
        self.g_idx = torch.zeros((n,), dtype=torch.int32, device="cuda")
        self.perm = torch.arange(n, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("n", [33, 1000, 4096])
def test_pack_matches_oracle(bits, n):
    rng = np.random.default_rng(bits + n)
    c = rng.integers(0, 1 << bits, (70, n)).astype(np.uint8)
    p = packing.pack_result(_Codes(torch.from_numpy(c).cuda(), 1), bits, n, False)
    got = p.qweight.cpu().numpy().view(np.uint32)
    assert np.array_equal(got, P.pack(c, bits))
    assert np.array_equal(packing.unpack_codes(p).cpu().numpy(), c)


@pytest.mark.parametrize("bits,sym", [(4, False), (3, False), (4, True)])
def test_packed_gptq_result_dequantizes_exactly(bits, sym, tmp_path):
    w, x = inputs.single_linear(0, m=96, n=512, tokens=2048)
    h = (x.astype(np.float64).T @ x / x.shape[0]).astype(np.float32)
    cfg = QuantConfig(w_bits=bits, group_size=128, sym=sym, ordering_mode="diag_h",
                      semantics="intended")
    res = gptq_quantize(w, h, cfg)
    p = packing.pack_result(res, bits, 128, sym)
    assert p.qweight.shape == (96, (512 * bits + 31) // 32)
    assert packing.dequantize(p).equal(res.dequant)
    assert packing.unpack_codes(p).equal(res.codes)
    path = str(tmp_path / "layer0.pt")
    packing.save_layer(path, {"q_proj": p})
    back = packing.load_layer(path, device="cuda")["q_proj"]
    assert back.bits == bits and back.sym == sym and back.n == 512
    assert packing.dequantize(back).equal(res.dequant)
