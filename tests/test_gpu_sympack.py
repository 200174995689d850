"""Packed upper triangle of a symmetric matrix (gq_sym_pack_upper /
gq_sym_unpack_upper), the form in which token-sharded Hessians are summed
across GPUs: round trips bit for bit, and a sum of packed buffers unpacks to
the exactly symmetric sum of the matrices."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import _arrays as A
from jax_gptq_b200 import _lib


def _packed_rows(d):
    """The packed layout restated on the host: (row, first column) per packed row."""
    out = []
    for b0 in range(0, d, 128):
        for r in range(b0, min(d, b0 + 128)):
            out.append((r, b0))
    return out


def _pack(h):
    d = h.shape[0]
    p = torch.empty((_lib.lib().gq_sym_packed_size(d),), dtype=torch.float32, device="cuda")
    _lib.call("gq_sym_pack_upper", A.ptr(h), d, h.stride(0), A.ptr(p), A.stream())
    return p


def _unpack(p, h):
    _lib.call("gq_sym_unpack_upper", A.ptr(p), h.shape[0], A.ptr(h), h.stride(0), A.stream())


@pytest.mark.parametrize("d", [1, 127, 128, 129, 300, 1000, 4096])
def test_pack_layout_and_round_trip(d):
    g = torch.Generator(device="cuda").manual_seed(d)
    a = torch.randn((d, d), generator=g, device="cuda")
    h = a + a.t()
    p = _pack(h)
    # layout: packed rows back to back, row r from column 128 (r // 128) on
    hn, pn = h.cpu().numpy(), p.cpu().numpy()
    ref = np.concatenate([hn[r, c0:] for r, c0 in _packed_rows(d)])
    assert np.array_equal(pn, ref)
    out = torch.full((d, d), float("nan"), device="cuda")
    _unpack(p, out)
    torch.cuda.synchronize()
    assert out.equal(h)


def test_sum_of_packed_buffers_unpacks_to_the_symmetric_sum():
    """What the all-reduce does: element-wise sums of packed buffers.  The
    inputs' diagonal tiles are made slightly asymmetric (as two summation
    orders would leave them); the result takes the upper entries and is
    exactly symmetric."""
    d = 700
    g = torch.Generator(device="cuda").manual_seed(3)
    mats = []
    for _ in range(3):
        a = torch.randn((d, d), generator=g, device="cuda")
        mats.append(a + a.t())
    # below the diagonal inside the 128 x 128 diagonal tiles (the only lower
    # entries the packed form carries)
    idx = torch.arange(d, device="cuda")
    in_tile_lower = (idx[:, None] // 128 == idx[None, :] // 128) & (idx[:, None] > idx[None, :])
    mats[0] = mats[0] + 1e-3 * in_tile_lower.float()
    packed = sum(_pack(m) for m in mats)
    total = sum(mats)
    out = torch.empty((d, d), device="cuda")
    _unpack(packed, out)
    torch.cuda.synchronize()
    assert out.equal(out.t())
    upper = torch.triu(torch.ones((d, d), dtype=torch.bool, device="cuda"))
    # the packed sum adds in the same order as the sum of the matrices
    assert torch.equal(out[upper], total[upper])
    assert not torch.equal(out[in_tile_lower], total[in_tile_lower])


def test_unpack_into_a_wider_leading_dimension_leaves_the_padding():
    d, ld = 260, 272
    g = torch.Generator(device="cuda").manual_seed(9)
    a = torch.randn((d, d), generator=g, device="cuda")
    h = a + a.t()
    p = _pack(h)
    buf = torch.full((d, ld), -7.0, device="cuda")
    _unpack(p, buf[:, :d])
    torch.cuda.synchronize()
    assert buf[:, :d].equal(h)
    assert torch.all(buf[:, d:] == -7.0)
