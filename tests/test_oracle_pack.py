"""The packed-format oracle: round trips for every width and the bit layout
pinned on hand-computed words (the reference has no packed format)."""

import numpy as np
import pytest

from oracle import pack as P


@pytest.mark.parametrize("bits", range(1, 9))
@pytest.mark.parametrize("n", [1, 7, 31, 32, 33, 100, 1000])
def test_round_trip(bits, n):
    rng = np.random.default_rng(bits * 1000 + n)
    c = rng.integers(0, 1 << bits, (5, n)).astype(np.uint8)
    pk = P.pack(c, bits)
    assert pk.shape == (5, P.packed_words(n, bits)) and pk.dtype == np.uint32
    assert np.array_equal(P.unpack(pk, n, bits), c)


def test_bit_layout():
    assert P.pack(np.array([[1, 2]], np.uint8), 4)[0, 0] == 0x21
    assert P.pack(np.array([[0xF] * 8 + [1]], np.uint8), 4).tolist() == [[0xFFFFFFFF, 1]]
    # 3-bit: code 10 straddles words (bits 30..32)
    c = np.zeros((1, 11), np.uint8)
    c[0, 10] = 0b111
    assert P.pack(c, 3).tolist() == [[0xC0000000, 0x1]]


def test_dequantize_matches_the_sweep_formula():
    codes = np.array([[0, 15, 7]], np.uint8)
    scales = np.array([[0.5, 2.0]], np.float32)
    zeros = np.array([[3.0, 1.0]], np.float32)
    g_idx = np.array([1, 0, 0])
    out = P.dequantize(codes, scales, zeros, g_idx, 4, False)
    assert np.array_equal(out, np.array([[(0 - 1.0) * 2.0, (15 - 3.0) * 0.5, (7 - 3.0) * 0.5]],
                                        np.float32))
