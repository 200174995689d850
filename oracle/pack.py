"""Packed quantized-weight format -- restates the layout `gq_pack_codes` writes.

Test infrastructure (see ``oracle/__init__.py``).  The reference has no packed
format (it returns dequantized floats, ``quant.py:37``); this module is the
specification the CUDA pack/unpack kernels are checked against:

* each row's codes, in original column order, form one little-endian bit
  stream: code ``c`` occupies stream bits ``[c*bits, (c+1)*bits)``, least
  significant bit first;
* the stream is cut into uint32 words, word ``w`` holding stream bits
  ``[32w, 32w+32)`` (bit ``32w + i`` is bit ``i`` of the word); the last word
  is zero-padded;
* dequantization is the sweep's: ``(code + qmin - zero[g]) * scale[g]`` in
  float32 with ``g = g_idx[c]``.
"""

from __future__ import annotations

import numpy as np

from .quant import qrange


def packed_words(n: int, bits: int) -> int:
    return (n * bits + 31) // 32


def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """uint8 [m, n] -> uint32 [m, packed_words(n, bits)]."""
    codes = np.asarray(codes, dtype=np.uint8)
    m, n = codes.shape
    stream = ((codes[:, :, None] >> np.arange(bits, dtype=np.uint8)) & 1).reshape(m, n * bits)
    words = packed_words(n, bits)
    padded = np.zeros((m, words * 32), dtype=np.uint64)
    padded[:, : n * bits] = stream
    weights = (np.uint64(1) << np.arange(32, dtype=np.uint64))
    return (padded.reshape(m, words, 32) * weights).sum(axis=2).astype(np.uint32)


def unpack(packed: np.ndarray, n: int, bits: int) -> np.ndarray:
    """uint32 [m, words] -> uint8 codes [m, n]."""
    packed = np.asarray(packed, dtype=np.uint32)
    m, words = packed.shape
    stream = ((packed[:, :, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(m, words * 32)
    bitsv = stream[:, : n * bits].reshape(m, n, bits).astype(np.uint32)
    return (bitsv << np.arange(bits, dtype=np.uint32)).sum(axis=2).astype(np.uint8)


def dequantize(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray, g_idx: np.ndarray,
               bits: int, sym: bool) -> np.ndarray:
    qmin, _ = qrange(bits, sym)
    q = np.asarray(codes, dtype=np.float32) + np.float32(qmin)
    g = np.asarray(g_idx)
    s = np.asarray(scales, dtype=np.float32)[:, g]
    z = np.asarray(zeros, dtype=np.float32)[:, g]
    return ((q - z) * s).astype(np.float32)
