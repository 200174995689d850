"""Round-to-nearest (RTN) group quantization -- restates ``src/jax_gptq/quant.py:6-37``.

Test infrastructure (see ``oracle/__init__.py``).  All arithmetic is float32
in the reference's op order so that integer codes are reproducible:

* ``qmax/qmin`` from ``w_bits`` and ``sym`` (quant.py:12-17);
* per (row, group of ``group_size`` consecutive columns) min/max or max|w|
  (quant.py:21-31); ``scale = max(range / qmax, 1e-8)``;
  ``zero = clip(round(-min / scale), 0, qmax)`` (asymmetric) or 0;
* ``q = clip(round(w / scale + zero), qmin, qmax)`` with round-half-to-even
  (quant.py:36); dequant ``(q - zero) * scale`` (quant.py:37).
"""

from __future__ import annotations

import numpy as np


def qrange(w_bits: int, sym: bool) -> tuple[float, float]:
    """quant.py:12-17."""
    if sym:
        qmax = float((1 << (w_bits - 1)) - 1)
        return -qmax, qmax
    return 0.0, float((1 << w_bits) - 1)


def check_rtn_args(w: np.ndarray, group_size: int) -> None:
    """The ValueError contract of quant.py:7-10."""
    if w.ndim != 2:
        raise ValueError(f"Expected 2D weight matrix, got shape={w.shape}")
    if group_size <= 0 or (w.shape[1] % group_size) != 0:
        raise ValueError("group_size must be positive and divide in_features exactly")


def group_params(w3: np.ndarray, w_bits: int, sym: bool) -> tuple[np.ndarray, np.ndarray]:
    """Scale and zero for groups laid out on the last axis (quant.py:23-31)."""
    qmin, qmax = qrange(w_bits, sym)
    qmax32 = np.float32(qmax)
    if sym:
        max_abs = np.max(np.abs(w3), axis=-1, keepdims=True)
        scale = np.maximum(max_abs / qmax32, np.float32(1e-8))
        zero = np.zeros_like(scale)
    else:
        mn = np.min(w3, axis=-1, keepdims=True)
        mx = np.max(w3, axis=-1, keepdims=True)
        scale = np.maximum((mx - mn) / qmax32, np.float32(1e-8))
        zero = np.clip(np.round(-mn / scale), np.float32(0.0), qmax32)
    return scale.astype(np.float32), zero.astype(np.float32)


def quantize_values(w: np.ndarray, scale: np.ndarray, zero: np.ndarray,
                    w_bits: int, sym: bool) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:36-37 for broadcast-compatible scale/zero; returns (q, dequant)."""
    qmin, qmax = qrange(w_bits, sym)
    q = np.clip(np.round(w / scale + zero), np.float32(qmin), np.float32(qmax))
    return q.astype(np.float32), ((q - zero) * scale).astype(np.float32)


def rtn(w, w_bits: int = 4, group_size: int = 128, sym: bool = False):
    """Full RTN pass.  Returns ``(dequant, q, scales, zeros)``.

    ``q`` holds the integer codes as float32 values in ``[qmin, qmax]``;
    ``scales``/``zeros`` are ``[m, n // group_size]``.
    """
    w = np.asarray(w, dtype=np.float32)
    check_rtn_args(w, group_size)
    m, n = w.shape
    g = group_size
    w3 = w.reshape(m, n // g, g)
    scale, zero = group_params(w3, w_bits, sym)
    q, dq = quantize_values(w3, scale, zero, w_bits, sym)
    return (dq.reshape(m, n), q.reshape(m, n), scale[..., 0], zero[..., 0])


def quantize_dequantize(w, w_bits: int = 4, group_size: int = 128, sym: bool = False) -> np.ndarray:
    """quant.py:6 -- dequantized weights only, like the reference."""
    return rtn(w, w_bits, group_size, sym)[0]


def tie_flip_mask(w, scale, zero, q_a, q_b, ulps: float = 4.0) -> np.ndarray:
    """Mark code mismatches that are legitimate rounding-tie flips.

    A mismatch between two code arrays counts as a tie flip only when the
    float64 value of ``w / scale + zero`` lies within ``ulps`` float32 ulps of
    a .5 rounding boundary (or of a clip boundary).
    """
    w = np.asarray(w, np.float64)
    t = w / np.asarray(scale, np.float64) + np.asarray(zero, np.float64)
    frac_dist = np.abs(np.abs(t - np.floor(t)) - 0.5)
    ulp = np.spacing(np.abs(t).astype(np.float32)).astype(np.float64)
    near = frac_dist <= ulps * np.maximum(ulp, np.finfo(np.float32).tiny)
    differ = np.asarray(q_a) != np.asarray(q_b)
    return differ & near
