"""Masked next-token NLL -- restates ``src/jax_gptq/eval.py:9-22``.

Test infrastructure (see ``oracle/__init__.py``): float64 numpy, the
reference's op order (shift by one, mask -100, ``log_softmax``, pick the
label, sum).  Out-of-range labels are clamped, as JAX clamps gathers.
"""

from __future__ import annotations

import numpy as np


def masked_nll_from_logits(logits, labels) -> tuple[float, int]:
    logits = np.asarray(logits, np.float64)
    labels = np.asarray(labels)
    shift_logits = logits[:, :-1, :]
    shift_labels = labels[:, 1:]
    mask = shift_labels != -100
    safe = np.clip(np.where(mask, shift_labels, 0), 0, logits.shape[-1] - 1)
    mx = shift_logits.max(axis=-1, keepdims=True)
    lse = mx[..., 0] + np.log(np.exp(shift_logits - mx).sum(axis=-1))
    picked = np.take_along_axis(shift_logits, safe[..., None], axis=-1)[..., 0] - lse
    nll = -np.where(mask, picked, 0.0)
    return float(nll.sum()), int(mask.sum())


def perplexity(nll_sum: float, tokens: int) -> float:
    return float("nan") if tokens == 0 else float(np.exp(nll_sum / tokens))
