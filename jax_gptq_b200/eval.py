"""Perplexity evaluation -- drop-in for ``src/jax_gptq/eval.py``.

``masked_nll_from_logits`` is ``_masked_nll_from_logits`` (eval.py:9-22):
shift by one position, skip labels equal to -100, sum ``-log_softmax`` at the
label.  It runs the ``gq_masked_nll`` kernel, which reads each logit once
(HBM-bound) and sums the per-position values in a fixed order.
``evaluate_perplexity_flax`` keeps the reference's loop and signature
(eval.py:25-48): ``model(input_ids=..., params=..., train=False)`` returns an
object with ``.logits``; ``evaluate_perplexity`` is the same loop for a plain
callable ``model(input_ids) -> logits`` (e.g. :class:`pipeline.TinyLM`).
"""

from __future__ import annotations

from typing import Callable, List

import numpy as np
import torch

from . import _arrays as A
from . import _lib


def masked_nll_from_logits(logits, labels) -> tuple[float, int]:
    """eval.py:9-22 -- ``(nll_sum, token_count)``.

    ``logits`` [B, T, V] float32 or bf16 (torch on the device, or numpy);
    ``labels`` [B, T] integers, -100 for positions that are not scored."""
    if len(tuple(logits.shape)) != 3 or len(tuple(labels.shape)) != 2 or \
            tuple(labels.shape) != tuple(logits.shape[:2]):
        raise ValueError(f"logits must be [B, T, V] and labels [B, T], got "
                         f"{tuple(logits.shape)} and {tuple(labels.shape)}")
    if isinstance(logits, torch.Tensor) and logits.dtype == torch.bfloat16:
        lg = A.to_device(logits, torch.bfloat16)
        dtype = 1
    else:
        lg = A.to_device(logits, torch.float32)
        dtype = 0
    lab = A.to_device(labels, torch.int64)
    b, t, v = lg.shape
    ws = A.workspace(_lib.lib().gq_masked_nll_workspace_size(b, t))
    out = torch.empty((1,), dtype=torch.float64, device="cuda")
    cnt = torch.empty((1,), dtype=torch.int64, device="cuda")
    _lib.call("gq_masked_nll", A.ptr(lg), dtype, b, t, v, A.ptr(lab), A.ptr(out), A.ptr(cnt),
              A.ptr(ws), ws.numel(), A.stream())
    return float(out.item()), int(cnt.item())


def evaluate_perplexity(model: Callable, windows: List, labels: List, batch_size: int = 1) -> float:
    """eval.py:25-48 for ``model(input_ids) -> logits [B, T, V]``."""
    total_nll, total_tokens = 0.0, 0
    for i in range(0, len(windows), batch_size):
        end = min(i + batch_size, len(windows))
        input_batch = np.concatenate([np.asarray(w) for w in windows[i:end]], axis=0)
        label_batch = np.concatenate([np.asarray(l) for l in labels[i:end]], axis=0)
        with torch.no_grad():
            logits = model(torch.from_numpy(input_batch).cuda())
        nll, tokens = masked_nll_from_logits(logits, label_batch)
        total_nll += nll
        total_tokens += tokens
    if total_tokens == 0:
        return float("nan")
    return float(np.exp(total_nll / total_tokens))


def evaluate_perplexity_flax(model, params, windows: List, labels: List,
                             batch_size: int = 1) -> float:
    """eval.py:25-48 with the reference's model calling convention."""
    return evaluate_perplexity(
        lambda ids: model(input_ids=ids, params=params, train=False).logits, windows, labels,
        batch_size)


__all__ = ["masked_nll_from_logits", "evaluate_perplexity", "evaluate_perplexity_flax"]
