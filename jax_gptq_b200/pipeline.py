"""Layer-by-layer quantization of a decoder stack: the caller of the hot path.

The reference quantizes one linear at a time from activations it is handed
(``noop_quant.py:4-6`` and ``scripts/run_noop_pipeline.py`` stop short of a
model walk).  ``quantize_stack`` is that walk for a Llama-style stack:

* the calibration hidden states go through the stack one block at a time;
* forward pre-hooks on one linear per input group (q_proj, o_proj,
  gate_proj, down_proj) stream the block's inputs into ``HessianAccumulator``
  (tcgen05 SYRK, and for Qronos also ``G = X^T Xt``);
* each group is factored once and its row-stacked linears swept (GPTQ) or
  updated (Qronos); the block's weights are replaced by the dequantized ones
  and packed (``packing.PackedLinear``) into ``layer{i}.pt``;
* the next block sees the quantized block's outputs (sequential GPTQ), while
  Qronos also carries the float model's hidden states for ``G``;
* with a checkpoint directory, blocks already on disk are reloaded instead of
  re-quantized, so an interrupted run resumes where it stopped.

The block itself (RMSNorm, rotary attention with grouped KV heads, SwiGLU
MLP) is plain torch: it is the model whose activations feed the kernels, not
part of the quantization path.
"""

from __future__ import annotations

import copy
import os
import time
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import packing, stats
from .config import QuantConfig
from .gptq_ref import SweepResult, factor_hessian, gptq_sweep
from .qronos_ref import qronos_quantize

# linear -> input group (linears of one group share an input and a factor)
GROUPS = {"q_proj": "attn_in", "k_proj": "attn_in", "v_proj": "attn_in", "o_proj": "attn_out",
          "gate_proj": "mlp_in", "up_proj": "mlp_in", "down_proj": "mlp_out"}
_CAPTURE = {"attn_in": "q_proj", "attn_out": "o_proj", "mlp_in": "gate_proj",
            "mlp_out": "down_proj"}


@dataclass
class BlockConfig:
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    eps: float = 1e-5
    rope_theta: float = 10000.0


class RMSNorm(torch.nn.Module):
    def __init__(self, d: int, eps: float):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


def _rope(x, theta: float):
    """Rotary position embedding on [B, heads, S, head_dim] (half-split form)."""
    b, h, s, hd = x.shape
    half = hd // 2
    inv = theta ** (-torch.arange(half, device=x.device, dtype=torch.float32) / half)
    ang = torch.arange(s, device=x.device, dtype=torch.float32)[:, None] * inv[None, :]
    cos, sin = ang.cos(), ang.sin()
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).to(x.dtype)


class DecoderBlock(torch.nn.Module):
    def __init__(self, cfg: BlockConfig):
        super().__init__()
        self.cfg = cfg
        hd = cfg.hidden // cfg.heads
        lin = lambda i, o: torch.nn.Linear(i, o, bias=False)
        self.q_proj = lin(cfg.hidden, cfg.heads * hd)
        self.k_proj = lin(cfg.hidden, cfg.kv_heads * hd)
        self.v_proj = lin(cfg.hidden, cfg.kv_heads * hd)
        self.o_proj = lin(cfg.heads * hd, cfg.hidden)
        self.gate_proj = lin(cfg.hidden, cfg.intermediate)
        self.up_proj = lin(cfg.hidden, cfg.intermediate)
        self.down_proj = lin(cfg.intermediate, cfg.hidden)
        self.input_layernorm = RMSNorm(cfg.hidden, cfg.eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden, cfg.eps)

    def forward(self, x):
        c = self.cfg
        b, s, _ = x.shape
        hd = c.hidden // c.heads
        h = self.input_layernorm(x)
        q = self.q_proj(h).view(b, s, c.heads, hd).transpose(1, 2)
        k = self.k_proj(h).view(b, s, c.kv_heads, hd).transpose(1, 2)
        v = self.v_proj(h).view(b, s, c.kv_heads, hd).transpose(1, 2)
        q, k = _rope(q, c.rope_theta), _rope(k, c.rope_theta)
        rep = c.heads // c.kv_heads
        k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.o_proj(a.transpose(1, 2).reshape(b, s, c.heads * hd))
        h = self.post_attention_layernorm(x)
        return x + self.down_proj(F.silu(self.gate_proj(h)) * self.up_proj(h))


def synth_stack(n_layers: int, cfg: BlockConfig, seed: int = 0, std: float = 0.02,
                dtype=torch.bfloat16) -> list[DecoderBlock]:
    """Random-init blocks (weights ~ N(0, std^2)) on the GPU."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    blocks = []
    for _ in range(n_layers):
        blk = DecoderBlock(cfg)
        with torch.no_grad():
            for name in GROUPS:
                lin = getattr(blk, name)
                lin.weight.copy_(torch.randn(lin.weight.shape, generator=gen) * std)
        blocks.append(blk.to(device="cuda", dtype=dtype).eval())
    return blocks


@dataclass
class LayerReport:
    layer: int
    resumed: bool
    tokens: int = 0
    stats_ms: float = 0.0
    quant_ms: float = 0.0
    attempts: dict = field(default_factory=dict)


def _capture_hooks(block, sink):
    """Pre-hooks that hand each captured group's input [tokens, in] to sink(grp, x)."""
    hooks = []
    for grp, name in _CAPTURE.items():
        def hook(_mod, args, grp=grp):
            x = args[0]
            sink(grp, x.reshape(-1, x.shape[-1]))
        hooks.append(getattr(block, name).register_forward_pre_hook(hook))
    return hooks


def _members(grp):
    return [name for name in GROUPS if GROUPS[name] == grp]


@torch.no_grad()
def quantize_stack(blocks: list[DecoderBlock], calib: list[torch.Tensor], cfg: QuantConfig,
                   method: str = "gptq", checkpoint_dir: str | None = None) -> list[LayerReport]:
    """Quantize ``blocks`` in place, layer by layer, from calibration hidden
    states ``calib`` (a list of [B, S, hidden] batches on the GPU).

    ``method``: "gptq" (H from the quantized model's inputs) or "qronos"
    (H = Xt^T Xt from the quantized model, G = X^T Xt with X from the float
    model).  Returns one :class:`LayerReport` per block."""
    if method not in ("gptq", "qronos"):
        raise ValueError(f"method must be 'gptq' or 'qronos', got {method!r}")
    if checkpoint_dir:
        os.makedirs(checkpoint_dir, exist_ok=True)
    xq = [x.clone() for x in calib]
    xf = [x.clone() for x in calib] if method == "qronos" else None
    reports = []
    for li, blk in enumerate(blocks):
        path = os.path.join(checkpoint_dir, f"layer{li}.pt") if checkpoint_dir else None
        float_blk = copy.deepcopy(blk) if method == "qronos" else None
        if path and os.path.exists(path):
            for name, p in packing.load_layer(path, device="cuda").items():
                getattr(blk, name).weight.copy_(packing.dequantize(p).to(blk.q_proj.weight.dtype))
            reports.append(LayerReport(li, True))
        else:
            rep = LayerReport(li, False)
            t0 = time.perf_counter()
            accs: dict[str, stats.HessianAccumulator] = {}

            def acc_for(grp, d):
                if grp not in accs:
                    accs[grp] = stats.HessianAccumulator(d, with_cross=(method == "qronos"))
                return accs[grp]

            if method == "gptq":
                hooks = _capture_hooks(blk, lambda g, x: acc_for(g, x.shape[1]).add(x))
                for b in xq:
                    blk(b)
            else:
                held = {}
                hooks = _capture_hooks(blk, lambda g, x: held.__setitem__(g, x))
                for bq, bf in zip(xq, xf):
                    blk(bf)
                    x_float = dict(held)
                    blk(bq)
                    for g, x in held.items():
                        acc_for(g, x.shape[1]).add(x, x_float[g])
            for h in hooks:
                h.remove()
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            packed = {}
            for grp, acc in accs.items():
                names = _members(grp)
                w = torch.cat([getattr(blk, n).weight.float() for n in names], dim=0)
                if method == "gptq":
                    f = factor_hessian(acc.h, cfg)
                    res = gptq_sweep(w, f.u, f.perm, cfg)
                else:
                    f = factor_hessian(acc.h, cfg, want_hd=True)
                    res = qronos_quantize(w, w, None, acc.g, cfg, factor=f)
                rep.attempts[grp] = f.attempt
                r0 = 0
                for n in names:
                    lin = getattr(blk, n)
                    m = lin.weight.shape[0]
                    part = SweepResult(res.dequant[r0:r0 + m], res.codes[r0:r0 + m],
                                       res.scales[r0:r0 + m], res.zeros[r0:r0 + m], res.g_idx,
                                       res.perm)
                    lin.weight.copy_(part.dequant.to(lin.weight.dtype))
                    packed[n] = packing.pack_result(part, cfg.w_bits, cfg.group_size, cfg.sym)
                    r0 += m
            torch.cuda.synchronize()
            rep.stats_ms = 1e3 * (t1 - t0)
            rep.quant_ms = 1e3 * (time.perf_counter() - t1)
            rep.tokens = accs["attn_in"].tokens if "attn_in" in accs else 0
            if path:
                packing.save_layer(path, packed)
            reports.append(rep)
        # the next block's inputs: the quantized model's (and the float model's)
        xq = [blk(b) for b in xq]
        if xf is not None:
            xf = [float_blk(b) for b in xf]
    return reports


class TinyLM(torch.nn.Module):
    """Token embedding -> decoder blocks -> RMSNorm -> LM head: a small
    language model around a block stack, for perplexity checks of a
    quantized stack (eval.py's role in the reference).  ``hidden(ids)`` is
    the blocks' input (the calibration batches of :func:`quantize_stack`);
    ``forward(ids)`` returns [B, T, vocab] logits."""

    def __init__(self, blocks, vocab: int, cfg: BlockConfig, seed: int = 0,
                 head_std: float | None = None, dtype=torch.bfloat16):
        super().__init__()
        gen = torch.Generator(device="cpu").manual_seed(seed)
        self.embed = torch.nn.Embedding(vocab, cfg.hidden)
        self.blocks = torch.nn.ModuleList(blocks)
        self.norm = RMSNorm(cfg.hidden, cfg.eps)
        self.lm_head = torch.nn.Linear(cfg.hidden, vocab, bias=False)
        std = head_std if head_std is not None else 4.0 / cfg.hidden ** 0.5
        with torch.no_grad():
            self.embed.weight.copy_(torch.randn(self.embed.weight.shape, generator=gen))
            self.lm_head.weight.copy_(torch.randn(self.lm_head.weight.shape, generator=gen) * std)
        self.embed.to(device="cuda", dtype=dtype)
        self.norm.to(device="cuda", dtype=dtype)
        self.lm_head.to(device="cuda", dtype=dtype)
        self.eval()

    def hidden(self, ids: torch.Tensor) -> torch.Tensor:
        return self.embed(ids)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        x = self.embed(ids)
        for blk in self.blocks:
            x = blk(x)
        return self.lm_head(self.norm(x))


def stack_forward(blocks, batches):
    with torch.no_grad():
        out = []
        for b in batches:
            for blk in blocks:
                b = blk(b)
            out.append(b)
        return out

