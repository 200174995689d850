"""Decoder-layer-set quantization on one GPU: the whole hot path per layer.

A layer set is the seven linears of a Llama-style decoder block, grouped by
the activation that feeds them (q/k/v share the attention input, gate/up
share the MLP input):

* per input group: ``H = X^T X`` on the tcgen05 tensor cores (and for
  Qronos ``G = X^T Xt``), act-order permutation, damped inverse-Cholesky
  factor -- computed once and shared by the group's linears;
* per linear: the GPTQ (or Qronos) column sweep.

Shapes follow the benchmark configurations (Llama-2-7B and Llama-3-70B
blocks).  Inputs are synthetic and generated on the device with seeded
torch generators.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import _lib, stats
from .config import QuantConfig
from .gptq_ref import (HessianFactor, SweepResult, factor_from_activations_attempt0,
                       factor_hessian, factor_hessian_attempt0, gptq_sweep)
from .qronos_ref import qronos_quantize

# (name, out_features, in_features, input group)
LLAMA2_7B = [
    ("q_proj", 4096, 4096, "attn_in"), ("k_proj", 4096, 4096, "attn_in"),
    ("v_proj", 4096, 4096, "attn_in"), ("o_proj", 4096, 4096, "attn_out"),
    ("gate_proj", 11008, 4096, "mlp_in"), ("up_proj", 11008, 4096, "mlp_in"),
    ("down_proj", 4096, 11008, "mlp_out"),
]
LLAMA3_70B = [
    ("q_proj", 8192, 8192, "attn_in"), ("k_proj", 1024, 8192, "attn_in"),
    ("v_proj", 1024, 8192, "attn_in"), ("o_proj", 8192, 8192, "attn_out"),
    ("gate_proj", 28672, 8192, "mlp_in"), ("up_proj", 28672, 8192, "mlp_in"),
    ("down_proj", 8192, 28672, "mlp_out"),
]
SHAPES = {"llama2-7b": LLAMA2_7B, "llama3-70b": LLAMA3_70B}


def group_dims(shapes) -> dict[str, int]:
    dims: dict[str, int] = {}
    for _, _, n, grp in shapes:
        dims[grp] = n
    return dims


def syrk_flops(tokens: int, d: int) -> float:
    """Algorithmic flops of ``H = X^T X`` counted as a symmetric rank-k update."""
    return float(tokens) * d * (d + 1)


def gemm_flops(tokens: int, d: int) -> float:
    return 2.0 * tokens * d * d


def synth_weights(shapes, std: float, seed: int, device="cuda") -> dict[str, torch.Tensor]:
    """bf16 N(0, std^2) weights, upcast exactly to float32."""
    gen = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, m, n, _ in shapes:
        w = torch.randn((m, n), generator=gen, device=device, dtype=torch.float32) * std
        out[name] = w.to(torch.bfloat16).to(torch.float32)
    return out


def synth_activations(tokens: int, d: int, seed: int, kind: str = "lognormal",
                      device="cuda", chunk: int = 32768):
    """bf16 [tokens, d] calibration activations and their per-channel std.

    ``lognormal``: N(0, 1) times a per-channel log-normal(0, 1) scale;
    ``student_t``: Student-t with 4 degrees of freedom.
    """
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.empty((tokens, d), dtype=torch.bfloat16, device=device)
    if kind == "lognormal":
        scale = torch.exp(torch.randn((d,), generator=gen, device=device))
    else:
        scale = torch.ones((d,), device=device)
    for t0 in range(0, tokens, chunk):
        t1 = min(tokens, t0 + chunk)
        z = torch.randn((t1 - t0, d), generator=gen, device=device)
        if kind == "student_t":
            # t_4 = Z / sqrt(chi2_4 / 4), chi2_4 = sum of 4 squared normals
            chi = torch.zeros((t1 - t0, d), device=device)
            for _ in range(4):
                chi += torch.randn((t1 - t0, d), generator=gen, device=device) ** 2
            z = z / torch.sqrt(chi / 4.0)
        x[t0:t1] = (z * scale).to(torch.bfloat16)
    std = scale if kind == "lognormal" else torch.full((d,), math.sqrt(2.0), device=device)
    return x, std


def perturb_activations(x: torch.Tensor, std: torch.Tensor, rel: float, seed: int,
                        chunk: int = 32768) -> torch.Tensor:
    """``Xt = X + N(0, (rel * sigma_c)^2)``: stand-in for quantized-model activations."""
    gen = torch.Generator(device=x.device).manual_seed(seed)
    out = torch.empty_like(x)
    for t0 in range(0, x.shape[0], chunk):
        t1 = min(x.shape[0], t0 + chunk)
        noise = torch.randn((t1 - t0, x.shape[1]), generator=gen, device=x.device) * (rel * std)
        out[t0:t1] = (x[t0:t1].float() + noise).to(torch.bfloat16)
    return out


@dataclass
class LayerTimes:
    """Milliseconds per phase (CUDA events on the compute stream)."""
    stats_ms: float = 0.0
    factor_ms: float = 0.0
    sweep_ms: float = 0.0
    per_group_stats_ms: dict = field(default_factory=dict)


class _Timer:
    def __init__(self, enabled: bool):
        self.enabled = enabled
        self.marks = []

    def mark(self, label: str):
        if self.enabled:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.marks.append((label, ev))

    def spans(self) -> list[tuple[str, float]]:
        if not self.enabled:
            return []
        torch.cuda.synchronize()
        out = []
        for (l0, e0), (_, e1) in zip(self.marks, self.marks[1:]):
            out.append((l0, e0.elapsed_time(e1)))
        return out


def _members(shapes, grp):
    return [(name, m) for name, m, _, g in shapes if g == grp]


def _split_rows(res: SweepResult, members) -> dict:
    """Per-linear views of a sweep run on row-stacked weights."""
    out, r0 = {}, 0
    for name, m in members:
        out[name] = SweepResult(res.dequant[r0:r0 + m], res.codes[r0:r0 + m],
                                res.scales[r0:r0 + m], res.zeros[r0:r0 + m], res.g_idx, res.perm)
        r0 += m
    return out


_SIDE_STREAMS: dict[int, list] = {}
# SMs that the persistent kernels launched while a higher-priority chain is
# running leave free to it.  12 on a 148-SM part: the d = 4096 Hessians then
# run in exactly two waves of 136 tiles.
RESERVED_SMS = 12
# Statistics formed while a chain is running are split into launches of this
# many tokens (bit-identical to one launch), so the chain's kernels, on a
# higher-priority stream, get the SMs between them.
STATS_TOKEN_CHUNK = 32768


def _side_streams(n: int) -> list:
    """A per-device pool of side streams, one per input group run concurrently;
    the first has the highest scheduling priority (it carries the longest
    chain: the largest Hessian's factor and its sweep)."""
    dev = torch.cuda.current_device()
    pool = _SIDE_STREAMS.setdefault(dev, [])
    while len(pool) < n:
        pool.append(torch.cuda.Stream(device=dev, priority=-1 if not pool else 0))
    return pool[:n]


# Form the largest group's factor straight from its activations
# (factor_from_activations_attempt0): the factor's first half then overlaps
# the rest of that group's Hessian.  Off by default: in the concurrent layer
# step the other groups' statistics and chains already keep the GPU busy
# while the largest chain runs, so the shorter chain did not shorten the step
# (measured on the 7B layer set), and the gathered copy of the activations
# costs tokens x d x 2 bytes.  It pays where a group's statistics overlap
# nothing else.
FACTOR_FROM_ACTIVATIONS = False


def _fused_factor_ok(x: torch.Tensor, cfg: QuantConfig) -> bool:
    return (x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
            and x.shape[1] % 8 == 0 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0
            and cfg.solver_mode == "chol" and cfg.ordering_mode in ("none", "diag_h"))


def _chain_sizes(inputs: dict, shapes) -> dict:
    """Per input group, the key that orders the chains, longest first: the
    feature count (the factor's cost, cubic), then the stacked row count (the
    sweep's).  The last group's chain is the only one that overlaps no
    statistics, so it should be the shortest."""
    return {grp: (x.shape[1], sum(m for _, m in _members(shapes, grp)))
            for grp, x in inputs.items()}


def _stack(weights: dict, members) -> torch.Tensor:
    return weights[members[0][0]] if len(members) == 1 else \
        torch.cat([weights[name] for name, _ in members], dim=0)


def _run_groups_concurrently(sizes: dict, form, work, redo, prepare=None, late=None,
                             fused=None) -> dict:
    """Run each input group's chain on its own side stream.

    ``sizes[grp]`` orders the groups (largest first).  ``form(grp, chunk)
    -> h`` runs on the current stream and forms the group's statistics, in
    launches of ``chunk`` tokens (None: one launch) once a chain is running;
    ``work(grp, h) -> (status, result)`` then runs on the group's side stream
    as soon as that h is ready, while the current stream goes on to the next
    group's statistics.  The largest group's chain (the longest) runs on the
    high-priority stream and starts first; every persistent kernel launched
    after it leaves ``RESERVED_SMS`` SMs free, so its latency-bound steps
    overlap the remaining statistics and the other chains.

    With ``prepare`` and ``late`` the chain is split around statistics that
    only its second half reads (Qronos' cross term): ``prepare(grp, h) ->
    state`` (the factor) is queued on the side stream first, then
    ``late(grp, chunk)`` forms the late statistics on the current stream,
    and ``work(grp, state)`` follows on the side stream once they are ready.
    With ``fused`` (and ``prepare``), the first group's statistics and
    factor are enqueued together by ``fused(grp, side_stream) -> state``
    (statistics on the current stream, the factor on the side stream, which
    can then start before the statistics are complete); ``redo`` then gets
    ``h = None`` for that group.

    ``status`` is the device word of the group's first damping attempt; the
    statuses are read once at the end, and a group whose damped Hessian was
    not positive definite is recomputed by ``redo(grp, h)`` (the retrying,
    synchronizing path), so the outcome equals the sequential one.  Result
    tensors are marked as used by the current stream, which waits for every
    side stream before returning."""
    main = torch.cuda.current_stream()
    order = sorted(sizes, key=lambda g: sizes[g], reverse=True)
    streams = _side_streams(len(order))
    sms = torch.cuda.get_device_properties(main.device).multi_processor_count
    lib = _lib.lib()
    pending, hs = {}, {}
    for idx, (grp, s) in enumerate(zip(order, streams)):
        lib.gq_set_cta_budget(0 if idx == 0 else max(1, sms - RESERVED_SMS))
        try:
            if idx == 0 and fused is not None:
                hs[grp] = None
                state = fused(grp, s)
            else:
                hs[grp] = form(grp, None if idx == 0 else STATS_TOKEN_CHUNK)
                s.wait_stream(main)
                if prepare is None:
                    with torch.cuda.stream(s):
                        pending[grp] = work(grp, hs[grp])
                    continue
                with torch.cuda.stream(s):
                    state = prepare(grp, hs[grp])
            if late is not None:
                # the chain is now running: leave it its SMs
                lib.gq_set_cta_budget(max(1, sms - RESERVED_SMS))
                late(grp, STATS_TOKEN_CHUNK)
                s.wait_stream(main)
            with torch.cuda.stream(s):
                pending[grp] = work(grp, state)
        finally:
            lib.gq_set_cta_budget(0)
    for s in streams:
        main.wait_stream(s)
    for status, res in pending.values():
        status.record_stream(main)
        for t in (res.dequant, res.codes, res.scales, res.zeros, res.g_idx, res.perm):
            t.record_stream(main)
    bad = torch.cat([st for st, _ in pending.values()]).cpu().tolist()
    _lib.check_device()  # a kernel whose bounded wait expired left incomplete outputs
    out = {}
    for (grp, (_, res)), b in zip(pending.items(), bad):
        out[grp] = redo(grp, hs[grp]) if b else res
    return out


def quantize_layer_gptq(weights: dict, inputs: dict, cfg: QuantConfig, shapes=LLAMA2_7B,
                        timed: bool = False, concurrent: bool = True):
    """GPTQ for every linear of a layer set.  ``inputs[group]`` = bf16 X on the device.

    Linears that share an input also share the Hessian factor, and their rows
    are independent, so they are swept together as one row-stacked matrix
    (more rows in flight per column step).

    With ``concurrent`` (ignored when ``timed``, whose per-phase events need
    one stream) each input group's factor and sweep run on a stream of their
    own as soon as that group's H is formed, largest group first: its
    latency-bound factor leaves and small GEMMs overlap the remaining H
    accumulations and the other groups' GEMMs and sweeps.
    """
    if timed or not concurrent:
        return _quantize_layer_gptq_sequential(weights, inputs, cfg, shapes, timed)
    def form(grp, chunk):
        x = inputs[grp]
        d = x.shape[1]
        h = torch.empty((d, d), dtype=torch.float32, device=x.device)
        stats.syrk_into(h, x, accumulate=False, token_chunk=chunk)
        return h

    def prepare(grp, h):
        return factor_hessian_attempt0(h, cfg)

    def fused(grp, side):
        return factor_from_activations_attempt0(inputs[grp], cfg, side, RESERVED_SMS)

    def work(grp, state):
        f, status = state
        return status, gptq_sweep(_stack(weights, _members(shapes, grp)), f.u, f.perm, cfg)

    def redo(grp, h):
        f = factor_hessian(form(grp, None) if h is None else h, cfg)
        return gptq_sweep(_stack(weights, _members(shapes, grp)), f.u, f.perm, cfg)

    sizes = _chain_sizes(inputs, shapes)
    first = max(sizes, key=lambda g: sizes[g])
    use_fused = FACTOR_FROM_ACTIVATIONS and _fused_factor_ok(inputs[first], cfg)
    results: dict[str, SweepResult] = {}
    for grp, res in _run_groups_concurrently(sizes, form, work, redo, prepare,
                                             fused=fused if use_fused else None).items():
        results.update(_split_rows(res, _members(shapes, grp)))
    return results, LayerTimes()


def _quantize_layer_gptq_sequential(weights, inputs, cfg, shapes, timed):
    tm = _Timer(timed)
    factors: dict[str, HessianFactor] = {}
    for grp, x in inputs.items():
        tm.mark(f"stats:{grp}")
        d = x.shape[1]
        h = torch.empty((d, d), dtype=torch.float32, device=x.device)
        stats.syrk_into(h, x, accumulate=False)
        tm.mark(f"factor:{grp}")
        factors[grp] = factor_hessian(h, cfg)
        del h
    results: dict[str, SweepResult] = {}
    for grp in inputs:
        members = _members(shapes, grp)
        tm.mark(f"sweep:{grp}")
        f = factors[grp]
        results.update(_split_rows(gptq_sweep(_stack(weights, members), f.u, f.perm, cfg), members))
    tm.mark("end")
    return results, _collect(tm)


def quantize_layer_qronos(weights: dict, inputs_float: dict, inputs_quant: dict,
                          cfg: QuantConfig, shapes=LLAMA2_7B, timed: bool = False,
                          concurrent: bool = True):
    """Qronos for every linear: ``h = Xt^T Xt``, ``g = X^T Xt`` per input group;
    linears sharing an input are updated together as one row-stacked matrix.
    ``concurrent`` as for :func:`quantize_layer_gptq`."""
    if timed or not concurrent:
        return _quantize_layer_qronos_sequential(weights, inputs_float, inputs_quant, cfg, shapes,
                                                 timed)
    gs = {}

    def form(grp, chunk):
        xq = inputs_quant[grp]
        d = xq.shape[1]
        h = torch.empty((d, d), dtype=torch.float32, device=xq.device)
        stats.syrk_into(h, xq, accumulate=False, token_chunk=chunk)
        return h

    def late(grp, chunk):
        # the cross term is read only by the sweep, so it is formed while the
        # group's factor runs
        xq = inputs_quant[grp]
        d = xq.shape[1]
        g = torch.empty((d, d), dtype=torch.float32, device=xq.device)
        stats.gemm_tn_into(g, inputs_float[grp], xq, accumulate=False, token_chunk=chunk)
        gs[grp] = g

    def prepare(grp, h):
        return factor_hessian_attempt0(h, cfg, want_hd=True)

    def work(grp, state):
        f, status = state
        w = _stack(weights, _members(shapes, grp))
        return status, qronos_quantize(w, w, None, gs[grp], cfg, factor=f)

    def redo(grp, h):
        f = factor_hessian(h, cfg, want_hd=True)
        w = _stack(weights, _members(shapes, grp))
        return qronos_quantize(w, w, None, gs[grp], cfg, factor=f)

    results = {}
    for grp, res in _run_groups_concurrently(_chain_sizes(inputs_quant, shapes), form, work, redo,
                                             prepare, late).items():
        results.update(_split_rows(res, _members(shapes, grp)))
    return results, LayerTimes()


def _quantize_layer_qronos_sequential(weights, inputs_float, inputs_quant, cfg, shapes, timed):
    tm = _Timer(timed)
    facts = {}
    for grp, xq in inputs_quant.items():
        tm.mark(f"stats:{grp}")
        d = xq.shape[1]
        h = torch.empty((d, d), dtype=torch.float32, device=xq.device)
        g = torch.empty((d, d), dtype=torch.float32, device=xq.device)
        stats.syrk_into(h, xq, accumulate=False)
        stats.gemm_tn_into(g, inputs_float[grp], xq, accumulate=False)
        tm.mark(f"factor:{grp}")
        facts[grp] = (factor_hessian(h, cfg, want_hd=True), g)
        del h
    results = {}
    for grp in inputs_quant:
        members = _members(shapes, grp)
        tm.mark(f"sweep:{grp}")
        f, g = facts[grp]
        w = _stack(weights, members)
        results.update(_split_rows(qronos_quantize(w, w, None, g, cfg, factor=f), members))
    tm.mark("end")
    return results, _collect(tm)


_COPY_STREAMS: dict[int, tuple] = {}


def _copy_streams():
    dev = torch.cuda.current_device()
    if dev not in _COPY_STREAMS:
        _COPY_STREAMS[dev] = (torch.cuda.Stream(), torch.cuda.Stream())
    return _COPY_STREAMS[dev]


# Activations cross PCIe in chunks of this many tokens; each chunk's H
# contribution is accumulated as soon as it lands (bit-identical to one
# launch over all tokens), so H is ready right after the last chunk.
HOST_TOKEN_CHUNK = 32768


def quantize_layer_gptq_host(weights_host: dict, inputs_host: dict, cfg: QuantConfig,
                             shapes=LLAMA2_7B):
    """GPTQ layer set from host buffers to host results.

    Activations (bf16) and weights (float32) are copied from (pinned) host
    memory on a copy stream, longest chain first (the order of
    :func:`quantize_layer_gptq`), activations in ``HOST_TOKEN_CHUNK``-token
    chunks whose H contribution is accumulated while the next chunk is in
    flight, then the group's weights straight into one row-stacked device
    buffer (for the last group, its weights first).  Each group's factor and
    sweep overlap the later groups' transfers, so what is left after the last
    byte arrives is the shortest chain: one small group's last H chunk,
    factor and sweep.  Codes, scales and zeros stream back on a second copy
    stream.  The results equal the device-resident
    :func:`quantize_layer_gptq` bit for bit.  Returns ``({name: (codes,
    scales, zeros, g_idx, perm)}, {"h2d": bytes, "d2h": bytes})`` with host
    tensors.
    """
    compute = torch.cuda.current_stream()
    h2d, d2h = _copy_streams()
    start = torch.cuda.Event()
    start.record(compute)
    h2d.wait_event(start)
    nbytes = {"h2d": 0, "d2h": 0}
    sizes = _chain_sizes(inputs_host, shapes)
    order = sorted(sizes, key=lambda g: sizes[g], reverse=True)
    dev_x, dev_w, ready_x, ready_w = {}, {}, {}, {}

    def copy_x(grp):
        src = inputs_host[grp]
        dst = torch.empty(src.shape, dtype=src.dtype, device="cuda")
        evs = []
        for t0 in range(0, src.shape[0], HOST_TOKEN_CHUNK):
            t1 = min(src.shape[0], t0 + HOST_TOKEN_CHUNK)
            dst[t0:t1].copy_(src[t0:t1], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
            evs.append((t0, t1, ev))
        nbytes["h2d"] += src.numel() * src.element_size()
        dev_x[grp], ready_x[grp] = dst, evs

    def copy_w(grp):
        members = _members(shapes, grp)
        n = weights_host[members[0][0]].shape[1]
        wdev = torch.empty((sum(m for _, m in members), n), dtype=torch.float32, device="cuda")
        r0 = 0
        for name, m in members:
            wsrc = weights_host[name]
            wdev[r0:r0 + m].copy_(wsrc, non_blocking=True)
            nbytes["h2d"] += wsrc.numel() * wsrc.element_size()
            r0 += m
        ev = torch.cuda.Event()
        ev.record(h2d)
        dev_w[grp], ready_w[grp] = wdev, ev

    with torch.cuda.stream(h2d):
        for grp in order:
            if grp == order[-1]:
                copy_w(grp)
                copy_x(grp)
            else:
                copy_x(grp)
                copy_w(grp)
    out = {}
    for grp in order:
        x = dev_x[grp]
        x.record_stream(compute)
        d = x.shape[1]
        h = torch.empty((d, d), dtype=torch.float32, device="cuda")
        for i, (t0, t1, ev) in enumerate(ready_x[grp]):
            compute.wait_event(ev)
            stats.syrk_into(h, x[t0:t1], accumulate=i > 0)
        f = factor_hessian(h, cfg)
        del h
        compute.wait_event(ready_w[grp])
        w = dev_w[grp]
        w.record_stream(compute)
        res = gptq_sweep(w, f.u, f.perm, cfg)
        done = torch.cuda.Event()
        done.record(compute)
        d2h.wait_event(done)
        with torch.cuda.stream(d2h):
            host = []
            for t in (res.codes, res.scales, res.zeros, res.g_idx, res.perm):
                t.record_stream(d2h)
                hb = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                hb.copy_(t, non_blocking=True)
                nbytes["d2h"] += t.numel() * t.element_size()
                host.append(hb)
        r0 = 0
        for name, m in _members(shapes, grp):
            out[name] = (host[0][r0:r0 + m], host[1][r0:r0 + m], host[2][r0:r0 + m], host[3],
                         host[4])
            r0 += m
    fin = torch.cuda.Event()
    fin.record(d2h)
    compute.wait_event(fin)
    return out, nbytes


def _collect(tm: _Timer) -> LayerTimes:
    t = LayerTimes()
    for label, ms in tm.spans():
        kind, _, what = label.partition(":")
        if kind == "stats":
            t.stats_ms += ms
            t.per_group_stats_ms[what] = ms
        elif kind == "factor":
            t.factor_ms += ms
        elif kind == "sweep":
            t.sweep_ms += ms
    return t
