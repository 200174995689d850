"""Benchmark: quantize a Llama-2-7B-shaped decoder layer set on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one layer set (q, k, v, o, gate, up, down) quantized with GPTQ
(4-bit, group 128, act-order, damp 0.01): H = X^T X over 262,144 bf16 tokens
for each of the four distinct layer inputs on the tcgen05 tensor cores, the
damped inverse-Cholesky factor per input, and the seven column sweeps.
Inputs are synthetic (seeded, generated on the device) and already resident
in HBM when the timed region starts; they total 12.2 GB, far above the
126 MB L2, so no flush is needed between steps.

Under torchrun each rank quantizes its own layer set (layer parallelism:
weak scaling, no data-path collective); ``value`` is seconds per layer for
the whole job: max-over-ranks step time / layers processed by all ranks.

Also reported: ``e2e`` (the same step through the host-buffer API
``quantize_layer_gptq_host``: activations and weights copied from pinned
host memory, codes/scales/zeros copied back, inside the timed region), the
live roofline of the H-accumulation kernel, Qronos on the same layer set
(3-bit), the pivoted-QR throughput, and a CPU baseline (the numpy oracle on
a bounded sample, extrapolated).

``--impl reference`` times the reference's own op sequence for this path
(h = x^T x, the five Cholesky attempts its process_hessian makes before
falling back, act-order, RTN) as a numpy port on the host cores, on a
bounded sample, extrapolated to seconds per layer.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TOKENS = 128 * 2048
METRIC = "7B-layer-set GPTQ+Qronos s/layer; H-accum TFLOP/s; pivoted-QR GFLOP/s"
WORKLOAD = "llama2-7b layer set (q,k,v,o 4096x4096; gate,up 11008x4096; down 4096x11008), " \
           "GPTQ 4-bit g128 act-order damp 0.01, H over 262144 bf16 tokens"
WORKLOAD_70B = "llama3-70b layer set (q,o 8192x8192; k,v 1024x8192; gate,up 28672x8192; " \
               "down 8192x28672), GPTQ 4-bit g128 act-order damp 0.01, H over 1048576 " \
               "Student-t bf16 tokens"


def _workload(args):
    """(shapes, weight std, activation kind, tokens, description) of --model."""
    from jax_gptq_b200 import layerset as LS
    if args.model == "llama3-70b":
        return LS.LLAMA3_70B, 0.01, "student_t", args.tokens or 256 * 4096, WORKLOAD_70B
    return LS.LLAMA2_7B, 0.02, "lognormal", args.tokens or TOKENS, WORKLOAD


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        # raw samples (one CSV per GPU); the JSON line carries their summary
        out = os.environ.get("GQ_CLOCKS_DIR", os.path.join(ROOT, "bench_clocks"))
        self.path = os.path.join(out, f"clocks_gpu{gpu_index}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU side

def _cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def reference_port_sample(shapes, sample_tokens=1024, sample_rows=512, chol_d=2048, seed=0):
    """Time the reference's op sequence on a bounded sample; extrapolate to s/layer.

    Per input group: h = x^T x (float32, stats.py:16) and the five Cholesky
    attempts of process_hessian (gptq_ref.py:80-89; each raises after the
    factorization, so the factorization cost is real), argsort of diag(h);
    per linear: RTN of the permuted weights (gptq_ref.py:152-155).
    """
    from oracle import gptq as og
    from oracle import quant as oq
    rng = np.random.default_rng(seed)
    total = 0.0
    dims = {}
    for _, _, n, grp in shapes:
        dims[grp] = n
    parts = {}
    for grp, d in dims.items():
        x = rng.standard_normal((sample_tokens, d)).astype(np.float32)
        t0 = time.perf_counter()
        h = x.T @ x
        t_h = time.perf_counter() - t0
        dc = min(chol_d, d)
        hs = h[:dc, :dc] + np.float32(0.01) * np.mean(np.diag(h[:dc, :dc])) * np.eye(dc, dtype=np.float32)
        t0 = time.perf_counter()
        for _ in range(5):
            np.linalg.cholesky(hs)
        t_c = time.perf_counter() - t0
        t0 = time.perf_counter()
        og.act_order_perm(h, "diag_h")
        t_p = time.perf_counter() - t0
        est = t_h * (TOKENS / sample_tokens) + t_c * (d / dc) ** 3 + t_p
        parts[f"stats+chol:{grp}"] = est
        total += est
    for name, m, n, grp in shapes:
        rows = min(sample_rows, m)
        w = (rng.standard_normal((rows, n)) * 0.02).astype(np.float32)
        perm = rng.permutation(n)
        t0 = time.perf_counter()
        og.gptq_forward_step_reference(w, perm, 4, 128, False)
        est = (time.perf_counter() - t0) * (m / rows)
        parts[f"rtn:{name}"] = est
        total += est
    return total, parts, (f"h = x^T x on {sample_tokens} tokens per input (x{TOKENS // sample_tokens}),"
                          f" 5 Cholesky attempts at d={chol_d} (x(d/{chol_d})^3), RTN on "
                          f"{sample_rows} rows per linear (x m/{sample_rows})")


def intended_port_sample(shapes, sample_tokens=2048, sample_rows=64, chol_d=1024, seed=0):
    """The oracle's intended GPTQ (the work the GPU step does) on a bounded sample."""
    from oracle import gptq as og
    rng = np.random.default_rng(seed + 1)
    total = 0.0
    dims = {}
    for _, _, n, grp in shapes:
        dims[grp] = n
    for grp, d in dims.items():
        x = rng.standard_normal((sample_tokens, d)).astype(np.float32)
        t0 = time.perf_counter()
        h = x.T @ x
        t_h = time.perf_counter() - t0
        dc = min(chol_d, d)
        t0 = time.perf_counter()
        og.process_hessian_intended(h[:dc, :dc].astype(np.float64) + np.eye(dc), "diag_h", 0.01,
                                    dtype=np.float32)
        t_f = time.perf_counter() - t0
        total += t_h * (TOKENS / sample_tokens) + t_f * (d / dc) ** 3
    for name, m, n, grp in shapes:
        rows = min(sample_rows, m)
        w = (rng.standard_normal((rows, n)) * 0.02).astype(np.float32)
        u = np.triu(rng.standard_normal((n, n)).astype(np.float32) * 1e-3) + np.eye(n, dtype=np.float32)
        t0 = time.perf_counter()
        og.gptq_sweep(w, u, np.arange(n), 4, 128, False, 128, np.float32)
        total += (time.perf_counter() - t0) * (m / rows)
    return total, (f"oracle intended GPTQ: H on {sample_tokens} tokens/input (x{TOKENS // sample_tokens}),"
                   f" damped factor at d={chol_d} (x(d/{chol_d})^3), sweep on {sample_rows} rows per "
                   f"linear (x m/{sample_rows})")


# ----------------------------------------------------------------------------- single linear

SINGLE_LINEAR = ("GPTQ on one 1024x1024 linear: W ~ N(0, 0.02^2) fp32, X 2048x1024 fp32 ~ N(0, 1) "
                 "with 8 channels x20, H = X^T X / n, damp 0.01, 4-bit asym g128, block 128, "
                 "no act-order, seed 0")


def _single_linear_inputs(seed=0, m=1024, n=1024, tokens=2048, n_outliers=8):
    """The single-linear configuration's inputs (numpy PCG64, the same bytes
    the oracle's generator makes)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    w = (rng.standard_normal((m, n)) * 0.02).astype(np.float32)
    x = rng.standard_normal((tokens, n)).astype(np.float32)
    cols = rng.choice(n, size=n_outliers, replace=False)
    x[:, cols] *= np.float32(20.0)
    return w, x


def run_single_linear(peaks, steps=20, warmup=3, cpu=True):
    """One linear end to end: H (fp32 activations), the damped factor and the
    sweep.  ``value`` = device-resident ms per linear; ``e2e`` = the same
    through the reference-facing calls h_g_from_activations ->
    process_hessian -> gptq_forward_step on host numpy arrays."""
    import torch
    from jax_gptq_b200 import QuantConfig, gptq_forward_step, h_g_from_activations
    from jax_gptq_b200 import process_hessian
    from jax_gptq_b200 import gptq_ref as G
    from jax_gptq_b200 import stats
    w, x = _single_linear_inputs(0)
    m, n = w.shape
    tokens = x.shape[0]
    cfg = QuantConfig(w_bits=4, group_size=128, sym=False, damp_percent=0.01,
                      ordering_mode="none", semantics="intended")
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    h = torch.empty((n, n), dtype=torch.float32, device="cuda")

    def step():
        stats.syrk_into(h, xd, accumulate=False)
        h.mul_(1.0 / tokens)
        f = G.factor_hessian(h, cfg)
        return G.gptq_sweep(wd, f.u, f.perm, cfg)

    ms = _time(step, steps, warmup)
    f = G.factor_hessian(h, cfg)
    sweep_ms = _time(lambda: G.gptq_sweep(wd, f.u, f.perm, cfg), steps, warmup)
    syrk_ms = _time(lambda: stats.syrk_into(h, xd, accumulate=False), steps, warmup)
    factor_ms = _time(lambda: G.factor_hessian(h, cfg), steps, warmup)

    # e2e: the reference's own call sequence on host arrays (each call copies in and out)
    def host_step():
        hh, _ = h_g_from_activations(x)
        hh = hh / np.float32(tokens)
        hinv, perm = process_hessian(hh, cfg)
        return gptq_forward_step(w, hinv, perm, cfg), hh, hinv, perm

    for _ in range(warmup):
        host_step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        out, hh, hinv, perm = host_step()
    e2e_s = (time.perf_counter() - t0) / steps
    h2d = x.nbytes + hh.nbytes + w.nbytes + hinv.nbytes + perm.nbytes
    d2h = hh.nbytes + hinv.nbytes + perm.nbytes + out.nbytes

    sweep_bytes = 4 * m * n + 4 * n * n + 4 * m * n + m * n // 2 + 8 * m * (n // 128)
    hbm = peaks["hbm_gbs"]
    res = {
        "workload": SINGLE_LINEAR, "value": ms, "unit": "ms/linear",
        "phases_ms": {"h": syrk_ms, "factor": factor_ms, "sweep": sweep_ms},
        "e2e": {"value": e2e_s * 1e3, "unit": "ms/linear", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h),
                "path": "h_g_from_activations -> process_hessian -> gptq_forward_step on numpy"},
        "roofline": {"bound": "hbm", "kernel": "gq_gptq_sweep (1024 x 1024)",
                     "achieved": sweep_bytes / (sweep_ms / 1e3) / 1e9, "peak": hbm,
                     "unit": "GB/s", "frac": sweep_bytes / (sweep_ms / 1e3) / 1e9 / hbm,
                     "algorithmic": f"{sweep_bytes} bytes per sweep (W, U, dequant, packed codes, "
                                    "scales/zeros)",
                     "note": "latency-bound: a chain of 1024 dependent columns; the trailing "
                             "updates are 0.94 GFLOP of 3xTF32 GEMMs"},
    }
    if cpu:
        from oracle import gptq as og
        with _all_host_threads():
            t_cpu = []
            for _ in range(2):
                t0 = time.perf_counter()
                hc = (x.T @ x) / np.float32(tokens)
                u, perm_c, _ = og.process_hessian_intended(hc, "none", 0.01, dtype=np.float32)
                og.gptq_sweep(w, u, perm_c, 4, 128, False, 128, np.float32)
                t_cpu.append(time.perf_counter() - t0)
        res["cpu_baseline"] = {"value": min(t_cpu) * 1e3, "unit": "ms/linear",
                               "cores": _cpu_cores(), "kind": "port",
                               "sample": "the whole configuration, not extrapolated: the oracle's "
                                         "float32 H, damped Cholesky factor and GPTQ sweep"}
    return res


def qronos_port_sample(shapes, sample_tokens=2048, sample_rows=64, dc=1024, seed=0):
    """The oracle's Qronos (the work the GPU does) on a bounded sample: h and g
    on ``sample_tokens`` tokens (x tokens / sample), the damped factor at
    d = ``dc`` (x (d/dc)^3), and the update of ``sample_rows`` rows at d = dc
    given that factor (x (m/rows)(d/dc)^2: its products are m d^2)."""
    from oracle import gptq as og
    from oracle import qronos as oqn
    rng = np.random.default_rng(seed + 2)
    total = 0.0
    dims, rows = {}, {}
    for _, m, n, grp in shapes:
        dims[grp] = n
        rows[grp] = rows.get(grp, 0) + m
    for grp, d in dims.items():
        x = rng.standard_normal((sample_tokens, d)).astype(np.float32)
        xt = (x + 0.05 * rng.standard_normal(x.shape)).astype(np.float32)
        t0 = time.perf_counter()
        h = xt.T @ xt
        g = x.T @ xt
        t_hg = time.perf_counter() - t0
        hs, gs = h[:dc, :dc].astype(np.float32), g[:dc, :dc].astype(np.float32)
        t0 = time.perf_counter()
        u, perm, _ = og.process_hessian_intended(hs, "diag_h", 0.01, dtype=np.float32)
        hd = og.damped_permuted(hs, perm, 0.01, np.float32)
        t_f = time.perf_counter() - t0
        w = (rng.standard_normal((sample_rows, dc)) * 0.02).astype(np.float32)
        t0 = time.perf_counter()
        oqn.qronos_intended(w, w, hs, gs, 3, 128, False, dtype=np.float32, factor=(u, perm, hd))
        t_u = time.perf_counter() - t0
        total += (t_hg * (TOKENS / sample_tokens) + t_f * (d / dc) ** 3 +
                  t_u * (rows[grp] / sample_rows) * (d / dc) ** 2)
    return total, (f"oracle Qronos: h and g on {sample_tokens} tokens/input "
                   f"(x{TOKENS // sample_tokens}), factor at d={dc} (x(d/{dc})^3), update of "
                   f"{sample_rows} rows at d={dc} (x(m/{sample_rows})(d/{dc})^2)")


def qr_cpu_baseline(n=4096, sample_n=1024):
    """The oracle's exact pivoted QR (the reference's eager path at panel 1,
    the factorization the intended GPU path computes) on a ``sample_n``
    matrix of the benchmark's construction, scaled by (n / sample_n)^3; plus
    LAPACK sgeqp3 through scipy on the full matrix (a library reference)."""
    import scipy.linalg as sl
    from oracle import inputs as oin
    from oracle import qr as oqr
    with _all_host_threads():
        a_s = oin.qr_matrix(1, sample_n, sample_n)
        t0 = time.perf_counter()
        oqr.exact_pivoted_qr(a_s, "largest")
        t_s = time.perf_counter() - t0
        a = oin.qr_matrix(1, n, n)
        t0 = time.perf_counter()
        sl.qr(a, mode="r", pivoting=True)
        t_l = time.perf_counter() - t0
    return {"value": t_s * (n / sample_n) ** 3 * 1e3, "unit": "ms", "cores": _cpu_cores(),
            "kind": "port",
            "sample": f"extrapolated from the oracle's exact QRCP of the {sample_n}^2 matrix of "
                      f"the same construction, x(n/{sample_n})^3",
            "lapack_sgeqp3_ms": t_l * 1e3,
            "lapack_note": f"scipy LAPACK sgeqp3 on the full {n}^2 matrix (library, measured)"}


def parity_sample(weights, inputs, cfg, shapes, rows=32):
    """Sampled parity of the timed configuration, outside the timed region:
    the first ``rows`` rows of o_proj (d = 4096) and down_proj (d = 11008)
    against the oracle's float32 sweep with the same factor (codes equal
    except rows whose first differing code is a rounding tie, counted), and a
    256 x 256 tile of the d = 11008 H against a float64 sum of the same bf16
    columns."""
    import torch
    from jax_gptq_b200 import layerset as LS
    from jax_gptq_b200 import stats
    from jax_gptq_b200.gptq_ref import factor_hessian
    from oracle import gptq as og
    from oracle import quant as oq
    tie_tol = 1e-5
    results, _ = LS.quantize_layer_gptq(weights, inputs, cfg, shapes)
    qmin = oq.qrange(cfg.w_bits, cfg.sym)[0]
    out = {"rows_per_linear": rows, "tie_tol": tie_tol}
    ok = True
    flips = 0
    for name, grp in (("o_proj", "attn_out"), ("down_proj", "mlp_out")):
        x = inputs[grp]
        d = x.shape[1]
        h = torch.empty((d, d), dtype=torch.float32, device="cuda")
        stats.syrk_into(h, x, accumulate=False)
        f = factor_hessian(h, cfg)
        u, perm = f.u.cpu().numpy(), f.perm.cpu().numpy()
        w = weights[name][:rows].cpu().numpy()
        with _all_host_threads():
            ref = og.gptq_sweep(w, u, perm, cfg.w_bits, cfg.group_size, cfg.sym, 128, np.float32,
                                return_pre=True)
        got = results[name].codes[:rows].cpu().numpy().astype(np.float32)[:, perm] + qmin
        diff = got != ref["q"][:, perm]
        bad = np.flatnonzero(diff.any(axis=1))
        dist = 0.0
        if bad.size:
            first = diff[bad].argmax(axis=1)
            pre = ref["pre"][bad, first].astype(np.float64)
            dist = float(np.max(np.abs(pre - np.floor(pre) - 0.5)))
        flips += int(bad.size)
        ok &= dist <= tie_tol
        out[name] = {"tie_flip_rows": int(bad.size), "codes_differing": int(diff.sum()),
                     "max_first_diff_dist": dist}
        if grp == "mlp_out":
            xr = x[:, :256].float().cpu().numpy().astype(np.float64)
            href = xr.T @ xr
            hg = h[:256, :256].cpu().numpy().astype(np.float64)
            dn = np.sqrt(np.diag(href))
            worst = float(np.max(np.abs(hg - href) / np.outer(dn, dn)))
            out["h_tile_worst_normalized"] = worst
            ok &= worst <= 1e-5
        del h, f
    out["tie_flips"] = flips
    out["pass"] = bool(ok)
    return out


# ----------------------------------------------------------------------------- distributed

def _dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def _barrier(world):
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(v: float, world: int) -> float:
    if world <= 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- arms

def _all_host_threads():
    """A context that lets numpy's BLAS use every host core this process may
    run on (torchrun sets OMP_NUM_THREADS=1 for its ranks)."""
    from threadpoolctl import threadpool_limits
    return threadpool_limits(limits=_cpu_cores())


def run_reference(args, world, rank):
    if rank != 0:
        return
    from jax_gptq_b200.layerset import LLAMA2_7B
    times, walls, samples = [], [], None
    with _all_host_threads():
        from threadpoolctl import threadpool_info
        blas_threads = max([i.get("num_threads", 0) for i in threadpool_info()] or [0])
        for i in range(args.warmup + args.steps):
            w0 = time.perf_counter()
            t, parts, samples = reference_port_sample(LLAMA2_7B, seed=i)
            if i >= args.warmup:
                times.append(t)
                walls.append(time.perf_counter() - w0)
    v = statistics.mean(times)
    cores = _cpu_cores()
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "s/layer", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        # the wall time of each timed step: the bounded sample actually run
        "ms_per_step": statistics.mean(walls) * 1000.0,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOAD, "tokens": TOKENS,
                                        "semantics": "reference: x^T x, the five Cholesky "
                                                     "attempts its process_hessian makes, "
                                                     "act-order, RTN (what the reference runs)"},
        "value_kind": "extrapolated: each step times a bounded sample of one layer set and "
                      "scales each part to the full layer set (see cpu_baseline.sample)",
        "cpu_baseline": {"value": v, "unit": "s/layer", "cores": cores, "kind": "port",
                         "blas_threads": blas_threads,
                         "sample": "extrapolated from " + samples, "cpu": _cpu_model()},
        "e2e": {"value": v, "unit": "s/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "numpy port of the reference's own CPU op sequence (JAX is not installable "
                "offline), BLAS on every host core; the value is whole-host seconds per layer "
                "set, the same at every N (the N GPU ranks share one host)",
    }
    print(json.dumps(line), flush=True)


def run_kernel_only(args):
    """``--only syrk``: just the H-accumulation kernel on [tokens, dim];
    ``--only gemmtn``: just the Qronos cross term G = X^T Xt (profiling runs)."""
    import torch
    from jax_gptq_b200 import _lib
    from jax_gptq_b200 import layerset as LS
    from jax_gptq_b200 import stats
    _lib.lib()
    args.tokens = args.tokens or TOKENS
    x, std = LS.synth_activations(args.tokens, args.dim, 7)
    h = torch.empty((args.dim, args.dim), dtype=torch.float32, device="cuda")
    if args.only == "gemmtn":
        xt = LS.perturb_activations(x, std, 0.05, 9)
        fn = lambda: stats.gemm_tn_into(h, x, xt, accumulate=False)
        flops = LS.gemm_flops(args.tokens, args.dim)
    else:
        fn = lambda: stats.syrk_into(h, x, accumulate=False)
        flops = LS.syrk_flops(args.tokens, args.dim)
    ms = _time(fn, args.steps, args.warmup)
    print(json.dumps({"kernel": args.only, "tokens": args.tokens, "d": args.dim, "ms": ms,
                      "tflops": flops / (ms / 1e3) / 1e12}), flush=True)


def _time(fn, steps: int, warmup: int) -> float:
    """Milliseconds per call of ``fn`` on the current stream (CUDA events)."""
    import torch
    for _ in range(warmup):
        fn()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(max(steps, 1)):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / max(steps, 1)


def run_component(args):
    """``--only gemm|factor|sweep``: one component in isolation (profiling runs).

    gemm:   C[m, n] += -A[m, k] B[n, k]^T on the 3xTF32 tensor-core kernel
            (beta 1: the sweep's lazy update shape);
    factor: damped inverse-Cholesky factor of a --dim x --dim H (from 4 * dim tokens);
    sweep:  GPTQ sweep of an --m x --dim weight with that factor."""
    import torch
    from jax_gptq_b200 import _arrays as A
    from jax_gptq_b200 import _lib
    from jax_gptq_b200 import layerset as LS
    from jax_gptq_b200 import stats
    from jax_gptq_b200.config import QuantConfig
    from jax_gptq_b200.gptq_ref import factor_hessian, gptq_sweep
    _lib.lib()
    out = {"kernel": args.only}
    if args.only == "gemm":
        m, n, k = args.m, args.n or args.dim, args.k
        a = torch.randn(m, k, device="cuda")
        b = torch.randn(n, k, device="cuda")
        c = torch.randn(m, n, device="cuda")
        ms = _time(lambda: _lib.call("gq_gemm_f32_tc", 1, m, n, k, -1.0, A.ptr(a), k, A.ptr(b), k,
                                     1.0, A.ptr(c), n, 0, A.stream()), args.steps, args.warmup)
        out.update(m=m, n=n, k=k, ms=ms, tflops=2.0 * m * n * k / (ms / 1e3) / 1e12,
                   c_gbs=8.0 * m * n / (ms / 1e3) / 1e9)
    else:
        d = args.dim
        x, _ = LS.synth_activations(4 * d, d, 7)
        h = torch.empty((d, d), dtype=torch.float32, device="cuda")
        stats.syrk_into(h, x, accumulate=False)
        cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
        if args.only == "factor":
            ms = _time(lambda: factor_hessian(h, cfg), args.steps, args.warmup)
            out.update(d=d, ms=ms, gflops=(2.0 * d ** 3 / 3.0) / (ms / 1e3) / 1e9)
        else:
            f = factor_hessian(h, cfg)
            w = torch.randn(args.m, d, device="cuda") * 0.02
            ms = _time(lambda: gptq_sweep(w, f.u, f.perm, cfg), args.steps, args.warmup)
            out.update(m=args.m, d=d, ms=ms)
    print(json.dumps(out), flush=True)


def run_ours(args, world, rank, local):
    import torch
    from jax_gptq_b200 import _lib
    from jax_gptq_b200 import layerset as LS
    from jax_gptq_b200 import stats
    from jax_gptq_b200.config import QuantConfig

    _lib.lib()
    peaks, peak_kind = _peaks()
    shapes, w_std, act_kind, args.tokens, workload = _workload(args)
    skipped = []
    if args.model == "llama3-70b":
        # a second copy of the 112 GB of activations (pinned host or X~) does not fit
        for flag, what in (("no_e2e", "e2e"), ("no_qronos", "qronos"), ("no_qr", "qr")):
            if not getattr(args, flag):
                setattr(args, flag, True)
                skipped.append(what)
    dims = LS.group_dims(shapes)
    seed = 1000 * rank
    cfg = QuantConfig(w_bits=4, group_size=128, sym=False, damp_percent=0.01,
                      ordering_mode="diag_h", semantics="intended")
    weights = LS.synth_weights(shapes, w_std, seed)
    inputs, stds = {}, {}
    for i, (grp, d) in enumerate(dims.items()):
        inputs[grp], stds[grp] = LS.synth_activations(args.tokens, d, seed + 10 + i, kind=act_kind)
    x_gb = sum(x.numel() * x.element_size() for x in inputs.values()) / 1e9
    torch.cuda.synchronize()

    # --- headline: device-resident GPTQ layer set
    for _ in range(args.warmup):
        LS.quantize_layer_gptq(weights, inputs, cfg, shapes)
    sampler = ClockSampler(local)
    _barrier(world)
    sampler.start()
    launches0 = _lib.lib().gq_launch_count()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    torch.cuda.nvtx.range_push("gptq_layer_step")  # ncu --nvtx-include selects these launches
    for _ in range(args.steps):
        LS.quantize_layer_gptq(weights, inputs, cfg, shapes)
    torch.cuda.nvtx.range_pop()
    e1.record()
    _barrier(world)
    launches = (_lib.lib().gq_launch_count() - launches0) // max(args.steps, 1)
    clocks = sampler.stop()
    ms = _max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    s_per_layer = ms / 1000.0 / world

    # --- phase breakdown (one extra timed step)
    LS.quantize_layer_gptq(weights, inputs, cfg, shapes, concurrent=False)  # warm its buffers
    _, phases = LS.quantize_layer_gptq(weights, inputs, cfg, shapes, timed=True)

    # --- the sweeps against both of their bounds: the lazy-update flops on
    # the 3xTF32 tensor-core GEMM (ceiling: the same kernel on a large square
    # product, timed here) and the algorithmic HBM bytes
    sweep_flop = float(sum(m * n * (n - 128) for _, m, n, _ in shapes))
    sweep_bytes = float(sum(8.5 * m * n + 8 * m * (n // 128) + 4 * n * n for _, m, n, _ in shapes))
    from jax_gptq_b200 import _arrays as A
    ga = torch.randn(4096, 4096, device="cuda")
    gb = torch.randn(4096, 4096, device="cuda")
    gc = torch.empty(4096, 4096, device="cuda")
    g_ms = _time(lambda: _lib.call("gq_gemm_f32_tc", 1, 4096, 4096, 4096, 1.0, A.ptr(ga), 4096,
                                   A.ptr(gb), 4096, 0.0, A.ptr(gc), 4096, 0, A.stream()), 5, 2)
    ceiling = 2.0 * 4096 ** 3 / (g_ms / 1e3) / 1e12
    del ga, gb, gc
    sw_s = phases.sweep_ms / 1e3
    sweep_roof = {
        "ms_all_linears_sequential": phases.sweep_ms,
        "tflops": sweep_flop / sw_s / 1e12, "gemm_ceiling_tflops": ceiling,
        "frac_of_gemm_ceiling": sweep_flop / sw_s / 1e12 / ceiling,
        "gbs": sweep_bytes / sw_s / 1e9, "frac_hbm": sweep_bytes / sw_s / 1e9 / peaks["hbm_gbs"],
        "algorithmic": f"sum m*n*(n-128) = {sweep_flop:.4g} flops (3xTF32 lazy updates); "
                       f"sum 8.5mn + 8m(n/128) + 4n^2 = {sweep_bytes:.4g} bytes",
        "note": "each column's quantize -> error -> update is a dependent chain (about 200 "
                "cycles per column per row), so neither bound is reached"}

    # --- roofline of the H-accumulation kernel (tcgen05), timed live on its stream
    syrk_ms, syrk_flop = [], []
    for grp, x in inputs.items():
        d = x.shape[1]
        h = torch.empty((d, d), dtype=torch.float32, device="cuda")
        for _ in range(2):
            stats.syrk_into(h, x, accumulate=False)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        reps = 3
        for _ in range(reps):
            stats.syrk_into(h, x, accumulate=False)
        b.record()
        torch.cuda.synchronize()
        syrk_ms.append(a.elapsed_time(b) / reps)
        syrk_flop.append(LS.syrk_flops(args.tokens, d))
        del h
    del x
    h_tflops = sum(syrk_flop) / (sum(syrk_ms) / 1e3) / 1e12
    # roofline of the dominant launch: the largest-d H accumulation
    top = max(range(len(syrk_ms)), key=lambda i: syrk_ms[i])
    top_d = list(dims.values())[top]
    top_tflops = syrk_flop[top] / (syrk_ms[top] / 1e3) / 1e12
    traffic = args.syrk_traffic
    if traffic is None and top_d == 11008:
        # DRAM bytes of one d = 11008 launch from an ncu capture at 32768 tokens
        # (10.575 GB read: each wave of the 946 pair tiles streams the X columns
        # of its tile group; 0.265 GB of H written), scaled to this launch's tokens
        traffic = 10.575e9 * args.tokens / 32768 + 0.265e9
    peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    roofline = {"bound": "tensor",
                "kernel": f"gq_tc gemm_tn_pair_kernel (H = X^T X, symmetric 256 x 256 tiles "
                          f"on CTA pairs), d = {top_d}",
                "achieved": top_tflops, "peak": peak, "unit": "TFLOP/s", "frac": top_tflops / peak,
                "peak_kind": f"{peak_kind} bf16 sustained (kernel timed inside a long step)",
                "peak_burst": peaks.get("bf16_tflops"),
                "frac_burst": top_tflops / peaks.get("bf16_tflops", peak),
                "algorithmic": f"tokens*d*(d+1) = {syrk_flop[top]:.4g} flops per launch",
                "traffic": traffic,
                "traffic_note": "dram read+write bytes per launch (ncu, scaled by tokens)"}

    # --- e2e through the host-buffer API
    e2e = None
    if not args.no_e2e:
        w_host = {k: v.cpu().pin_memory() for k, v in weights.items()}
        x_host = {k: v.cpu().pin_memory() for k, v in inputs.items()}
        for _ in range(max(1, min(args.warmup, 2))):
            LS.quantize_layer_gptq_host(w_host, x_host, cfg, shapes)
        _barrier(world)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            out, nbytes = LS.quantize_layer_gptq_host(w_host, x_host, cfg, shapes)
        b.record()
        _barrier(world)
        e2e_ms = _max_over_ranks(a.elapsed_time(b) / args.steps, world)
        # the link's own rate for pinned host-to-device copies of the largest
        # input (the step's lower bound is its h2d bytes at this rate)
        big = max(x_host.values(), key=lambda t: t.numel())
        dev = torch.empty(big.shape, dtype=big.dtype, device="cuda")
        dev.copy_(big, non_blocking=True)
        a.record()
        for _ in range(3):
            dev.copy_(big, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        link_gbs = 3 * big.numel() * big.element_size() / (a.elapsed_time(b) / 1e3) / 1e9
        del dev
        e2e = {"value": e2e_ms / 1000.0 / world, "unit": "s/layer",
               "h2d_bytes_per_step": nbytes["h2d"], "d2h_bytes_per_step": nbytes["d2h"],
               "h2d_link_gbs": link_gbs,
               "h2d_bound_s_per_step": nbytes["h2d"] / (link_gbs * 1e9)}
        del w_host, x_host

    # --- Qronos on the same layer set (3-bit), Xt = X + N(0, (0.05 sigma_c)^2)
    qronos = None
    if not args.no_qronos:
        qcfg = QuantConfig(w_bits=3, group_size=128, sym=False, damp_percent=0.01,
                           ordering_mode="diag_h", semantics="intended")
        xq = {g: LS.perturb_activations(inputs[g], stds[g], 0.05, seed + 50 + i)
              for i, g in enumerate(inputs)}
        LS.quantize_layer_qronos(weights, inputs, xq, qcfg, shapes)
        _barrier(world)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        qsteps = max(1, min(args.steps, 3))
        for _ in range(qsteps):
            LS.quantize_layer_qronos(weights, inputs, xq, qcfg, shapes)
        b.record()
        _barrier(world)
        q_ms = _max_over_ranks(a.elapsed_time(b) / qsteps, world)
        LS.quantize_layer_qronos(weights, inputs, xq, qcfg, shapes, concurrent=False)
        _, qph = LS.quantize_layer_qronos(weights, inputs, xq, qcfg, shapes, timed=True)
        qronos = {"s_per_layer": q_ms / 1000.0 / world, "steps": qsteps,
                  "workload": "Qronos 3-bit g128 act-order on the same layer set; h = Xt^T Xt, "
                              "g = X^T Xt, Xt = X + N(0, (0.05 sigma_c)^2), seed 2 offsets",
                  "phases_ms": {"h_and_g": qph.stats_ms, "factor": qph.factor_ms,
                                "qronos_sweeps": qph.sweep_ms}}
        gx, gq_ = inputs["mlp_out"], xq["mlp_out"]
        gd = gx.shape[1]
        gbuf = torch.empty((gd, gd), dtype=torch.float32, device="cuda")
        g_ms = _time(lambda: stats.gemm_tn_into(gbuf, gx, gq_, accumulate=False), 3, 1)
        g_tf = LS.gemm_flops(args.tokens, gd) / (g_ms / 1e3) / 1e12
        qronos["roofline"] = {
            "bound": "tensor", "kernel": f"gq_tc gemm_tn_pair_kernel (G = X^T Xt, full 256 x 256 "
                                         f"tiles on CTA pairs), d = {gd}",
            "achieved": g_tf, "peak": peak, "unit": "TFLOP/s", "frac": g_tf / peak,
            "frac_burst": g_tf / peaks.get("bf16_tflops", peak),
            "peak_kind": f"{peak_kind} bf16 sustained",
            "algorithmic": f"2*tokens*d^2 = {LS.gemm_flops(args.tokens, gd):.4g} flops per launch",
            "ms": g_ms}
        del gbuf, gx, gq_, xq

    # --- blocked pivoted QR (4096 x 4096 fp32, panel 64)
    qr = None
    if not args.no_qr:
        try:
            import importlib
            BQ = importlib.import_module("jax_gptq_b200.pallas.blocked_pivoted_qr")
            qr = BQ.benchmark(n=4096, panel=64, reps=2)
            # the BLAS-2 part reads the trailing block once per pivot step
            blas2 = 4.0 * sum(i * i for i in range(1, qr["n"] + 1))
            qr["blas2_bytes"] = blas2
            for v in qr.values():
                if isinstance(v, dict) and "ms" in v:
                    v["blas2_gbs"] = blas2 / (v["ms"] / 1e3) / 1e9
            il = qr["intended_largest"]
            qr["roofline"] = {
                "bound": "hbm", "kernel": "gq_qrcp intended/largest: the per-pivot exposed-row "
                                          "pass over the trailing block (BLAS-2)",
                "achieved": il["blas2_gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": il["blas2_gbs"] / peaks["hbm_gbs"],
                "algorithmic": "4 * sum_{i=1..n} i^2 = 91.7 GB per factorization (one trailing-"
                               "block read per pivot step), over the whole factorization's time",
                "note": "the 64 MB matrix stays in the 126 MB L2, so these reads come from L2; "
                        "the pivot chain (4096 dependent steps) bounds the factorization"}
            if rank == 0 and not args.no_cpu_baseline:
                qr["cpu_baseline"] = qr_cpu_baseline(qr["n"])
        except Exception as exc:  # report, do not hide
            qr = {"error": repr(exc)[:200]}

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        with _all_host_threads():
            v, sample = intended_port_sample(shapes)
            if qronos is not None:
                qv, qsample = qronos_port_sample(shapes)
                qronos["cpu_baseline"] = {"value": qv, "unit": "s/layer", "cores": _cpu_cores(),
                                          "kind": "port", "sample": "extrapolated from " + qsample}
        cpu = {"value": v, "unit": "s/layer", "cores": _cpu_cores(), "kind": "port",
               "sample": "extrapolated from " + sample, "cpu": _cpu_model()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": s_per_layer, "unit": "s/layer", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 in / f32 accumulate (H); f32 sweep", "data": "synthetic",
            "config": {"workload": workload, "tokens": args.tokens, "layers_per_rank": 1,
                       "semantics": "intended: damped inverse-Cholesky factor + GPTQ column "
                                    "sweep (the reference's own chol path returns the identity "
                                    "factor and RTN, strictly less work; the reference arm "
                                    "times that op sequence)",
                       "parallelism": f"layer-parallel x{world}",
                       "l2": f"inputs ({x_gb:.1f} GB) larger than L2; no flush",
                       "skipped_for_memory": skipped},
            "phases_ms": {"h_accum": phases.stats_ms, "factor": phases.factor_ms,
                          "sweeps": phases.sweep_ms, "h_by_group": phases.per_group_stats_ms},
            "h_accum": {"tflops": h_tflops, "ms_by_group": dict(zip(dims, syrk_ms)),
                        "tflop_per_layer_distinct_inputs": sum(syrk_flop) / 1e12,
                        "tflop_per_layer_per_linear":
                            sum(LS.syrk_flops(args.tokens, n) for _, _, n, _ in shapes) / 1e12},
            "roofline": roofline, "sweep_roofline": sweep_roof, "e2e": e2e,
            "gpu_launches": int(launches), "clocks": clocks,
            "qronos": qronos, "qr": qr, "cpu_baseline": cpu,
        }
        if not args.no_parity:
            line["parity"] = parity_sample(weights, inputs, cfg, shapes)
    del weights, inputs
    torch.cuda.empty_cache()
    if rank == 0 and not args.no_single and args.model == "llama2-7b":
        line["single_linear"] = run_single_linear(peaks, cpu=not args.no_cpu_baseline)
    # strong scaling of one layer set over all ranks (token-sharded H + row-sharded sweep)
    if not args.no_sharded and args.model == "llama2-7b":
        sharded = {}
        for model in ("llama2-7b", "llama3-70b"):
            if model == "llama3-70b" and args.no_70b:
                continue
            _barrier(world)
            sharded[model] = sharded_layer_set(model, None, 2, 1, world, rank, local)
        if rank == 0:
            line["sharded"] = sharded
    if rank == 0:
        print(json.dumps(line), flush=True)


def sharded_layer_set(model, tokens, steps, warmup, world, rank, local, check=True):
    """One layer set spread over all ranks (strong scaling): every rank holds
    a 1/N token shard of each input and all weights; the partial H are summed
    by NCCL all-reduce, every rank factors the summed H, and each sweeps its
    1/N of the rows (outputs gathered).  Returns the measured figures (rank 0)
    or None."""
    import torch
    import torch.distributed as dist
    from jax_gptq_b200 import _lib
    from jax_gptq_b200 import distributed as D
    from jax_gptq_b200 import layerset as LS
    from jax_gptq_b200 import stats
    from jax_gptq_b200.config import QuantConfig
    from jax_gptq_b200.gptq_ref import factor_hessian, gptq_sweep

    class _A:
        pass
    a = _A()
    a.model, a.tokens = model, tokens
    shapes, w_std, act_kind, tokens, workload = _workload(a)
    dims = LS.group_dims(shapes)
    cfg = QuantConfig(w_bits=4, group_size=128, sym=False, damp_percent=0.01,
                      ordering_mode="diag_h", semantics="intended")
    weights = LS.synth_weights(shapes, w_std, 0)
    t0, t1 = D.shard_range(tokens, rank, world)
    inputs = {grp: LS.synth_activations(t1 - t0, d, 10 + i + 100 * rank, kind=act_kind)[0]
              for i, (grp, d) in enumerate(dims.items())}
    torch.cuda.synchronize()
    for _ in range(warmup):
        D.quantize_layer_gptq_sharded(weights, inputs, cfg, shapes)
    _barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        D.quantize_layer_gptq_sharded(weights, inputs, cfg, shapes)
    e1.record()
    _barrier(world)
    ms = _max_over_ranks(e0.elapsed_time(e1) / max(steps, 1), world)

    # per-phase figures from a sequential, instrumented pass (one stream),
    # taken twice: the timed steps allocated their buffers on side streams,
    # whose cached blocks the caller's stream does not reuse, so the first
    # pass would time fresh allocations; the second pass is reported
    for _pass in range(2):
        phases = {}
        factors = {}
        for grp, x in inputs.items():
            d = x.shape[1]
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            h = torch.empty((d, d), dtype=torch.float32, device="cuda")
            _barrier(world)
            ev[0].record()
            stats.syrk_into(h, x, accumulate=False)
            ev[1].record()
            # every rank's partial H is complete before the all-reduce is timed, so
            # the figure is the transfer, not the wait for the slowest rank's SYRK
            _barrier(world)
            ar0 = torch.cuda.Event(enable_timing=True)
            ar0.record()
            D.allreduce_sym_(h)  # packed upper triangle: pack, all-reduce, unpack
            ev[2].record()
            f, fst = D.factor_hessian_sharded_attempt0(h, cfg)
            if int(fst.item()) != 0:  # the same on every rank: redo with more damping
                f = factor_hessian(h, cfg)
            ev[3].record()
            members = [(nm, m) for nm, m, _, g in shapes if g == grp]
            w = D._stacked(weights, members)
            r0, r1 = D.shard_range(w.shape[0], rank, world, D.SWEEP_ROW_ALIGN)
            res = gptq_sweep(w[r0:r1], f.u, f.perm, cfg)
            ev[4].record()
            torch.cuda.synchronize()
            t = [ev[0].elapsed_time(ev[1]), ar0.elapsed_time(ev[2]), ev[2].elapsed_time(ev[3]),
                 ev[3].elapsed_time(ev[4])]
            t = [_max_over_ranks(v, world) for v in t]
            ar_bytes = 4 * _lib.lib().gq_sym_packed_size(d)
            # NCCL's bus-bandwidth convention for all-reduce: 2 (N - 1) / N of the buffer per rank
            bus = ar_bytes * 2 * (world - 1) / world / (t[1] / 1e3) / 1e9 if world > 1 else None
            phases[grp] = {"d": d, "rows_per_rank": r1 - r0, "h_partial_ms": t[0],
                           "allreduce_ms": t[1], "allreduce_bytes": ar_bytes,
                           "allreduce_busbw_gbs": bus, "factor_ms": t[2], "sweep_ms": t[3]}
            factors[grp] = (h, f, res, (r0, r1), w)

    parity = None
    if check:
        # (1) all-reduced H against the ranks' partial tiles summed in rank order
        grp0 = min(dims, key=lambda g: dims[g])
        h, f, res, (r0, r1), w = factors[grp0]
        x = inputs[grp0]
        tile = torch.empty((256, 256), dtype=torch.float32, device="cuda")
        stats.syrk_into(tile, x[:, :256].contiguous(), accumulate=False)
        parts = [torch.empty_like(tile) for _ in range(world)]
        if world > 1:
            dist.all_gather(parts, tile)
        else:
            parts = [tile]
        ref = sum(p.double() for p in parts)
        got = h[:256, :256].double()
        h_rel = float((got - ref).abs().max() / ref.abs().max())
        # (2) this rank's row shard against the unsharded sweep (same U): bit-exact
        whole = gptq_sweep(w, f.u, f.perm, cfg)
        rows_equal = bool(torch.equal(whole.codes[r0:r1], res.codes) and
                          torch.equal(whole.dequant[r0:r1], res.dequant))
        flags = torch.tensor([0.0 if rows_equal else 1.0, h_rel], dtype=torch.float64,
                             device="cuda")
        if world > 1:
            dist.all_reduce(flags, op=dist.ReduceOp.MAX)
        parity = {"group": grp0, "h_tile_max_rel_vs_rank_sum": float(flags[1].item()),
                  "row_shards_bitexact_vs_unsharded": bool(flags[0].item() == 0.0),
                  "pass": bool(flags[0].item() == 0.0 and flags[1].item() <= 1e-6)}
    del factors, inputs, weights
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    top = max(phases, key=lambda g: phases[g]["d"])
    return {"workload": workload, "tokens": tokens, "n_gpus": world, "s_per_layer": ms / 1e3,
            "steps": steps, "warmup": warmup, "per_group": phases,
            "factor_ms_sum": sum(p["factor_ms"] for p in phases.values()),
            "factor_note": f"factors of d >= {D.FACTOR_SHARD_MIN_D} split their products "
                           "by rows across the ranks, recursively for diagonal blocks at "
                           f"least {D.FACTOR_SPLIT_MIN_N} wide; narrower diagonal blocks "
                           "are factored by every rank; timed on a second, warm pass",
            "limiter": f"the d = {phases[top]['d']} group's chain: its H shard, "
                       f"{phases[top]['allreduce_bytes'] / 1e9:.2f} GB all-reduce and factor "
                       f"({phases[top]['factor_ms']:.1f} ms)",
            "parity": parity}


def run_sharded(args, world, rank, local):
    """``--strategy sharded``: one layer set over all ranks, as the headline line."""
    sampler = ClockSampler(local)
    sampler.start()
    r = sharded_layer_set(args.model, args.tokens, args.steps, args.warmup, world, rank, local)
    clocks = sampler.stop()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": r["s_per_layer"], "unit": "s/layer", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["s_per_layer"] * 1e3,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, on device)",
            "config": {"workload": r["workload"], "tokens": r["tokens"],
                       "parallelism": f"token-sharded H (NCCL all-reduce) + row-sharded sweep x{world}",
                       "l2_flush": "inputs larger than L2"},
            "sharded": r, "clocks": clocks}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per input (default: 262144 for llama2-7b, 1048576 for llama3-70b)")
    ap.add_argument("--model", choices=["llama2-7b", "llama3-70b"], default="llama2-7b",
                    help="layer set: the 7B set is the headline; the 70B block (Student-t "
                         "activations, 112 GB of them) runs GPTQ only")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-qronos", action="store_true")
    ap.add_argument("--no-qr", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the sampled parity check")
    ap.add_argument("--no-single", action="store_true", help="skip the single-linear workload")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the strong-scaling (token/row-sharded) layer-set runs")
    ap.add_argument("--no-70b", action="store_true",
                    help="skip the 70B block in the strong-scaling runs")
    ap.add_argument("--syrk-traffic", type=float, default=None,
                    help="DRAM bytes per H-accumulation launch from an ncu capture")
    ap.add_argument("--only", choices=["all", "syrk", "gemmtn", "qr", "gemm", "factor", "sweep"],
                    default="all",
                    help="syrk: time only the H kernel on [--tokens, --dim]; qr: only the "
                         "pivoted QR on a --dim x --dim matrix; gemm / factor / sweep: one "
                         "component (profiling)")
    ap.add_argument("--m", type=int, default=12288)
    ap.add_argument("--n", type=int, default=None)
    ap.add_argument("--k", type=int, default=128)
    ap.add_argument("--dim", type=int, default=4096)
    ap.add_argument("--panel", type=int, default=64)
    ap.add_argument("--qr-variants", default=None,
                    help="comma-separated subset of the QR variants for --only qr "
                         "(intended_largest, reference_largest, intended_rankdef_smallest, "
                         "intended_rankdef_largest)")
    ap.add_argument("--strategy", choices=["layer", "sharded"], default="layer",
                    help="layer: each rank quantizes its own layer set (weak scaling, no "
                         "collective); sharded: one layer set over all ranks (strong scaling)")
    args = ap.parse_args()
    if args.only != "all":
        import torch
        torch.cuda.set_device(0)
        if args.only in ("syrk", "gemmtn"):
            run_kernel_only(args)
        elif args.only in ("gemm", "factor", "sweep"):
            run_component(args)
        else:
            import importlib
            BQ = importlib.import_module("jax_gptq_b200.pallas.blocked_pivoted_qr")
            print(json.dumps({"kernel": "qr", **BQ.benchmark(n=args.dim, panel=args.panel,
                                                            variants=args.qr_variants,
                                                            reps=max(1, args.steps))}), flush=True)
        return
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = _dist_init()
    try:
        if args.strategy == "sharded":
            run_sharded(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
