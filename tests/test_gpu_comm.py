"""NCCL all-reduce through libgq's C ABI (gq_handle_create_nccl /
gq_allreduce_sum_f32): one rank on one GPU, and -- when the process sees two
or more GPUs -- two ranks in spawned processes, one per GPU, summing
token-shard partial Hessians."""

import os
import pickle

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

from jax_gptq_b200 import distributed as D
from jax_gptq_b200 import stats


def test_single_rank_allreduce_is_identity():
    uid = D.CommHandle.unique_id()
    h = D.CommHandle(torch.cuda.current_device(), uid, 1, 0)
    try:
        t = torch.randn(1000, device="cuda")
        ref = t.clone()
        h.allreduce_sum_(t)
        torch.cuda.synchronize()
        assert t.equal(ref)
        with pytest.raises(ValueError):
            h.allreduce_sum_(t.double())
    finally:
        h.close()


def _rank(rank, world, uid, out_dir):
    torch.cuda.set_device(rank)
    from jax_gptq_b200 import _lib
    _lib.lib()
    gen = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn((4096, 384), generator=gen, device="cuda").to(torch.bfloat16)
    t0, t1 = D.shard_range(x.shape[0], rank, world)
    h = torch.empty((384, 384), dtype=torch.float32, device="cuda")
    stats.syrk_into(h, x[t0:t1], accumulate=False)
    hs = h.clone()
    handle = D.CommHandle(rank, uid, world, rank)
    try:
        handle.allreduce_sum_(h)
        handle.allreduce_sym_(hs)  # packed upper triangle
        torch.cuda.synchronize()
        full = torch.empty_like(h)
        stats.syrk_into(full, x, accumulate=False)
        rel = (torch.linalg.norm(h - full) / torch.linalg.norm(full)).item()
        rel_sym = (torch.linalg.norm(hs - full) / torch.linalg.norm(full)).item()
        with open(os.path.join(out_dir, f"r{rank}.pkl"), "wb") as f:
            pickle.dump({"rel": rel, "h": h.cpu().numpy(), "rel_sym": rel_sym,
                         "hs": hs.cpu().numpy(), "sym_exact": bool(hs.equal(hs.t()))}, f)
    finally:
        handle.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_hessian_allreduce(tmp_path):
    world = 2
    uid = D.CommHandle.unique_id()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, world, uid, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0, p.exitcode
    outs = [pickle.load(open(tmp_path / f"r{r}.pkl", "rb")) for r in range(world)]
    for o in outs:
        assert o["rel"] < 1e-6, o["rel"]
        assert o["rel_sym"] < 1e-6 and o["sym_exact"], o["rel_sym"]
    assert np.array_equal(outs[0]["h"], outs[1]["h"])
    assert np.array_equal(outs[0]["hs"], outs[1]["hs"])


def test_single_rank_packed_symmetric_allreduce_is_identity():
    """gq_allreduce_sym_f32 with one rank: pack, all-reduce, unpack give back
    the symmetric input bit for bit, for a width that is not a multiple of
    128 and a leading dimension wider than the matrix."""
    uid = D.CommHandle.unique_id()
    h = D.CommHandle(torch.cuda.current_device(), uid, 1, 0)
    try:
        a = torch.randn(300, 300, device="cuda")
        buf = torch.zeros(300, 320, device="cuda")
        buf[:, :300] = a + a.t()
        ref = buf.clone()
        h.allreduce_sym_(buf[:, :300])
        torch.cuda.synchronize()
        assert buf.equal(ref)
    finally:
        h.close()


def test_single_rank_check_then_abort():
    """A healthy communicator reports no asynchronous error; after an abort
    (what a host watchdog does when a peer is lost) every collective on the
    handle fails at once with GQ_ENCCL instead of waiting."""
    from jax_gptq_b200 import _lib
    uid = D.CommHandle.unique_id()
    h = D.CommHandle(torch.cuda.current_device(), uid, 1, 0)
    try:
        h.check()
        h.abort()
        t = torch.randn(64, device="cuda")
        with pytest.raises(_lib.GQError, match="aborted"):
            h.allreduce_sum_(t)
        with pytest.raises(_lib.GQError, match="aborted"):
            h.check()
    finally:
        h.close()


def _factor_rank(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    from jax_gptq_b200 import layerset as LS
    from jax_gptq_b200.config import QuantConfig
    from jax_gptq_b200.gptq_ref import factor_hessian
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        x = LS.synth_activations(8192, 4096, 31)[0]
        h = torch.empty((4096, 4096), dtype=torch.float32, device="cuda")
        stats.syrk_into(h, x, accumulate=False)
        cfg = QuantConfig(w_bits=4, group_size=128, ordering_mode="diag_h", semantics="intended")
        # split the diagonal blocks down to 1024 wide: 4096 -> 2048 -> 1024
        D.FACTOR_SPLIT_MIN_N = 1024
        f, status = D.factor_hessian_sharded_attempt0(h, cfg)
        torch.cuda.synchronize()
        whole = factor_hessian(h, cfg)
        rel = (torch.linalg.norm(f.u - whole.u) / torch.linalg.norm(whole.u)).item()
        # token-shard partial H summed through the packed upper triangle, once
        # synchronously and once asynchronously with the unpack on a side stream
        t0, t1 = D.shard_range(x.shape[0], rank, world)
        hp = torch.empty_like(h)
        stats.syrk_into(hp, x[t0:t1], accumulate=False)
        hp2 = hp.clone()
        D.allreduce_sym_(hp)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        work = D.allreduce_sym_(hp2, async_op=True)
        with torch.cuda.stream(side):
            work.wait()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        sym_rel = max((torch.linalg.norm(t - h) / torch.linalg.norm(h)).item() for t in (hp, hp2))
        with open(os.path.join(out_dir, f"f{rank}.pkl"), "wb") as fh:
            pickle.dump({"status": int(status.item()), "rel": rel,
                         "u": f.u.cpu().numpy(), "perm_equal": bool(f.perm.equal(whole.perm)),
                         "sym_rel": sym_rel, "sym_exact": bool(hp.equal(hp.t())),
                         "sym_same": bool(hp.equal(hp2)), "hp": hp.cpu().numpy()}, fh)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_split_factor(tmp_path):
    """The factor with its split products divided across two GPUs (NCCL
    all-gathers, three levels of splits): the same U on both ranks, bit for
    bit, within 1e-5 of the unsplit factor.  Also the token-sharded H summed
    through its packed upper triangle (``allreduce_sym_``, synchronous and
    asynchronous): within 1e-6 of the whole H, exactly symmetric, the same
    on both ranks."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    world = 2
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_factor_rank, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0, p.exitcode
    outs = [pickle.load(open(tmp_path / f"f{r}.pkl", "rb")) for r in range(world)]
    for o in outs:
        assert o["status"] == 0 and o["perm_equal"] and o["rel"] <= 1e-5, o["rel"]
        assert o["sym_rel"] < 1e-6 and o["sym_exact"] and o["sym_same"], o["sym_rel"]
    assert np.array_equal(outs[0]["u"], outs[1]["u"])
    assert np.array_equal(outs[0]["hp"], outs[1]["hp"])
