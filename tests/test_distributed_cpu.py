"""Host-side multi-rank logic of ``jax_gptq_b200.distributed`` on CPU.

Pure functions (sharding, LPT schedule) are checked directly; the collective
paths run as two gloo ranks in spawned processes on 127.0.0.1.
"""

import datetime
import itertools
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from jax_gptq_b200 import distributed as D
from jax_gptq_b200 import layerset as LS


@pytest.mark.parametrize("n,world,align", [(0, 1, 1), (1, 4, 1), (100, 3, 32), (4096, 8, 32),
                                           (22016, 3, 32), (97, 5, 1), (64, 8, 32)])
def test_shard_range_tiles_rows(n, world, align):
    spans = [D.shard_range(n, r, world, align) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and a0 <= a1
    for a, b in spans:
        assert a % align == 0 or a == n
    sizes = [b - a for a, b in spans]
    blocks = [-(-s // align) for s in sizes]
    assert max(blocks) - min(blocks) <= 1


def test_shard_range_rejects_bad_arguments():
    with pytest.raises(ValueError):
        D.shard_range(10, 2, 2)
    with pytest.raises(ValueError):
        D.shard_range(-1, 0, 1)


@pytest.mark.parametrize("n,world", [(14336, 8), (5504, 2), (1280, 3), (2816, 4), (128, 8),
                                     (640, 8)])
def test_split_factor_row_spans_cover_and_balance(n, world):
    """The split factor's per-rank row slices: contiguous, 128-aligned,
    covering [0, n); the triangular partition gives every rank about the same
    lower-triangular work (row i costs ~i) where the rows allow it."""
    for tri in (False, True):
        spans = D._row_spans(n, world, triangular=tri)
        assert len(spans) == world and spans[0][0] == 0 and spans[-1][1] == n
        for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
            assert a1 == b0
        for r0, r1 in spans:
            assert r0 <= r1 and r0 % 128 == 0 and (r1 % 128 == 0 or r1 == n)
    if n >= 2048 * world // 2:
        work = [(r1 - r0) * (r0 + r1) / 2 for r0, r1 in D._row_spans(n, world, True)]
        assert max(work) <= 1.2 * (n * n / 2) / world, work


def test_lpt_assign_is_a_deterministic_partition_within_the_lpt_bound():
    rng = np.random.default_rng(0)
    for world in (1, 2, 3, 4):
        costs = {f"u{i}": float(c) for i, c in enumerate(rng.uniform(1, 10, 7))}
        a = D.lpt_assign(costs, world)
        assert a == D.lpt_assign(dict(reversed(list(costs.items()))), world)
        flat = [k for ks in a for k in ks]
        assert sorted(flat) == sorted(costs)
        makespan = max(sum(costs[k] for k in ks) for ks in a)
        best = min(max(sum(costs[k] for k, r in zip(costs, lab) if r == i) for i in range(world))
                   for lab in itertools.product(range(world), repeat=len(costs)))
        assert makespan <= (4.0 / 3.0 - 1.0 / (3 * world)) * best + 1e-9


def test_layer_set_cost_orders_models():
    c7 = D.layer_set_cost(LS.LLAMA2_7B, 262144)
    c70 = D.layer_set_cost(LS.LLAMA3_70B, 262144)
    assert 0 < c7 < c70


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        res = {}
        # token-sharded Gram matrix: partial sums all-reduced in place
        rng = np.random.default_rng(7)
        x = rng.standard_normal((1000, 48)).astype(np.float32)
        t0, t1 = D.shard_range(x.shape[0], rank, world)
        xl = x[t0:t1].astype(np.float64)
        h = torch.from_numpy((xl.T @ xl).astype(np.float32))
        assert D.rank_world() == (rank, world)
        w = D.allreduce_sum_(h, async_op=True)
        w.wait()
        res["h"] = h.numpy()
        # row gather of uneven shards, several dtypes
        m = 100
        full_f = torch.arange(m * 6, dtype=torch.float32).reshape(m, 6)
        full_u8 = (torch.arange(m * 5) % 251).to(torch.uint8).reshape(m, 5)
        full_v = torch.arange(m, dtype=torch.float32)
        r0, r1 = D.shard_range(m, rank, world, D.SWEEP_ROW_ALIGN)
        res["gf"] = D.gather_rows(full_f[r0:r1].clone(), m).numpy()
        res["gu"] = D.gather_rows(full_u8[r0:r1].clone(), m).numpy()
        res["gv"] = D.gather_rows(full_v[r0:r1].clone(), m).numpy()
        with pytest.raises(ValueError):
            D.gather_rows(full_f[:1].clone(), m)
        res["layers"] = D.layer_sets_for_rank(7, LS.LLAMA2_7B, 4096)
        res["tokens"] = D.tokens_for_rank(1001)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), res, allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0, p.exitcode
    outs = [np.load(tmp_path / f"rank{r}.npy", allow_pickle=True).item() for r in range(world)]
    rng = np.random.default_rng(7)
    x = rng.standard_normal((1000, 48)).astype(np.float32).astype(np.float64)
    h_ref = x.T @ x
    for o in outs:
        assert np.allclose(o["h"], h_ref, rtol=1e-5, atol=1e-3)
    assert np.array_equal(outs[0]["h"], outs[1]["h"])  # identical on every rank
    m = 100
    for o in outs:
        assert np.array_equal(o["gf"], np.arange(m * 6, dtype=np.float32).reshape(m, 6))
        assert np.array_equal(o["gu"], (np.arange(m * 5) % 251).astype(np.uint8).reshape(m, 5))
        assert np.array_equal(o["gv"], np.arange(m, dtype=np.float32))
    assert sorted(outs[0]["layers"] + outs[1]["layers"]) == list(range(7))
    assert not set(outs[0]["layers"]) & set(outs[1]["layers"])
    assert outs[0]["tokens"] == (0, 501) and outs[1]["tokens"] == (501, 1001)


def _worker_lost_peer(rank, world, port, store_port, out_dir):
    """Rank 1 misses the step-1 heartbeat and never joins the all-reduce."""
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    store = dist.TCPStore("127.0.0.1", store_port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=60))
    hb = D.Heartbeat(store, rank, world)
    res = {}
    hb.beat(0)
    hb.wait_all(0, timeout_s=30)
    if rank == 0:
        hb.beat(1)
        t0 = time.monotonic()
        try:
            hb.wait_all(1, timeout_s=1.0)
            res["heartbeat"] = "no error"
        except D.RankFailure as exc:
            res["heartbeat"] = str(exc)
        res["heartbeat_s"] = time.monotonic() - t0
        t0 = time.monotonic()
        try:
            D.allreduce_sum_(torch.ones(8))
            res["allreduce"] = "no error"
        except D.RankFailure as exc:
            res["allreduce"] = str(exc)
        res["allreduce_s"] = time.monotonic() - t0
        np.save(os.path.join(out_dir, "lost.npy"), res, allow_pickle=True)
        store.set("done", b"1")
        store.wait(["ack"])  # rank 0 hosts the store: keep it up until rank 1 has read "done"
    else:
        store.wait(["done"])  # stays alive (a lost peer, not a closed connection) until rank 0 is done
        store.set("ack", b"1")
    os._exit(0)  # no teardown collective with a peer that did not take part


def test_gloo_rank_that_never_contributes_is_detected(tmp_path):
    """Failure detection on the host: a missing heartbeat names the lost rank
    before the next launch, and a collective the lost rank never joins ends
    with RankFailure after the process group's timeout, not a hang."""
    world = 2
    ctx = mp.get_context("spawn")
    port, store_port = _free_port(), _free_port()
    procs = [ctx.Process(target=_worker_lost_peer, args=(r, world, port, store_port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0, p.exitcode
    res = np.load(tmp_path / "lost.npy", allow_pickle=True).item()
    assert "rank(s) [1]" in res["heartbeat"], res
    assert 0.9 <= res["heartbeat_s"] < 10, res
    assert "did not contribute" in res["allreduce"], res
    assert res["allreduce_s"] < 60, res
