"""Multi-GPU partitioning of the quantization path (one process per GPU).

The reference runs on a single device; these are the ways its path splits
across GPUs, each tied to an independence in the computation:

* token-sharded statistics -- ``H = sum_r X_r^T X_r`` (``stats.py:4-18`` is a
  sum over tokens): every rank forms the Gram matrix of its own tokens on its
  tensor cores, then one in-place float32 all-reduce per input group (NCCL
  over NVLink; the reduction of one group overlaps the next group's SYRK);
* split factor -- the inverse-Cholesky recursion of the identical reduced H
  (``gptq_ref.py:44-93``) has its products divided by rows across the ranks
  and joined by all-gathers, recursively for wide diagonal blocks; narrow
  diagonal blocks are factored by every rank (deterministic), so the ranks'
  ``U`` agree bit for bit (``shard_factor=False``: every rank factors the
  whole H, nothing is communicated);
* row-sharded sweep -- rows of ``W`` are independent once ``U`` and the
  permutation are fixed (``gptq_ref.py:136-155`` quantizes row-wise), so each
  rank sweeps a contiguous block of rows with no communication, and one
  all-gather assembles the outputs when the caller wants them whole;
* layer parallelism -- whole layer sets are independent units and go to ranks
  by a longest-processing-time-first schedule on their cost, no collective.

Pivoted QR does not shard (a global argmax per pivot step); it runs as
independent replicas.

Process groups are the caller's (``torch.distributed`` with the NCCL backend
on GPUs); every function takes an optional ``group``.  The collective helpers
also accept CPU tensors under gloo.
"""

from __future__ import annotations

from typing import Hashable

import torch

from . import _arrays as A
from . import _lib
from . import stats
from .config import QuantConfig
from .gptq_ref import SweepResult, factor_hessian, gptq_sweep

SWEEP_ROW_ALIGN = 32  # the sweep kernel runs one warp per 32 rows


def _dist():
    import torch.distributed as dist
    return dist


def rank_world(group=None) -> tuple[int, int]:
    """(rank, world size) in ``group``; (0, 1) without an initialized process group."""
    dist = _dist()
    if not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_range(n: int, rank: int, world: int, align: int = 1) -> tuple[int, int]:
    """Contiguous block ``[start, stop)`` of ``n`` items owned by ``rank``.

    Items are dealt in blocks of ``align`` (only the last block may be short);
    the first ``n_blocks % world`` ranks get one block more.  Ranges of all
    ranks tile ``[0, n)`` in rank order; a rank may get an empty range.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    if n < 0 or align < 1:
        raise ValueError(f"bad n={n} or align={align}")
    nb = -(-n // align)
    base, extra = divmod(nb, world)
    b0 = rank * base + min(rank, extra)
    b1 = b0 + base + (1 if rank < extra else 0)
    return min(n, b0 * align), min(n, b1 * align)


def lpt_assign(costs: dict[Hashable, float], world: int) -> list[list[Hashable]]:
    """Longest-processing-time-first schedule: units in decreasing cost (ties
    by key order), each to the currently least-loaded rank (ties to the lower
    rank).  Deterministic, so every rank computes the same assignment."""
    if world < 1:
        raise ValueError("world must be >= 1")
    loads = [0.0] * world
    out: list[list[Hashable]] = [[] for _ in range(world)]
    for key, cost in sorted(costs.items(), key=lambda kv: (-float(kv[1]), str(kv[0]))):
        r = min(range(world), key=lambda i: (loads[i], i))
        out[r].append(key)
        loads[r] += float(cost)
    return out


# Relative throughputs used by the layer-set cost model (only compared with
# each other): bf16 tensor-core SYRK, fp32 (3xTF32) tensor-core factor and
# sweep GEMMs.
_BF16_RATE = 1.0e15
_F32_RATE = 1.7e14


def layer_set_cost(shapes, tokens: int) -> float:
    """Modelled seconds for one GPTQ layer set: SYRK per input group
    (tokens * d^2), inverse-Cholesky factor (2 d^3 / 3) and sweep GEMMs
    (m * n^2 per group of row-stacked linears)."""
    dims: dict[str, int] = {}
    rows: dict[str, int] = {}
    for _name, m, n, grp in shapes:
        dims[grp] = n
        rows[grp] = rows.get(grp, 0) + m
    t = 0.0
    for grp, d in dims.items():
        t += tokens * d * d / _BF16_RATE
        t += (2.0 * d ** 3 / 3.0) / _F32_RATE
        t += rows[grp] * d * d / _F32_RATE
    return t


class RankFailure(RuntimeError):
    """A peer rank failed, left, or never contributed to a collective.

    Raised on the surviving ranks, on the host, between launches: by
    :class:`Heartbeat` when a rank's beat for a step does not arrive in time,
    and by the collective helpers when the process group's timeout (or a
    broken connection) ends a collective with an error."""


def _collective(what: str, fn):
    try:
        return fn()
    except RankFailure:
        raise
    except RuntimeError as exc:  # DistBackendError and gloo/NCCL timeouts derive from it
        raise RankFailure(f"{what} failed: a peer rank did not contribute ({exc})") from exc


class _Work:
    """Wraps an async collective's work handle so ``wait`` raises RankFailure."""

    def __init__(self, what: str, work):
        self._what, self._work = what, work

    def wait(self):
        return _collective(self._what, self._work.wait)


def allreduce_sum_(t: torch.Tensor, group=None, async_op: bool = False):
    """In-place sum over the ranks of ``group``; returns the work handle when
    ``async_op`` (None for a single rank).  A rank that never joins ends the
    call (or the handle's ``wait``) with :class:`RankFailure` once the
    process group's timeout expires."""
    dist = _dist()
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return None
    work = _collective("all_reduce", lambda: dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group,
                                                             async_op=async_op))
    return _Work("all_reduce", work) if async_op else work


class _SymWork:
    """An in-flight packed all-reduce of a symmetric matrix: ``wait`` makes
    the current stream wait for the sum, then unpacks it into the matrix on
    that stream (upper entries, mirrored)."""

    def __init__(self, work, packed: torch.Tensor, h: torch.Tensor):
        self._work, self._packed, self._h = work, packed, h

    def wait(self):
        if self._packed is None:  # already waited for and unpacked
            return
        self._work.wait()
        # the unpack may run on another stream than the one that allocated
        # the buffer: keep it from being reused before the unpack has read it
        self._packed.record_stream(torch.cuda.current_stream())
        d = self._h.shape[0]
        _lib.call("gq_sym_unpack_upper", A.ptr(self._packed), d, A.ptr(self._h),
                  self._h.stride(0), A.stream())
        self._packed = None


def allreduce_sym_(h: torch.Tensor, group=None, async_op: bool = False):
    """In-place sum over the ranks of ``group`` of a symmetric float32 CUDA
    matrix through its packed upper triangle (``gq_sym_pack_upper``: about
    half the bytes of the full matrix).  The result is exactly symmetric.
    Returns the work handle when ``async_op`` (its ``wait`` also unpacks, on
    the stream current at that time); None for a single rank."""
    dist = _dist()
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return None
    if h.dtype != torch.float32 or not h.is_cuda or h.dim() != 2 or h.shape[0] != h.shape[1] \
            or h.stride(1) != 1:
        raise ValueError("allreduce_sym_ needs a square float32 CUDA matrix with unit column stride")
    d = h.shape[0]
    packed = torch.empty((_lib.lib().gq_sym_packed_size(d),), dtype=torch.float32, device=h.device)
    _lib.call("gq_sym_pack_upper", A.ptr(h), d, h.stride(0), A.ptr(packed), A.stream())
    work = _SymWork(allreduce_sum_(packed, group, async_op=True), packed, h)
    if async_op:
        return work
    work.wait()
    return None


class Heartbeat:
    """Host-side liveness check between steps, through a ``torch.distributed``
    key-value store (``TCPStore`` / ``FileStore``).

    Each rank calls :meth:`beat` with the step it is about to start and then
    :meth:`wait_all`, which returns once every rank has beaten for that step
    and raises :class:`RankFailure` naming the missing ranks after
    ``timeout_s``.  Ranks thus learn of a lost peer before launching the
    step's kernels or collectives, instead of inside a collective."""

    def __init__(self, store, rank: int, world: int, prefix: str = "gq/alive"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), b"1")

    def wait_all(self, step: int, timeout_s: float = 5.0, poll_s: float = 0.02) -> None:
        import time
        keys = [self._key(step, r) for r in range(self.world)]
        deadline = time.monotonic() + timeout_s
        while True:
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            if not missing:
                return
            if time.monotonic() >= deadline:
                raise RankFailure(f"step {step}: no heartbeat from rank(s) {missing} within "
                                  f"{timeout_s:g} s")
            time.sleep(poll_s)


def gather_rows(local: torch.Tensor, n_rows: int, group=None,
                align: int = SWEEP_ROW_ALIGN) -> torch.Tensor:
    """Inverse of row sharding: every rank passes its ``shard_range(n_rows,
    rank, world, align)`` block of rows; every rank gets the whole
    ``[n_rows, ...]`` tensor (one all-gather of equal-size padded blocks)."""
    rank, world = rank_world(group)
    r0, r1 = shard_range(n_rows, rank, world, align)
    if local.shape[0] != r1 - r0:
        raise ValueError(f"rank {rank}: expected {r1 - r0} rows, got {local.shape[0]}")
    if world == 1:
        return local
    spans = [shard_range(n_rows, r, world, align) for r in range(world)]
    rows_max = max(b - a for a, b in spans)
    tail = tuple(local.shape[1:])
    pad = torch.zeros((rows_max,) + tail, dtype=local.dtype, device=local.device)
    pad[: r1 - r0] = local
    blocks = [torch.empty_like(pad) for _ in range(world)]
    _collective("all_gather", lambda: _dist().all_gather(blocks, pad, group=group))
    return torch.cat([blocks[r][: b - a] for r, (a, b) in enumerate(spans)], dim=0)


def hessians_token_sharded(inputs_local: dict[str, torch.Tensor], group=None,
                           inputs_float_local: dict[str, torch.Tensor] | None = None):
    """``{group: H}`` (and ``{group: G}`` when float inputs are given) summed
    over the ranks' token shards, identical on every rank.

    ``inputs_local[grp]`` is this rank's ``[tokens_r, d]`` activations on the
    device (bf16 runs the tcgen05 SYRK).  Each group's all-reduce is issued
    asynchronously, so NCCL moves one group's H while the next SYRK runs."""
    A.require_cuda()
    hs: dict[str, torch.Tensor] = {}
    gs: dict[str, torch.Tensor] = {}
    pending = []
    for grp, x in inputs_local.items():
        d = x.shape[1]
        h = torch.empty((d, d), dtype=torch.float32, device=x.device)
        stats.syrk_into(h, x, accumulate=False)
        pending.append(allreduce_sym_(h, group, async_op=True))
        hs[grp] = h
        if inputs_float_local is not None:
            g = torch.empty((d, d), dtype=torch.float32, device=x.device)
            stats.gemm_tn_into(g, inputs_float_local[grp], x, accumulate=False)
            pending.append(allreduce_sum_(g, group, async_op=True))
            gs[grp] = g
    for w in pending:
        if w is not None:
            w.wait()
    return (hs, gs) if inputs_float_local is not None else hs


# Hessians at least this wide split their factor's products across the
# ranks (factor_hessian_sharded_attempt0); smaller ones are factored whole on
# every rank.
FACTOR_SHARD_MIN_D = 2048
# Below the top level, diagonal blocks at least this wide are split again
# across the ranks; narrower ones are factored whole by every rank (their
# products are too small to outweigh the all-gathers and copies: at
# d = 28672 on two B200s, 88 ms with this bound, 91 ms with 4096, 89 ms
# splitting the top level only, 109 ms unsplit).
FACTOR_SPLIT_MIN_N = 8192
_FACTOR_GROUPS: dict = {}


def _factor_group(group):
    """A second communicator over the same ranks for the factor's
    all-gathers, so they queue on their own NCCL stream and a group's H
    all-reduce never waits behind another group's factor (created once per
    process group, collectively, in the same order on every rank)."""
    dist = _dist()
    key = id(group) if group is not None else None
    if key not in _FACTOR_GROUPS:
        ranks = list(range(dist.get_world_size(group))) if group is None else \
            dist.get_process_group_ranks(group)
        _FACTOR_GROUPS[key] = dist.new_group(ranks)
    return _FACTOR_GROUPS[key]


def _split_n1(n: int, nb: int = 128) -> int:
    """The leading block of the factor's top split (a multiple of 128, about n/2)."""
    n1 = ((n // 2 + nb - 1) // nb) * nb
    return n - nb if n1 >= n else n1


def _inv_chol_split(b: torch.Tensor, o: int, n: int, world: int, mine: list, gather,
                    ws: torch.Tensor, status: torch.Tensor, min_split: int) -> None:
    """In-place inverse Cholesky of the n x n lower block of ``b`` at
    (o, o): on return it holds X = L^-1.  Split at n1 (``_split_n1``):
    X11 and X22 come from this function again while at least ``min_split``
    wide (else ``gq_inv_chol`` on every rank); L21 = B21 X11^T,
    T^T = L21 X11, the Schur update B22 -= L21 L21^T and X21 = -X22 T^T are
    each computed for this rank's row slices (``mine``: the rank indices
    whose slices this process computes) and combined by
    ``gather(part, rows_per_rank)`` into all ranks' rows.  At one level those
    four products are three quarters of the block's flops."""
    from . import gptq_ref as GR
    st = A.stream()
    call = GR._lib.call
    d = b.shape[1]
    if n < min_split:
        call("gq_inv_chol", A.ptr(b[o:, o:]), n, d, A.ptr(ws), ws.numel(), A.ptr(status), st)
        return
    n1 = _split_n1(n)
    n2 = n - n1
    p1 = o + n1  # first row / column of the trailing block
    _inv_chol_split(b, o, n1, world, mine, gather, ws, status, min_split)
    # row slices: equal for the products whose rows cost the same (L21, T^T);
    # for the lower-triangular outputs (Schur update, X21), whose row i costs
    # about i, boundaries at n2 sqrt(r / world) give every rank the same work
    flat = _row_spans(n2, world, triangular=False)
    tri = _row_spans(n2, world, triangular=True)

    def assemble(parts, spans, width):
        pmax = max(r1 - r0 for r0, r1 in spans)
        full = gather(parts, pmax)
        return torch.cat([full[r * pmax:r * pmax + (r1 - r0)] for r, (r0, r1) in
                          enumerate(spans)], dim=0) if len(spans) > 1 else full[:n2]

    def slot(spans, width):
        # rows past this rank's slice are padding for the equal-size gather,
        # dropped by assemble: left unwritten
        pmax = max(r1 - r0 for r0, r1 in spans)
        return torch.empty((pmax, width), dtype=torch.float32, device="cuda")

    def row_ptr(t, row, col=0):
        return A.ptr(t[row:, col:]) if row < t.shape[0] else A.ptr(t)

    def sgemm_tri(m, nn, k, alpha, a, lda, bb, ldb, beta, c, ldc, tri_mode):
        if m > 0 and nn > 0 and k > 0:
            call("gq_sgemm_tri", 0, 1, m, nn, k, float(alpha), a, lda, bb, ldb, float(beta), c,
                 ldc, tri_mode, st)

    xt = b[o:p1, o:p1].t().contiguous()           # X11^T (upper)
    # 1. L21 = B21 X11^T (B operand lower: tri 3)
    parts = {}
    for r in mine:
        r0, r1 = flat[r]
        out = slot(flat, n1)
        sgemm_tri(r1 - r0, n1, n1, 1.0, row_ptr(b, p1 + r0, o), d, A.ptr(b[o:, o:]), d, 0.0,
                  A.ptr(out), n1, 3)
        parts[r] = out
    l21 = assemble(parts, flat, n1)               # [n2, n1]
    # 2. T^T = L21 X11 (B = X11^T upper: tri 4)
    parts = {}
    for r in mine:
        r0, r1 = flat[r]
        out = slot(flat, n1)
        sgemm_tri(r1 - r0, n1, n1, 1.0, row_ptr(l21, r0), n1, A.ptr(xt), n1, 0.0, A.ptr(out), n1,
                  4)
        parts[r] = out
    tt = assemble(parts, flat, n1).t().contiguous()  # T [n1, n2]
    # 3. B22 -= L21 L21^T on this rank's rows: columns left of its diagonal
    #    block in full, the diagonal block's lower tiles
    parts = {}
    for r in mine:
        r0, r1 = tri[r]
        if r1 > r0 and r0 > 0:
            call("gq_sgemm", 0, 1, r1 - r0, r0, n1, -1.0, row_ptr(l21, r0), n1, A.ptr(l21), n1,
                 1.0, row_ptr(b, p1 + r0, p1), d, 0, st)
        if r1 > r0:
            call("gq_sgemm", 0, 1, r1 - r0, r1 - r0, n1, -1.0, row_ptr(l21, r0), n1,
                 row_ptr(l21, r0), n1, 1.0, row_ptr(b, p1 + r0, p1 + r0), d, 1, st)
        out = slot(tri, n2)
        out[:r1 - r0] = b[p1 + r0:p1 + r1, p1:o + n]
        parts[r] = out
    b[p1:o + n, p1:o + n] = assemble(parts, tri, n2)
    # only T is read after the recursion below: free X11^T and L21 first
    # (stream-ordered, so the pending kernels that read them are unaffected)
    del xt, l21, parts
    # 4. X22 = L22^-1
    _inv_chol_split(b, p1, n2, world, mine, gather, ws, status, min_split)
    # 5. X21 = -X22 T^T: rows [r0, r1) of the lower X22 are zero past column
    #    r1, so K stops there (no triangle of the call's own: tri 0)
    parts = {}
    for r in mine:
        r0, r1 = tri[r]
        out = slot(tri, n1)
        sgemm_tri(r1 - r0, n1, r1, -1.0, row_ptr(b, p1 + r0, p1), d, A.ptr(tt), n2, 0.0,
                  A.ptr(out), n1, 0)
        parts[r] = out
    b[p1:o + n, o:p1] = assemble(parts, tri, n1)


def _row_spans(n: int, world: int, triangular: bool, nb: int = 128) -> list:
    """Per rank, the rows [r0, r1) of an n-row product it computes: nb-aligned
    boundaries, equal counts, or (``triangular``) at n sqrt(r / world) so
    that the lower-triangular work (row i costs ~i) is split evenly."""
    import math
    bounds = [0]
    for r in range(1, world):
        x = n * (math.sqrt(r / world) if triangular else r / world)
        bounds.append(min(n, max(bounds[-1], int(-(-round(x) // nb)) * nb)))
    bounds.append(n)
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def _factor_top_split(h: torch.Tensor, cfg: QuantConfig, world: int, mine: list, gather,
                      min_split: int | None = None):
    """Attempt 0 of the damped inverse-Cholesky factor with its split
    products divided by output rows over ``world`` ranks (``_inv_chol_split``
    on B = J (H_perm + damp I) J, lower; blocks at least ``min_split`` wide,
    default ``FACTOR_SPLIT_MIN_N``, are split again below the top level).
    Returns the factor (U = J X J) and its device status word (0 = positive
    definite)."""
    from . import gptq_ref as GR
    GR._check_hessian(h, cfg)
    d = h.shape[0]
    st = A.stream()
    call = GR._lib.call
    perm = GR.act_order_perm(h, cfg.ordering_mode)
    b = A.empty((d, d))
    mean = A.empty((1,))
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    call("gq_hessian_prepare", A.ptr(h), d, h.stride(0), A.ptr(perm), float(cfg.damp_percent), 0,
         A.ptr(b), None, A.ptr(mean), st)
    lib = GR._lib.lib()
    n1 = _split_n1(d)
    ws = A.workspace(lib.gq_inv_chol_workspace_size(max(n1, d - n1)))
    inner = FACTOR_SPLIT_MIN_N if min_split is None else min_split
    # the top level is always split (the caller checked the width)
    _inv_chol_split(b, 0, d, world, mine, gather, ws, status, min(d, max(inner, 256)))
    u = A.empty((d, d))
    call("gq_reverse_lower", A.ptr(b), d, d, A.ptr(u), d, st)
    return GR.HessianFactor(u, perm, 0, None), status


def factor_hessian_sharded_attempt0(h: torch.Tensor, cfg: QuantConfig, group=None):
    """Attempt 0 of the damped factor (``gptq_ref.factor_hessian_attempt0``)
    with its products split by rows across the ranks of ``group``
    (``_inv_chol_split``): every rank passes the same (all-reduced) H and
    gets the same factor.  Hessians
    narrower than ``FACTOR_SHARD_MIN_D`` or a single rank use the unsplit
    factor.  Returns ``(factor, status)``; a non-zero status (damping too
    small) is the same on every rank, which then redo the group with the
    retrying factor."""
    from .gptq_ref import factor_hessian_attempt0
    rank, world = rank_world(group)
    if world == 1 or h.shape[0] < FACTOR_SHARD_MIN_D:
        return factor_hessian_attempt0(h, cfg)
    fgroup = _factor_group(group)

    def gather(parts, per):
        part = parts[rank]
        full = torch.empty((per * world,) + tuple(part.shape[1:]), dtype=part.dtype,
                           device=part.device)
        _collective("all_gather", lambda: _dist().all_gather_into_tensor(full, part, group=fgroup))
        return full

    return _factor_top_split(h, cfg, world, [rank], gather)


def factor_hessian_split_emulated(h: torch.Tensor, cfg: QuantConfig, world: int,
                                  min_split: int | None = None):
    """The sharded factor's arithmetic on one GPU: every rank's row slices
    computed in turn and concatenated instead of all-gathered (for tests)."""
    def gather(parts, per):
        return torch.cat([parts[r] for r in range(world)], dim=0)
    return _factor_top_split(A.to_device(h), cfg, world, list(range(world)), gather, min_split)


def _members(shapes, grp):
    return [(name, m) for name, m, _, g in shapes if g == grp]


def _stacked(weights: dict, members) -> torch.Tensor:
    return weights[members[0][0]] if len(members) == 1 else \
        torch.cat([weights[name] for name, _ in members], dim=0)


def quantize_layer_gptq_sharded(weights: dict, inputs_local: dict, cfg: QuantConfig, shapes,
                                group=None, gather: bool = True, concurrent: bool = True,
                                shard_factor: bool = True) -> dict[str, SweepResult]:
    """GPTQ for one layer set spread over the ranks of ``group``.

    ``inputs_local[grp]``: this rank's token shard of the group's activations.
    ``weights[name]``: the whole weight (every rank holds it; each sweeps only
    its ``shard_range`` rows of the group's row-stacked linears).  With
    ``gather`` every rank returns whole results keyed by linear name;
    otherwise results are keyed by input group and hold this rank's rows of
    the group's row-stacked matrix.

    With ``concurrent`` the groups run as chains, largest first (the
    layer-set schedule of ``layerset.quantize_layer_gptq``): a group's
    partial H is formed on the current stream and its all-reduce issued
    asynchronously; the group's factor and row-shard sweep then run on a side
    stream that waits for that all-reduce, while the current stream goes on
    to the next group's partial H.  The factor's first damping attempt reads
    no status on the host; a group that needed more damping is redone at the
    end.  With ``shard_factor`` the factors of Hessians at least
    ``FACTOR_SHARD_MIN_D`` wide split their products across the ranks
    (``factor_hessian_sharded_attempt0``); every rank still ends with the
    same factor.  The results equal the sequential order bit for bit."""
    rank, world = rank_world(group)
    out: dict[str, SweepResult] = {}
    if shard_factor and world > 1:
        _factor_group(group)  # created before any collective is in flight
    if concurrent:
        from . import layerset as LS
        from .gptq_ref import factor_hessian_attempt0
        works: dict = {}

        def form(grp, chunk):
            x = inputs_local[grp]
            d = x.shape[1]
            h = torch.empty((d, d), dtype=torch.float32, device=x.device)
            stats.syrk_into(h, x, accumulate=False, token_chunk=chunk)
            works[grp] = allreduce_sym_(h, group, async_op=True)
            return h

        def prepare(grp, h):
            if works.get(grp) is not None:
                # the side stream (current here) waits for the all-reduce and unpacks
                works[grp].wait()
            if shard_factor:
                return factor_hessian_sharded_attempt0(h, cfg, group)
            return factor_hessian_attempt0(h, cfg)

        def rows(grp):
            w = _stacked(weights, _members(shapes, grp))
            r0, r1 = shard_range(w.shape[0], rank, world, SWEEP_ROW_ALIGN)
            return w[r0:r1]

        def work(grp, state):
            f, status = state
            return status, gptq_sweep(rows(grp), f.u, f.perm, cfg)

        def redo(grp, h):
            f = factor_hessian(h, cfg)
            return gptq_sweep(rows(grp), f.u, f.perm, cfg)

        sizes = LS._chain_sizes(inputs_local, shapes)
        local = LS._run_groups_concurrently(sizes, form, work, redo, prepare)
        items = [(grp, local[grp]) for grp in inputs_local]
    else:
        hs = hessians_token_sharded(inputs_local, group)
        items = []
        for grp, h in hs.items():
            f = factor_hessian(h, cfg)
            w = _stacked(weights, _members(shapes, grp))
            r0, r1 = shard_range(w.shape[0], rank, world, SWEEP_ROW_ALIGN)
            items.append((grp, gptq_sweep(w[r0:r1], f.u, f.perm, cfg)))
    for grp, res in items:
        members = _members(shapes, grp)
        if not gather:
            out[grp] = res
            continue
        m = sum(mi for _, mi in members)
        deq = gather_rows(res.dequant, m, group)
        codes = gather_rows(res.codes, m, group)
        scales = gather_rows(res.scales, m, group)
        zeros = gather_rows(res.zeros, m, group)
        i0 = 0
        for name, mi in members:
            out[name] = SweepResult(deq[i0:i0 + mi], codes[i0:i0 + mi], scales[i0:i0 + mi],
                                    zeros[i0:i0 + mi], res.g_idx, res.perm)
            i0 += mi
    return out


def layer_sets_for_rank(n_layers: int, shapes, tokens: int, group=None) -> list[int]:
    """Layer-parallel schedule: the layer indices this rank quantizes (LPT on
    :func:`layer_set_cost`; equal-cost layers are dealt round-robin)."""
    rank, world = rank_world(group)
    cost = layer_set_cost(shapes, tokens)
    return sorted(lpt_assign({i: cost for i in range(n_layers)}, world)[rank])


def tokens_for_rank(n_tokens: int, group=None) -> tuple[int, int]:
    """This rank's token shard ``[start, stop)`` for token-sharded statistics."""
    rank, world = rank_world(group)
    return shard_range(n_tokens, rank, world)


class CommHandle:
    """libgq's per-device handle with a library-owned NCCL communicator (the
    C ABI ``gq_handle_create_nccl`` / ``gq_allreduce_sum_f32``), for callers
    that sum Hessians without torch.distributed.  Rank 0 makes the id with
    :meth:`unique_id` and shares it with the other ranks out of band; every
    rank then constructs its handle (a collective call), one per GPU."""

    def __init__(self, device: int, unique_id: bytes, nranks: int, rank: int):
        from . import _lib
        import ctypes
        self._lib = _lib
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(unique_id), len(unique_id))
        _lib.call("gq_handle_create_nccl", device, buf, nranks, rank, ctypes.byref(h))
        self._h = h
        self.device, self.nranks, self.rank = device, nranks, rank

    @staticmethod
    def unique_id() -> bytes:
        from . import _lib
        import ctypes
        buf = ctypes.create_string_buffer(128)
        _lib.call("gq_nccl_unique_id", buf, 128)
        return buf.raw

    def allreduce_sum_(self, t: torch.Tensor) -> None:
        """In-place sum of a contiguous float32 tensor on this handle's GPU,
        ordered on the current stream."""
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("allreduce_sum_ needs a contiguous float32 CUDA tensor")
        self._lib.call("gq_allreduce_sum_f32", self._h, A.ptr(t), t.numel(), A.stream())

    def allreduce_sym_(self, h: torch.Tensor) -> None:
        """In-place sum of a symmetric float32 matrix through its packed upper
        triangle (``gq_allreduce_sym_f32``: half the bytes), ordered on the
        current stream; the result is exactly symmetric."""
        if h.dtype != torch.float32 or not h.is_cuda or h.dim() != 2 or \
                h.shape[0] != h.shape[1] or h.stride(1) != 1:
            raise ValueError("allreduce_sym_ needs a square float32 CUDA matrix")
        d = h.shape[0]
        packed = torch.empty((self._lib.lib().gq_sym_packed_size(d),), dtype=torch.float32,
                             device=h.device)
        self._lib.call("gq_allreduce_sym_f32", self._h, A.ptr(h), d, h.stride(0),
                       A.ptr(packed), A.stream())

    def check(self, abort: bool = True) -> None:
        """Raise ``GQError`` (GQ_ENCCL) if NCCL reports an asynchronous error
        (a failed or lost peer); the communicator is aborted first when
        ``abort``, so no later collective waits on the lost rank."""
        self._lib.call("gq_comm_check", self._h, int(abort))

    def abort(self) -> None:
        """Abort the communicator: a collective stuck on a rank that never
        joins ends with an error.  Callable from a watchdog thread."""
        self._lib.call("gq_handle_abort", self._h)

    def close(self) -> None:
        if self._h is not None and self._h.value:
            self._lib.call("gq_handle_destroy", self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = [
    "SWEEP_ROW_ALIGN", "RankFailure", "Heartbeat", "FACTOR_SHARD_MIN_D",
    "factor_hessian_sharded_attempt0", "factor_hessian_split_emulated", "rank_world", "shard_range", "lpt_assign", "layer_set_cost",
    "allreduce_sum_", "allreduce_sym_", "gather_rows", "hessians_token_sharded", "quantize_layer_gptq_sharded",
    "layer_sets_for_rank", "tokens_for_rank", "CommHandle",
]
