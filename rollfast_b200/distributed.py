"""Multi-GPU Muon: FLOP-balanced leaf ownership + all-gather of the
orthogonalised leaves.

One process per GPU.  Every rank holds the (data-parallel, already reduced)
gradients of all leaves.  The Muon leaves are assigned to ranks by
longest-processing-time-first on their Newton-Schulz FLOPs
(4 m^2 n + 2 m^3 per matrix per iteration, m <= n); each rank runs the
momentum + Newton-Schulz pipeline for its own leaves only, writing O in the
leaf layout into its slot of a per-bucket gathered buffer, and the slots are
exchanged bucket by bucket while the next bucket's Newton-Schulz runs:

* ``transport="ce"`` (default when every rank is on one host): the copy
  engines push each owner's slot into the peers' IPC-mapped buffers, ordered
  by device-side epoch flags (``peer.py``); the gather uses no SMs;
* ``transport="nccl"``: ``all_gather_into_tensor`` on a side stream.

Every rank then applies the tail -lr (shape * O + decay * p) to all leaves.

Momentum for a leaf is kept current only on the rank that owns it; the
ownership plan is deterministic for a given leaf list and world size.

The reference has no collective on this path (its Muon runs every leaf on
every device); ownership + all-gather is the B200 scaling design.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch

from . import _lib, _runtime

_ctx = None


@dataclass
class ShardContext:
    rank: int
    world_size: int
    group: object = None
    buckets: int = 4
    reserve_sms: int = 0
    plans: dict = field(default_factory=dict)
    comm_stream: object = None
    transport: str = "nccl"           # "ce" | "nccl" | "auto" (ce, else nccl)
    owned_state: list = field(default_factory=list)  # [(momentum tensor, owner rank)] of the last update
    errors: "ErrorWatch" = None
    steps: int = 0                    # sharded updates run with this context
    owner_tail: bool = True           # copy-engine transport: update arena (AdamW split, pushed float32)
    fp32_buckets: int = 0             # leading Muon buckets whose owners push float32 updates (rest: O)
    last_parts: tuple = ((), ())      # see owned_parts()
    updates: str = "all"              # "all": every rank returns the whole tree; "owned": owners only

    def close(self) -> None:
        """Releases the plans' peer mappings (collective when any exist)."""
        for entry in self.plans.values():
            peer = entry.updates if isinstance(entry, ArenaPlan) else entry[2]
            if peer is not None:
                peer.close()
        self.plans.clear()


class ErrorWatch:
    """Bounded device-side waits of the sharded update (cross-rank flag waits,
    the tensor-core kernels' pipeline waits) that give up set an error word
    instead of hanging; the results of that step are then invalid.

    After every sharded step the two words are copied, stream-ordered, into a
    small pinned host buffer (``rf_error_snapshot``).  The next step reads the
    snapshots whose copies have landed and, at the latest, the one taken two
    steps earlier (waiting for it if need be, which by then costs nothing),
    so a timeout in step s raises ``RollfastError`` (``RF_ETIMEOUT``) at the
    start of step s+1 or s+2: the updates returned by step s and any later
    step already returned are invalid.  ``check(block=True)`` (used by
    ``consolidate_momentum`` and ``clear``) waits for every snapshot."""

    DEPTH = 2

    def __init__(self):
        self.ring = [torch.zeros(2, dtype=torch.int32, pin_memory=True) for _ in range(self.DEPTH + 1)]
        self.pending = []  # [(slot, event, step, stream)]
        self.next_slot = 0

    def snapshot(self, stream: torch.cuda.Stream, step: int) -> None:
        slot = self.next_slot
        self.next_slot = (slot + 1) % len(self.ring)
        _lib.error_snapshot(self.ring[slot].data_ptr(), stream.cuda_stream)
        ev = torch.cuda.Event()
        ev.record(stream)
        self.pending.append((slot, ev, step, stream))

    def check(self, block: bool = False) -> None:
        while self.pending:
            slot, ev, step, stream = self.pending[0]
            if not (block or len(self.pending) >= self.DEPTH or ev.query()):
                break
            ev.synchronize()
            self.pending.pop(0)
            words = self.ring[slot].tolist()
            if words[0] or words[1]:
                self.pending.clear()
                try:
                    _lib.sync_check(stream.cuda_stream)  # reports and clears the words
                except _lib.RollfastError as exc:
                    raise _lib.RollfastError(
                        exc.status, f"sharded Muon step {step}: {exc}; the updates of step {step} and of every "
                        "later step already returned are invalid") from None
                raise _lib.RollfastError(_lib.RF_ETIMEOUT, f"sharded Muon step {step}: a bounded device-side "
                                         f"wait gave up (words {words})")


TRANSPORTS = ("auto", "ce", "nccl")


def configure(group=None, *, buckets: int | None = None, reserve_sms: int | None = None,
              transport: str | None = None, owner_tail: bool | None = None, updates: str = "all",
              fp32_buckets: int | None = None) -> ShardContext:
    """Enable sharded Muon updates over ``group`` (default: the world group).

    ``transport``: how owners' leaves reach the other ranks: ``"ce"`` (copy
    engine pushes into IPC-mapped peer buffers; one host only), ``"nccl"``
    (all-gather), or ``"auto"`` (default; ``ROLLFAST_DIST_GATHER`` overrides):
    ``ce`` when every rank can map its peers' memory, else ``nccl``.

    ``owner_tail`` (copy-engine transport; default on, ``ROLLFAST_DIST_OWNER_TAIL=0``
    turns it off): every rank holds the update tree in one float32 arena that
    its peers write into (``peer.PeerUpdates``); the returned update tensors
    are views of it, valid until the next update is queued on the caller's
    stream.  The AdamW leaves are split by element range: each rank runs
    AdamW on its range and the copy engines push the float32 updates.  Muon
    buckets are exchanged as 16-bit O (owners' NS writes O, the copy engines
    push it, every rank runs the tail into its arena), except the first
    ``fp32_buckets`` (``ROLLFAST_DIST_FP32_BUCKETS``, default 0), whose owners
    write the final float32 updates in the fused epilogue and push those:
    twice the NVLink bytes, no tail.  Off: the gathered-O exchange with
    AdamW replicated on every rank, into fresh buffers.

    ``updates="owned"``: no exchange at all; each rank updates and returns
    only the leaves it owns (``ownership``), for models whose replicated
    update tree does not fit one GPU (Llama-3-70B: 274 GB of float32
    updates).  Leaves a rank does not own may be passed as meta tensors
    (shape only) in the gradients, parameters and state, and come back as
    meta tensors in the updates; their momentum is not advanced there.

    ``reserve_sms``: SMs the Newton-Schulz GEMM grid leaves free so the
    all-gather (NCCL) runs beside it without displacing GEMM CTAs; default:
    the NCCL channel cap ``NCCL_MAX_NCHANNELS`` when that is set, else 0.
    """
    if reserve_sms is None:
        reserve_sms = int(os.environ.get("NCCL_MAX_NCHANNELS", "0") or 0)
    if buckets is None:
        buckets = int(os.environ.get("ROLLFAST_DIST_BUCKETS", "4") or 4)
    if transport is None:
        transport = os.environ.get("ROLLFAST_DIST_GATHER", "auto") or "auto"
    if owner_tail is None:
        owner_tail = os.environ.get("ROLLFAST_DIST_OWNER_TAIL", "1") != "0"
    if fp32_buckets is None:
        fp32_buckets = int(os.environ.get("ROLLFAST_DIST_FP32_BUCKETS", "0") or 0)
    transport = transport.lower()
    if transport not in TRANSPORTS:
        raise ValueError(f"transport must be one of {TRANSPORTS}, got {transport!r}")
    if updates not in ("all", "owned"):
        raise ValueError(f"updates must be 'all' or 'owned', got {updates!r}")
    import torch.distributed as dist

    global _ctx
    if not dist.is_initialized():
        raise RuntimeError("torch.distributed must be initialised before rollfast_b200.distributed.configure")
    if _ctx is not None:
        _ctx.close()
    _ctx = ShardContext(rank=dist.get_rank(group), world_size=dist.get_world_size(group), group=group,
                        buckets=max(1, int(buckets)), reserve_sms=max(0, int(reserve_sms)), transport=transport,
                        owner_tail=bool(owner_tail), updates=updates, fp32_buckets=max(0, int(fp32_buckets)))
    return _ctx


def current() -> ShardContext | None:
    return _ctx


def use(ctx: ShardContext | None) -> ShardContext | None:
    """Make ``ctx`` (or no sharding, for None) current without releasing the
    previous context's resources; returns the previous context."""
    global _ctx
    prev, _ctx = _ctx, ctx
    return prev


def clear() -> None:
    """Turn sharding off.  Collective when the copy-engine transport has
    mapped peer buffers: every rank of the group must call it.  Raises
    ``RollfastError`` afterwards if a bounded wait of a sharded step gave up."""
    global _ctx
    ctx, _ctx = _ctx, None
    if ctx is not None:
        ctx.close()
        if ctx.errors is not None:
            ctx.errors.check(block=True)


# ---------------------------------------------------------------------------
# Planning (pure host logic; exercised by CPU tests)
# ---------------------------------------------------------------------------


def ns_flops(batch: int, rows: int, cols: int) -> int:
    """Dense NS FLOPs per iteration for a (batch, rows, cols) leaf."""
    m, n = min(rows, cols), max(rows, cols)
    return batch * (4 * m * m * n + 2 * m * m * m)


def lpt_assign(costs: Sequence[int], world_size: int) -> list[int]:
    """Longest-processing-time-first: leaves in decreasing cost order go to
    the currently least-loaded rank (ties: lowest rank, then input order)."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0] * world_size
    owner = [0] * len(costs)
    for i in order:
        r = min(range(world_size), key=lambda k: (load[k], k))
        owner[i] = r
        load[r] += costs[i]
    return owner


SEG_ALIGN = 64  # elements: segments start 128-byte aligned for 16-bit O (vectorised tail loads)


@dataclass
class BucketPlan:
    leaves: list[int]                 # global leaf indices in this bucket
    seg: int                          # per-rank segment length (elements, multiple of SEG_ALIGN)
    offsets: dict                     # leaf -> (owner, offset within owner's segment)
    used: list = field(default_factory=list)  # elements of each rank's segment holding leaves
    index: int = 0                    # position in ShardPlan.buckets


@dataclass
class ShardPlan:
    owner: list[int]
    buckets: list[BucketPlan]
    loads: list[int]


def bucket_weights(n_buckets: int) -> list[float]:
    """Cost shares of the buckets, halving towards the end (the exposed final
    gather and tail are short): 4 -> [8, 4, 2, 1].  Measured on 8 B200s this
    beat a small-large-small pyramid: overlapping more of the gather with the
    GEMMs slows the power-capped GEMMs by about as much as it hides."""
    return [2.0 ** (n_buckets - 1 - k) for k in range(n_buckets)]


def make_plan(sizes: Sequence[int], costs: Sequence[int], world_size: int, n_buckets: int) -> ShardPlan:
    """Ownership + bucket layout: the leaf list (in order) is cut into
    ``n_buckets`` runs whose NS costs follow ``bucket_weights``."""
    owner = lpt_assign(costs, world_size)
    n = len(sizes)
    total = sum(costs) or 1
    weights = bucket_weights(n_buckets)
    wsum = sum(weights)
    bounds, acc, k = [], 0.0, 0
    target = weights[0] / wsum * total
    start = 0
    for i in range(n):
        acc += costs[i]
        if acc >= target and k < n_buckets - 1 and i + 1 < n:
            bounds.append((start, i + 1))
            start = i + 1
            k += 1
            target += weights[k] / wsum * total
    bounds.append((start, n))
    buckets = []
    for lo, hi in bounds:
        if lo >= hi:
            continue
        used = [0] * world_size
        offsets = {}
        for i in range(lo, hi):
            r = owner[i]
            offsets[i] = (r, used[r])
            used[r] += sizes[i]
        seg = (max(used) + SEG_ALIGN - 1) // SEG_ALIGN * SEG_ALIGN if used else 0
        buckets.append(BucketPlan(list(range(lo, hi)), seg, offsets, used, len(buckets)))
    loads = [0] * world_size
    for i, r in enumerate(owner):
        loads[r] += costs[i]
    return ShardPlan(owner, buckets, loads)


def exchange_bucket(send: torch.Tensor, recv: torch.Tensor, group=None) -> None:
    """All-gather one bucket's per-rank segments into recv ([world * seg])."""
    import torch.distributed as dist

    dist.all_gather_into_tensor(recv, send, group=group)


def leaf_view(bucket: BucketPlan, recv: torch.Tensor, leaf: int, numel: int) -> torch.Tensor:
    r, off = bucket.offsets[leaf]
    base = r * bucket.seg + off
    return recv[base:base + numel]


def run_buckets(plan: ShardPlan, rank: int, world_size: int, sizes: Sequence[int], compute_owned: Callable,
                exchange: Callable, buffers: list) -> list:
    """Drive the bucketed owner-computes / all-gather exchange.

    ``buffers[k] = (send, recv)`` for bucket k (``send`` holds ``seg``
    elements, ``recv`` ``world * seg``).  For each bucket,
    ``compute_owned(leaf_ids, offsets, send)`` writes this rank's owned leaves
    (``offsets[i]`` = element offset of leaf i in ``send``), then
    ``exchange(bucket, send, recv)`` gathers every rank's segment into
    ``recv``.  Returns ``[(leaf, view)]`` for every leaf, ``view`` being its
    data in the gathered buffer.  Every rank makes the same sequence of
    ``exchange`` calls.
    """
    out = []
    for b, (send, recv) in zip(plan.buckets, buffers):
        mine = [i for i in b.leaves if plan.owner[i] == rank]
        if mine:
            compute_owned(mine, {i: b.offsets[i][1] for i in mine}, send)
        exchange(b, send, recv)
        for i in b.leaves:
            out.append((i, leaf_view(b, recv, i, sizes[i])))
    return out


def bucket_buffers(plan: ShardPlan, world_size: int, dtype: torch.dtype, device: torch.device) -> list:
    """Persistent (send, recv) pairs, one per bucket, reused every step."""
    return [(torch.empty(max(b.seg, 1), dtype=dtype, device=device)[: b.seg],
             torch.empty(world_size * b.seg, dtype=dtype, device=device)) for b in plan.buckets]


# ---------------------------------------------------------------------------
# GPU path
# ---------------------------------------------------------------------------

_O_DTYPE = {_lib.RF_NS_F16: torch.float16, _lib.RF_NS_BF16: torch.bfloat16, _lib.RF_NS_F32: torch.float32}


def sharded_muon_update(ctx: ShardContext, ml, prm, cbuf, scales, decays, lr: float, decay_f32=None):
    """Sharded version of the fused Muon-branch update (see module doc)."""
    if decay_f32 is None:
        decay_f32 = [False] * len(ml)
    from .base import SIDE_CTAS_PER_SM, rf_dtype, run_tail
    from .muon import _finish_leaves, _leaf_table, run_muon_table
    from .peer import PeerGather

    if not ml:
        return []
    dev = ml[0].g.device
    sizes = [L.out.numel() for L in ml]
    odt = _O_DTYPE[prm.precision]
    key = (tuple((L.layout.flat_shape, L.g.dtype) for L in ml), odt, dev)
    entry = ctx.plans.get(key)
    if entry is None:
        steps = prm.n_coeff_rows or prm.ns_steps
        costs = [ns_flops(*L.layout.flat_shape) * steps for L in ml]
        plan = make_plan(sizes, costs, ctx.world_size, ctx.buckets)
        gather = None
        if ctx.transport in ("ce", "auto") and ctx.world_size > 1:
            gather = PeerGather.create(plan, ctx, odt, dev, required=ctx.transport == "ce")
        # Stream order makes reuse of the NCCL buffers safe: a bucket's send
        # buffer is rewritten only after the compute stream waited for the
        # previous step's gathers, and its recv buffer is regathered only
        # after the tail has read it.  The copy-engine buffers are guarded by
        # the epoch flags (peer.py).
        buffers = gather.buffers if gather is not None else bucket_buffers(plan, ctx.world_size, odt, dev)
        entry = (plan, buffers, gather)
        ctx.plans[key] = entry
    plan, buffers, gather = entry
    if ctx.errors is None:
        ctx.errors = ErrorWatch()
    ctx.errors.check()  # a wait of step s-1 or s-2 that gave up raises here
    ctx.steps += 1
    ctx.owned_state = [(L.mu_state, plan.owner[i]) for i, L in enumerate(ml)]
    compute = torch.cuda.current_stream(dev)
    # Streams per rank: compute, tail, and either one copy stream (peer.py)
    # or the NCCL side stream, well inside the device's hardware queues.
    if gather is None and ctx.comm_stream is None:
        ctx.comm_stream = torch.cuda.Stream(device=dev)
    comm = ctx.comm_stream
    tail_stream = _runtime.aux_stream(dev)
    prm.fuse_tail = 0

    side = gather.copy_stream if gather is not None else comm
    trace = _Trace(compute, side) if os.environ.get("ROLLFAST_DIST_PROFILE") == "1" else None

    def compute_owned(ids, offsets, send):
        # Momentum + NS for this rank's leaves of the bucket, O written (leaf
        # layout, 16-bit) straight into their segment of the send buffer.
        if trace is not None:
            trace.mark("compute", "ns")
        sub = [ml[i] for i in ids]
        arr = _leaf_table(sub, [1.0] * len(sub), [0.0] * len(sub))
        for j, i in enumerate(ids):
            arr[j].out = send.data_ptr() + offsets[i] * send.element_size()
            arr[j].out_dtype = rf_dtype(send)
        run_muon_table(arr, len(sub), prm, dev)

    def tail(bucket, recv):
        # -lr (shape O + decay p) for all the bucket's leaves, on the tail
        # stream beside the next bucket's GEMMs.
        with torch.cuda.stream(tail_stream):
            if trace is not None:
                trace.mark("tail", "tail")
            items = []
            for i in bucket.leaves:
                L = ml[i]
                o = leaf_view(bucket, recv, i, sizes[i])
                p = L.p.reshape(-1) if (L.p is not None and decays[i] != 0.0) else None
                items.append((o, p, L.out.view(-1), scales[i], decays[i], decay_f32[i]))
            run_tail(items, lr, SIDE_CTAS_PER_SM)
            if trace is not None:
                trace.mark("tail", "tail_end")

    def exchange_nccl(bucket, send, recv):
        # Gather on the side stream once this bucket's NS is done, while the
        # compute stream moves on to the next bucket.
        ready = torch.cuda.Event()
        ready.record(compute)
        if trace is not None:
            trace.mark("compute", "ns_end")
        comm.wait_event(ready)
        with torch.cuda.stream(comm):
            if trace is not None:
                trace.mark("comm", "gather")
            exchange_bucket(send, recv, ctx.group)
            if trace is not None:
                trace.mark("comm", "gather_end")
        # The tail gets its own stream so the next bucket's gather does not
        # queue behind it.
        gathered = torch.cuda.Event()
        gathered.record(comm)
        tail_stream.wait_event(gathered)
        tail(bucket, recv)

    def exchange_ce(bucket, send, recv):
        # Copy engines push this rank's slot to every peer while the compute
        # stream moves on to the next bucket's GEMMs (no SMs taken).
        ready = torch.cuda.Event()
        ready.record(compute)
        if trace is not None:
            trace.mark("compute", "ns_end")
        gather.push(bucket.index, ready)
        if trace is not None:
            trace.mark("comm", "push_end")

    if gather is not None:
        gather.begin_step()
        run_buckets(plan, ctx.rank, ctx.world_size, sizes, compute_owned, exchange_ce, buffers)
        # Tails after the last GEMM, at full occupancy on the compute stream:
        # run beside the power-capped GEMMs, their HBM traffic slowed the
        # GEMMs by more than it hid (8 B200s: GEMMs 49 -> 77 ms).  By now the
        # earlier buckets have long arrived; only the last one's push can be
        # exposed.
        for b, (_, recv) in zip(plan.buckets, buffers):
            gather.wait_bucket(b.index, compute)
            with torch.cuda.stream(compute):
                if trace is not None:
                    trace.mark("compute", "tail")
                items = []
                for i in b.leaves:
                    L = ml[i]
                    p = L.p.reshape(-1) if (L.p is not None and decays[i] != 0.0) else None
                    items.append((leaf_view(b, recv, i, sizes[i]), p, L.out.view(-1), scales[i], decays[i],
                                  decay_f32[i]))
                run_tail(items, lr)
        if trace is not None:
            trace.mark("compute", "tail_end")
        gather.end_step(compute, compute)
    else:
        run_buckets(plan, ctx.rank, ctx.world_size, sizes, compute_owned, exchange_nccl, buffers)
        for side in (comm, tail_stream):
            done = torch.cuda.Event()
            done.record(side)
            compute.wait_event(done)
    ctx.errors.snapshot(compute, ctx.steps)
    if trace is not None:
        trace.report(ctx.rank, [sum(sizes[i] for i in b.leaves) for b in plan.buckets])
    return _finish_leaves(ml)


@dataclass
class ArenaPlan:
    """Ownership, arena layout and the mapped arena of one sharded tree
    (owner-side tail)."""

    plan: ShardPlan                   # Muon leaf owners and buckets
    updates: object                   # peer.PeerUpdates
    muon_offsets: list                # arena offset of each Muon leaf
    adam_offsets: list                # arena offset of each AdamW leaf
    adam_spans: list                  # [(start, end)] of the AdamW region per owner rank
    adam_region: int                  # region index of the AdamW leaves
    o_regions: set = field(default_factory=set)  # Muon buckets exchanged as 16-bit O


def _arena_plan(ctx: ShardContext, ml, a_items, prm, dev):
    from .peer import PeerUpdates, arena_layout, split_range

    sizes = [L.out.numel() for L in ml]
    steps = prm.n_coeff_rows or prm.ns_steps
    costs = [ns_flops(*L.layout.flat_shape) * steps for L in ml]
    plan = make_plan(sizes, costs, ctx.world_size, ctx.buckets) if ml else ShardPlan([], [], [0] * ctx.world_size)
    regions = [[(i, plan.owner[i], sizes[i]) for i in b.leaves] for b in plan.buckets]
    offs, ranges, total = arena_layout(regions, ctx.world_size)
    muon_offsets = [offs[i] for i in range(len(ml))]
    o_regions = {b.index for b in plan.buckets if b.index >= ctx.fp32_buckets}
    o_span = None
    if o_regions:
        o_span = (min(ranges[k][0][0] for k in o_regions), max(ranges[k][-1][1] for k in o_regions))
    # AdamW leaves: laid out one after another and split by element count.
    adam_offsets, acc = [], total
    for it in a_items:
        adam_offsets.append(acc)
        acc += (it[0].numel() + 63) // 64 * 64
    adam_region = len(ranges)
    adam_spans = split_range(total, acc - total, ctx.world_size)
    if a_items:
        ranges.append(adam_spans)
    updates = PeerUpdates.create(ranges, max(acc, 1), ctx, dev, required=ctx.transport == "ce", o_span=o_span,
                                 o_dtype=_O_DTYPE[prm.precision])
    if updates is None:
        return None
    return ArenaPlan(plan, updates, muon_offsets, adam_offsets, adam_spans, adam_region, o_regions)


def sharded_update(ctx: ShardContext, ml, prm, cbuf, scales, decays, lr: float, decay_f32, a_items, adam_kw,
                   a_seeds=None, a_pos=()):
    """Sharded Muon branch + AdamW leaves over the update arena (copy-engine
    transport).  Returns ``(muon_outs, adam_outs)`` in the order of ``ml`` and
    ``a_items``, or None when the peers cannot be mapped (the caller then
    takes the gathered-O path).

    Per step: every rank signals that its stream reached the step; it runs
    AdamW on its element range of the AdamW leaves (final float32 updates in
    its arena) and momentum + Newton-Schulz on the Muon leaves it owns,
    bucket by bucket, writing 16-bit O (or, for the first ``fp32_buckets``,
    final float32 updates through the fused tail); after each piece the copy
    engines push the owner's span to every peer.  Every rank then runs the
    tail of the O buckets into its arena, each behind its bucket's arrival,
    and the step ends when every owner's pushes have landed.  The NVLink
    bytes per Muon element are 2 for O buckets, 4 for float32 ones: on 8
    B200s the float32 form slowed the power-capped GEMMs more than the tail it
    saves (96.5 vs 88.2 ms per Llama-3-8B step), hence O by default."""
    from .adam import run_adam
    from .base import rf_dtype, run_tail
    from .muon import _finish_leaves, _leaf_table, run_muon_table

    dev = (ml[0].g if ml else a_items[0][0]).device
    key = ("arena", ctx.fp32_buckets, tuple((L.layout.flat_shape, L.g.dtype) for L in ml),
           tuple((tuple(it[0].shape), it[0].dtype) for it in a_items), prm.n_coeff_rows or prm.ns_steps, dev)
    entry = ctx.plans.get(key)
    if entry is None:
        entry = _arena_plan(ctx, ml, a_items, prm, dev)
        if entry is None:
            return None
        ctx.plans[key] = entry
    if ctx.errors is None:
        ctx.errors = ErrorWatch()
    ctx.errors.check()  # a wait of step s-1 or s-2 that gave up raises here
    ctx.steps += 1
    plan, up = entry.plan, entry.updates
    arena = up.arena
    compute = torch.cuda.current_stream(dev)
    ml = [L._replace(out=arena[o: o + L.out.numel()].view(L.out.shape)) for L, o in zip(ml, entry.muon_offsets)]
    a_outs = [arena[o: o + it[0].numel()].view(it[0].shape) for it, o in zip(a_items, entry.adam_offsets)]
    owned = [(L.mu_state, plan.owner[i]) for i, L in enumerate(ml)]
    trace = _Trace(compute, up.copy_stream) if os.environ.get("ROLLFAST_DIST_PROFILE") == "1" else None

    def mark(stream, label):
        if trace is not None:
            trace.mark(stream, label)

    up.begin_step(compute)
    # AdamW first: its push overlaps the first bucket's Newton-Schulz.
    if a_items:
        mark("compute", "adam")
        mine, seeds = [], []
        for j, (it, o, out) in enumerate(zip(a_items, entry.adam_offsets, a_outs)):
            g, mu, nu, p = it[0], it[1], it[2], it[3]
            n = g.numel()
            for r, (slo, shi) in enumerate(entry.adam_spans):
                a, b = max(slo - o, 0), min(shi - o, n)
                if a >= b:
                    continue
                owned += [(mu.view(-1)[a:b], r), (nu.view(-1)[a:b], r)]
                if r == ctx.rank:
                    mine.append((g.view(-1)[a:b], mu.view(-1)[a:b], nu.view(-1)[a:b],
                                 None if p is None else p.reshape(-1)[a:b], out.view(-1)[a:b], *it[5:7]))
                    if a_seeds is not None:  # a slice keeps its leaf's noise streams
                        seeds += [a_seeds[2 * j], a_seeds[2 * j + 1]]
        run_adam(mine, seeds=seeds if a_seeds is not None else None, **adam_kw)
        mark("compute", "adam_end")
        ev = torch.cuda.Event()
        ev.record(compute)
        up.push(entry.adam_region, ev)
        mark("comm", "adam_push_end")
    fuse = prm.fuse_tail
    for b in plan.buckets:
        o_mode = b.index in entry.o_regions
        ids = [i for i in b.leaves if plan.owner[i] == ctx.rank]
        mark("compute", f"ns{b.index}")
        if ids:
            sub = [ml[i] for i in ids]
            if o_mode:  # O (16-bit, leaf layout) into the exchanged buffer; the tail comes after the exchange
                sub = [L._replace(out=up.o_view(o, L.out.numel()))
                       for L, o in zip(sub, (entry.muon_offsets[i] for i in ids))]
            arr = _leaf_table(sub, [scales[i] for i in ids], [decays[i] for i in ids],
                              [decay_f32[i] for i in ids])
            for j in range(len(ids)):
                arr[j].out_dtype = rf_dtype(sub[j].out)
            prm.fuse_tail = 0 if o_mode else fuse
            run_muon_table(arr, len(ids), prm, dev)
            prm.fuse_tail = fuse
        mark("compute", f"ns_end{b.index}")
        ev = torch.cuda.Event()
        ev.record(compute)
        up.push(b.index, ev, o_region=o_mode)
        mark("comm", f"push_end{b.index}")
    # Tails of the O buckets (every rank, the owners' own leaves too, so all
    # replicas hold identical updates), each behind its bucket's arrival.
    for b in plan.buckets:
        if b.index not in entry.o_regions:
            continue
        up.wait_region(b.index, compute)
        mark("compute", f"tail{b.index}")
        items = []
        for i in b.leaves:
            L, o = ml[i], entry.muon_offsets[i]
            p = L.p.reshape(-1) if (L.p is not None and decays[i] != 0.0) else None
            items.append((up.o_view(o, L.out.numel()), p, L.out.view(-1), scales[i], decays[i], decay_f32[i]))
        run_tail(items, lr)
        mark("compute", f"tail_end{b.index}")
    up.finish(compute)
    mark("compute", "finish")
    if trace is not None:
        trace.report(ctx.rank, [sum(ml[i].out.numel() for i in b.leaves) for b in plan.buckets])
    ctx.owned_state = owned
    adam_parts = []
    if a_items:
        lo, hi = entry.adam_spans[ctx.rank]
        for pos, it, o in zip(a_pos, a_items, entry.adam_offsets):
            a, b = max(lo - o, 0), min(hi - o, it[0].numel())
            if a < b:
                adam_parts.append((pos, a, b))
    ctx.last_parts = (tuple(L.pos for i, L in enumerate(ml) if plan.owner[i] == ctx.rank), tuple(adam_parts))
    ctx.errors.snapshot(compute, ctx.steps)
    return _finish_leaves(ml), a_outs


def owner_ranks(muon_shapes, adam_numels, world_size: int) -> tuple[list[int], list[int]]:
    """Owners under ``updates="owned"``: Muon leaves (``(batch, rows, cols)``
    in tree order) by longest-processing-time-first on their Newton-Schulz
    FLOPs, the same assignment every sharded mode uses; AdamW leaves by
    longest-processing-time-first on their element counts."""
    muon = lpt_assign([ns_flops(*s) for s in muon_shapes], world_size) if muon_shapes else []
    adam = lpt_assign(list(adam_numels), world_size) if adam_numels else []
    return muon, adam


def ownership(params, muon_weight_dimension_numbers=None, world_size: int | None = None):
    """A tree like ``params`` holding the rank that owns each leaf under
    ``configure(updates="owned")`` for a ``muon(...)`` built with the same
    ``muon_weight_dimension_numbers`` (None for aux leaves).  Shapes and
    dtypes are all it reads, so meta tensors work: a caller can allocate
    gradients, parameters and state only for the leaves it owns."""
    from .dimension_numbers import _compute_matrix_layout, _make_matrix_partition_fns
    from .muon import _flatten_specs
    from .tree import is_aux_leaf, tree_flatten, tree_unflatten

    if world_size is None:
        world_size = _ctx.world_size if _ctx is not None else 1
    part = _make_matrix_partition_fns(muon_weight_dimension_numbers, "muon")
    leaves, treedef = tree_flatten(params, is_leaf=is_aux_leaf)
    labels = tree_flatten(part.labels(params), is_leaf=lambda x: x is None or isinstance(x, str))[0]
    specs = _flatten_specs(part.masked_specs(params), len(leaves))
    muon_pos, muon_shapes, adam_pos, adam_numels = [], [], [], []
    for i, (x, lab, spec) in enumerate(zip(leaves, labels, specs)):
        if is_aux_leaf(x):
            continue
        if lab == "muon":
            muon_pos.append(i)
            muon_shapes.append(_compute_matrix_layout(x.shape, x.dtype, spec).flat_shape)
        else:
            adam_pos.append(i)
            adam_numels.append(x.numel())
    mo, ao = owner_ranks(muon_shapes, adam_numels, world_size)
    out = [None] * len(leaves)
    for i, r in zip(muon_pos, mo):
        out[i] = r
    for i, r in zip(adam_pos, ao):
        out[i] = r
    return tree_unflatten(treedef, out)


def owned_update(ctx: ShardContext, ml, prm, cbuf, scales, decays, decay_f32, a_items, adam_kw, a_seeds=None,
                 a_pos=()):
    """``updates="owned"``: momentum + Newton-Schulz + fused tail for the Muon
    leaves this rank owns and AdamW for the AdamW leaves it owns, into fresh
    float32 buffers; every other leaf's update is a meta tensor.  No data
    crosses ranks."""
    from .adam import run_adam
    from .base import require_cuda
    from .muon import _finish_leaves, _leaf_table, run_muon_table

    mo, ao = owner_ranks([L.layout.flat_shape for L in ml], [it[0].numel() for it in a_items], ctx.world_size)
    mine = [i for i, r in enumerate(mo) if r == ctx.rank]
    for i in mine:
        require_cuda(ml[i].g, "gradient of an owned leaf")
    ml = [L._replace(out=torch.empty(L.out.shape, dtype=torch.float32, device=L.g.device)) if r == ctx.rank else L
          for L, r in zip(ml, mo)]
    if mine:
        sub = [ml[i] for i in mine]
        arr = _leaf_table(sub, [scales[i] for i in mine], [decays[i] for i in mine], [decay_f32[i] for i in mine])
        run_muon_table(arr, len(sub), prm, sub[0].g.device)
    outs = []
    for L, r in zip(ml, mo):
        if r == ctx.rank:
            outs.append(_finish_leaves([L])[0])
        else:
            outs.append(torch.empty(L.shape, dtype=torch.float32, device="meta"))
    a_outs, items, seeds = [], [], []
    for j, (it, r) in enumerate(zip(a_items, ao)):
        if r == ctx.rank:
            require_cuda(it[0], "gradient of an owned leaf")
            o = torch.empty(it[0].shape, dtype=torch.float32, device=it[0].device)
            items.append((*it[:4], o, *it[5:]))
            if a_seeds is not None:
                seeds += [a_seeds[2 * j], a_seeds[2 * j + 1]]
        else:
            o = torch.empty(it[0].shape, dtype=torch.float32, device="meta")
        a_outs.append(o)
    run_adam(items, seeds=seeds if a_seeds is not None else None, **adam_kw)
    ctx.owned_state = []
    ctx.last_parts = (tuple(L.pos for L, r in zip(ml, mo) if r == ctx.rank),
                      tuple((pos, 0, it[0].numel()) for pos, it, r in zip(a_pos, a_items, ao) if r == ctx.rank))
    return outs, a_outs


def owned_parts(ctx: ShardContext | None = None) -> tuple:
    """What this rank computed in the context's last sharded update:
    ``(muon_positions, adam_ranges)`` -- the tree positions (flattened leaf
    order) of the Muon leaves it owns, and ``(position, start, end)`` element
    ranges of the AdamW leaves it owns.  Those are the gradient elements the
    rank reads and the update elements it produces, so a host pipeline that
    holds one gradient tree can feed each rank only its part (the update
    arena then holds every rank's results)."""
    ctx = ctx or _ctx
    return ctx.last_parts if ctx is not None else ((), ())


def consolidate_momentum(ctx: ShardContext | None = None) -> int:
    """Make the Muon momentum current on every rank (collective over the
    group), e.g. before saving a checkpoint from one rank.

    A sharded update advances a leaf's momentum only on the rank that owns it;
    everything else in the optimizer state (counts, keys, AdamW moments) is
    replicated.  This broadcasts each leaf's momentum from its owner, as
    recorded by the last sharded update, so afterwards every rank holds the
    same full state.  Returns the number of leaves broadcast."""
    import torch.distributed as dist

    ctx = ctx or _ctx
    if ctx is None or ctx.world_size == 1:
        return 0
    if ctx.errors is not None:
        ctx.errors.check(block=True)  # momentum of a step whose waits gave up is not current anywhere
    for t, owner in ctx.owned_state:
        src = dist.get_global_rank(ctx.group, owner) if ctx.group is not None else owner
        dist.broadcast(t, src=src, group=ctx.group)
    return len(ctx.owned_state)


def active_transport(ctx: ShardContext | None = None) -> str:
    """The transport the context's plans use: "ce+owner_tail", "ce",
    "nccl", or the configured value when no plan has been built yet."""
    ctx = ctx or _ctx
    if ctx is None:
        return "none"
    kinds = {("ce+owner_tail" if isinstance(e, ArenaPlan) else ("ce" if e[2] is not None else "nccl"))
             for e in ctx.plans.values()}
    return kinds.pop() if len(kinds) == 1 else ctx.transport


class _Trace:
    """Opt-in (ROLLFAST_DIST_PROFILE=1) timeline of the sharded update: CUDA
    events on the compute and comm streams, printed by every rank after a
    synchronisation (diagnostics only; it serialises the host)."""

    def __init__(self, compute, comm):
        self.streams = {"compute": compute, "comm": comm or compute, "tail": _runtime.aux_stream(compute.device)}
        self.marks = []
        self.t0 = torch.cuda.Event(enable_timing=True)
        self.t0.record(compute)

    def mark(self, stream: str, label: str) -> None:
        e = torch.cuda.Event(enable_timing=True)
        e.record(self.streams[stream])
        self.marks.append((stream, label, e))

    def report(self, rank: int, bucket_elems) -> None:
        torch.cuda.synchronize()
        rows = [f"{st}:{lab}@{self.t0.elapsed_time(e):.2f}" for st, lab, e in self.marks]
        print(f"[rollfast_b200 dist trace rank {rank}] buckets={list(bucket_elems)} " + " ".join(rows), flush=True)
