"""Copy-engine all-gather of the sharded Muon update (host side of
``csrc/rf_peer.cu``).

Every rank keeps one flat *gathered buffer* holding, per bucket, a region of
``world`` slots; slot ``r`` receives rank r's orthogonalised leaves.  An owner's
Newton-Schulz pipeline writes its O straight into its own slot; the copy
engines then push that slot into the same slot of every peer's buffer, which
is mapped into this process through CUDA IPC.  The push takes no SMs, so it
runs beside the next bucket's tcgen05 GEMMs without displacing them (on 8
B200s: ~700 GB/s per rank, the GEMMs ~3% slower, where an NCCL all-gather of
the same bytes slowed them 15-35%).

Cross-rank ordering, with a 32-bit epoch ``e`` per step (all ranks count
steps identically) and a small flag array per rank
(``arrive[bucket][sender]`` then ``ack[sender]``):

* before its first push of step e, an owner waits until every peer's
  ``ack >= e - 1`` (the peer finished reading step e-1's data);
* after pushing bucket k to every peer, the owner stores
  ``arrive[k][owner] = e`` into each peer's flags;
* a receiver's tail of bucket k waits until ``arrive[k][*] >= e``; the tails
  run after the rank's last Newton-Schulz GEMM, on the compute stream
  (distributed.py);
* after its last tail, a rank stores ``ack[rank] = e`` into every peer.

Waits are bounded device-side polls (``rf_flags_wait``); one that gives up
sets a device error word instead of hanging, which the sharded update reads
back asynchronously after every step (``distributed.ErrorWatch``) and reports
as ``RF_ETIMEOUT`` one or two steps later.

All pushes go through ONE copy stream, peer after peer in a rotation that
starts at rank+1 (so every GPU receives from one peer at a time): one stream
pushes as fast as seven (~720 GB/s), and more streams would exceed the
device's hardware work queues (8 by default) together with the compute and
tail streams, aliasing streams onto shared queues where one stream's wait
stalls another's work.
"""

from __future__ import annotations

import os
import socket
from dataclasses import dataclass

import torch

from . import _lib

_ALIGN = 64  # elements: every region starts 128-byte aligned (16-bit O)


def ce_layout(bucket_segs, world_size: int) -> tuple[list[int], int]:
    """Element offset of each bucket's ``world * seg`` region in the flat
    gathered buffer, and the buffer's total length."""
    offs, acc = [], 0
    for seg in bucket_segs:
        offs.append(acc)
        acc += (world_size * seg + _ALIGN - 1) // _ALIGN * _ALIGN
    return offs, acc


def flag_index(bucket: int, sender: int, world_size: int) -> int:
    """Index of ``arrive[bucket][sender]`` in a rank's flag array."""
    return bucket * world_size + sender


def ack_index(sender: int, n_buckets: int, world_size: int) -> int:
    """Index of ``ack[sender]`` in a rank's flag array."""
    return n_buckets * world_size + sender


def default_timeout_s() -> float:
    return float(os.environ.get("ROLLFAST_PEER_TIMEOUT_S", "30"))


@dataclass
class _Remote:
    buf: int = 0      # address of the peer's gathered buffer in this process
    flags: int = 0    # address of the peer's flag array in this process


class PeerGather:
    """IPC-mapped gathered buffers and flags for one ownership plan."""

    def __init__(self, plan, rank: int, world_size: int, group, dtype: torch.dtype, device: torch.device,
                 timeout_s: float | None = None):
        self.plan, self.rank, self.world, self.group = plan, rank, world_size, group
        self.device = device
        self.timeout_s = default_timeout_s() if timeout_s is None else float(timeout_s)
        segs = [b.seg for b in plan.buckets]
        self.regions, total = ce_layout(segs, world_size)
        self.buf = torch.empty(max(total, 1), dtype=dtype, device=device)
        nb = len(plan.buckets)
        self.flags = torch.zeros(nb * world_size + world_size, dtype=torch.int32, device=device)
        self.esize = self.buf.element_size()
        self.epoch = 0
        self.remote = [None] * world_size
        self._mapped: list[int] = []
        self.copy_stream = torch.cuda.Stream(device=device) if world_size > 1 else None
        # (slot view, region view) per bucket, in the shape run_buckets expects.
        self.buffers = []
        for b, off in zip(plan.buckets, self.regions):
            region = self.buf[off: off + world_size * b.seg]
            self.buffers.append((region[rank * b.seg: (rank + 1) * b.seg], region))

    # -- set-up / tear-down (collective over the group) ----------------------
    @classmethod
    def create(cls, plan, ctx, dtype, device, *, required: bool):
        """Maps every peer's buffers; returns None (on every rank) when some
        rank cannot take part and ``required`` is False."""
        import torch.distributed as dist

        g = cls(plan, ctx.rank, ctx.world_size, ctx.group, dtype, device)
        torch.cuda.synchronize(device)  # flags are zero before any peer can signal
        try:
            hb, ob = _lib.ipc_export(g.buf.data_ptr())
            hf, of = _lib.ipc_export(g.flags.data_ptr())
            mine = (True, socket.gethostname(), hb, ob, hf, of)
        except Exception as exc:  # noqa: BLE001 - reported to every rank below
            mine = (False, repr(exc))
        infos = [None] * ctx.world_size
        dist.all_gather_object(infos, mine, group=ctx.group)
        why = next((f"rank {r}: {i[1]}" for r, i in enumerate(infos) if not i[0]), None)
        if why is None and len({i[1] for i in infos}) != 1:
            why = "ranks are on more than one host"
        opened = why is None
        if opened:
            try:
                for r, info in enumerate(infos):
                    if r == ctx.rank:
                        continue
                    _, _, hb, ob, hf, of = info
                    bb = _lib.ipc_open(hb)
                    g._mapped.append(bb)
                    fb = _lib.ipc_open(hf)
                    g._mapped.append(fb)
                    g.remote[r] = _Remote(bb + ob, fb + of)
            except Exception as exc:  # noqa: BLE001
                opened, why = False, f"rank {ctx.rank}: {exc!r}"
        oks = [None] * ctx.world_size
        dist.all_gather_object(oks, (opened, why), group=ctx.group)
        failed = next((w for o, w in oks if not o), None)
        if failed is None:
            return g
        g.close(barrier=False)
        if required:
            raise RuntimeError(f"copy-engine gather unavailable: {failed}")
        return None

    def close(self, barrier: bool = True) -> None:
        """Unmaps the peers' buffers.  With ``barrier`` (collective), first
        waits until every rank's device is idle so no push is in flight."""
        if barrier:
            import torch.distributed as dist

            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        for base in self._mapped:
            _lib.ipc_close(base)
        self._mapped = []
        self.remote = [None] * self.world

    # -- one step -----------------------------------------------------------
    def _peers(self):
        return [(self.rank + 1 + j) % self.world for j in range(self.world - 1)]

    def begin_step(self) -> None:
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        if self.copy_stream is None:
            return
        acks = self.flags.data_ptr() + 4 * ack_index(0, len(self.plan.buckets), self.world)
        _lib.flags_wait(acks, self.world, self.rank, self.epoch - 1, self.timeout_s,
                        self.copy_stream.cuda_stream)

    def push(self, k: int, ready: torch.cuda.Event) -> None:
        """Push this rank's slot of bucket ``k`` (complete at ``ready``) to every peer."""
        b = self.plan.buckets[k]
        off = (self.regions[k] + self.rank * b.seg) * self.esize
        nbytes = b.used[self.rank] * self.esize
        src = self.buf.data_ptr() + off
        fidx = 4 * flag_index(k, self.rank, self.world)
        s = self.copy_stream
        if s is None:
            return
        s.wait_event(ready)
        peers = self._peers()
        if nbytes:
            for r in peers:
                _lib.peer_copy(self.remote[r].buf + off, src, nbytes, s.cuda_stream)
        _lib.flags_signal([self.remote[r].flags + fidx for r in peers], self.epoch, s.cuda_stream)

    def wait_bucket(self, k: int, stream: torch.cuda.Stream) -> None:
        """Block ``stream`` until every peer's slot of bucket ``k`` has landed."""
        if self.world > 1:
            addr = self.flags.data_ptr() + 4 * flag_index(k, 0, self.world)
            _lib.flags_wait(addr, self.world, self.rank, self.epoch, self.timeout_s, stream.cuda_stream)

    def end_step(self, tail_stream: torch.cuda.Stream, compute: torch.cuda.Stream) -> None:
        """Acknowledge the step to every peer once ``tail_stream`` has read the
        gathered buffer, and order ``compute`` after the pushes and the tail."""
        nb = len(self.plan.buckets)
        if self.world > 1:
            aidx = 4 * ack_index(self.rank, nb, self.world)
            _lib.flags_signal([self.remote[r].flags + aidx for r in self._peers()], self.epoch,
                              tail_stream.cuda_stream)
        for s in [self.copy_stream, tail_stream]:
            if s is None or s == compute:
                continue
            ev = torch.cuda.Event()
            ev.record(s)
            compute.wait_event(ev)


# ---------------------------------------------------------------------------
# Owner-side tail: a float32 update arena pushed by its owners.
# ---------------------------------------------------------------------------


def arena_layout(regions, world_size: int, align: int = 64):
    """Element layout of the update arena.

    ``regions``: one list per exchange region (the Muon buckets) of
    ``(key, owner, numel)`` leaves.  Within a region the leaves are grouped
    by owner (in rank order, leaf order kept within an owner), so each
    owner's leaves form one contiguous span; every leaf starts
    ``align``-element aligned (vector epilogue stores).  Returns
    ``(offsets, ranges, total)``: ``offsets[key]`` a leaf's element offset,
    ``ranges[k][r] = (start, end)`` owner r's span of region k, ``total``
    the elements laid out."""
    acc = 0
    offsets, ranges = {}, []
    for leaves in regions:
        span = []
        for owner in range(world_size):
            start = acc
            for key, o, n in leaves:
                if o == owner:
                    offsets[key] = acc
                    acc += (n + align - 1) // align * align
            span.append((start, acc))
        ranges.append(span)
    return offsets, ranges, acc


def split_range(start: int, total: int, world_size: int, align: int = 64):
    """``world_size`` contiguous spans covering ``[start, start + total)``,
    boundaries ``align``-element aligned, as equal as the alignment allows."""
    units = (total + align - 1) // align
    spans, lo = [], start
    for r in range(world_size):
        hi = start + min(total, (units * (r + 1) // world_size) * align)
        spans.append((lo, hi))
        lo = hi
    return spans


def _map_peer_buffers(ctx, tensors, required: bool):
    """Collective: exports ``tensors`` (device buffers) and maps every peer's
    counterparts.  Returns ``(remote, mapped, why)``: ``remote[r]`` the list of
    rank r's buffer addresses in this process (None for this rank),
    ``mapped`` the bases to close, ``why`` None on success on every rank."""
    import torch.distributed as dist

    try:
        exported = [_lib.ipc_export(t.data_ptr()) for t in tensors]
        mine = (True, socket.gethostname(), exported)
    except Exception as exc:  # noqa: BLE001 - reported to every rank below
        mine = (False, repr(exc), None)
    infos = [None] * ctx.world_size
    dist.all_gather_object(infos, mine, group=ctx.group)
    why = next((f"rank {r}: {i[1]}" for r, i in enumerate(infos) if not i[0]), None)
    if why is None and len({i[1] for i in infos}) != 1:
        why = "ranks are on more than one host"
    remote, mapped = [None] * ctx.world_size, []
    if why is None:
        try:
            for r, info in enumerate(infos):
                if r == ctx.rank:
                    continue
                addrs = []
                for handle, off in info[2]:
                    base = _lib.ipc_open(handle)
                    mapped.append(base)
                    addrs.append(base + off)
                remote[r] = addrs
        except Exception as exc:  # noqa: BLE001
            why = f"rank {ctx.rank}: {exc!r}"
    oks = [None] * ctx.world_size
    dist.all_gather_object(oks, why, group=ctx.group)
    failed = next((w for w in oks if w is not None), None)
    if failed is not None:
        for base in mapped:
            _lib.ipc_close(base)
        if required:
            raise RuntimeError(f"copy-engine exchange unavailable: {failed}")
        return None, [], failed
    return remote, mapped, None


class PeerUpdates:
    """The float32 update arena of one ownership plan, mapped by every peer.

    Each rank holds the whole sharded update tree in one flat float32 buffer
    (``arena_layout``); the update tensors the step returns are views of it.
    A region (a Muon bucket, or the AdamW leaves) reaches the peers in one of
    two forms: the owners' final float32 updates, written into the owner's
    arena by the fused epilogue or the AdamW kernel and pushed span by span;
    or the owners' 16-bit O, written into a 16-bit buffer mirroring the
    arena's offsets (``o_buf``) and pushed, after which every rank runs the
    tail ``-lr (shape O + decay p)`` into its arena.

    Ordering, with epoch ``e`` per step and flags ``arrive[region][sender]``
    then ``ready[sender]``:

    * at the start of step e each rank stores ``ready[rank] = e`` into every
      peer, on its compute stream, i.e. after whatever the caller queued
      before the step (applying step e-1's updates, which are overwritten
      now);
    * an owner's first push of step e waits until every peer's ``ready >= e``;
    * after pushing region k an owner stores ``arrive[k][owner] = e`` into
      every rank (itself included);
    * the step ends with the compute stream waiting for ``arrive[*][*] >= e``
      and for this rank's own pushes.

    Updates returned by step e therefore stay valid until the next update is
    queued on the caller's stream."""

    def __init__(self, ranges, total, rank, world_size, group, device, timeout_s=None, o_span=None,
                 o_dtype=torch.float16):
        self.ranges, self.rank, self.world, self.group = ranges, rank, world_size, group
        self.device = device
        self.timeout_s = default_timeout_s() if timeout_s is None else float(timeout_s)
        self.arena = torch.empty(total, dtype=torch.float32, device=device)
        # Optional 16-bit O buffer for the regions exchanged as O: it mirrors
        # the arena's element offsets over [o_base, o_base + len).
        self.o_base = o_span[0] if o_span else 0
        self.o_buf = (torch.empty(max(o_span[1] - o_span[0], 1), dtype=o_dtype, device=device) if o_span
                      else None)
        self.n_regions = len(ranges)
        if self.n_regions * world_size > 64:
            raise ValueError("too many exchange regions for one flag wait (regions x ranks must be <= 64)")
        self.flags = torch.zeros(self.n_regions * world_size + world_size, dtype=torch.int32, device=device)
        self.epoch = 0
        self.remote = [None] * world_size
        self._mapped: list[int] = []
        self.copy_stream = torch.cuda.Stream(device=device)

    @classmethod
    def create(cls, ranges, total, ctx, device, *, required: bool, o_span=None, o_dtype=torch.float16):
        g = cls(ranges, total, ctx.rank, ctx.world_size, ctx.group, device, o_span=o_span, o_dtype=o_dtype)
        torch.cuda.synchronize(device)  # flags are zero before any peer can signal
        bufs = [g.arena, g.flags] + ([g.o_buf] if g.o_buf is not None else [])
        remote, mapped, why = _map_peer_buffers(ctx, bufs, required)
        if why is not None:
            return None
        g.remote, g._mapped = remote, mapped
        return g

    def close(self, barrier: bool = True) -> None:
        if barrier:
            import torch.distributed as dist

            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        for base in self._mapped:
            _lib.ipc_close(base)
        self._mapped = []
        self.remote = [None] * self.world

    def _peers(self):
        return [(self.rank + 1 + j) % self.world for j in range(self.world - 1)]

    def _flag_addr(self, r: int, index: int) -> int:
        base = self.flags.data_ptr() if r == self.rank else self.remote[r][1]
        return base + 4 * index

    def begin_step(self, compute: torch.cuda.Stream) -> None:
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        ready = self.n_regions * self.world + self.rank
        _lib.flags_signal([self._flag_addr(r, ready) for r in self._peers()], self.epoch, compute.cuda_stream)
        readys = self.flags.data_ptr() + 4 * self.n_regions * self.world
        _lib.flags_wait(readys, self.world, self.rank, self.epoch, self.timeout_s, self.copy_stream.cuda_stream)

    def o_view(self, start: int, n: int) -> torch.Tensor:
        """The 16-bit O buffer's elements at arena offsets [start, start + n)."""
        return self.o_buf[start - self.o_base: start - self.o_base + n]

    def push(self, k: int, ready: torch.cuda.Event, o_region: bool = False) -> None:
        """Push this rank's span of region ``k`` (complete at ``ready``): the
        float32 updates, or (``o_region``) the 16-bit O of that span."""
        start, end = self.ranges[k][self.rank]
        s = self.copy_stream
        s.wait_event(ready)
        if end > start:
            if o_region:
                es = self.o_buf.element_size()
                off = (start - self.o_base) * es
                src, nbytes, buf = self.o_buf.data_ptr() + off, (end - start) * es, 2
            else:
                off = start * 4
                src, nbytes, buf = self.arena.data_ptr() + off, (end - start) * 4, 0
            for r in self._peers():
                _lib.peer_copy(self.remote[r][buf] + off, src, nbytes, s.cuda_stream)
        idx = k * self.world + self.rank
        _lib.flags_signal([self._flag_addr(r, idx) for r in range(self.world)], self.epoch, s.cuda_stream)

    def wait_region(self, k: int, stream: torch.cuda.Stream) -> None:
        """Block ``stream`` until every owner's span of region ``k`` has landed."""
        _lib.flags_wait(self.flags.data_ptr() + 4 * k * self.world, self.world, -1, self.epoch, self.timeout_s,
                        stream.cuda_stream)

    def finish(self, compute: torch.cuda.Stream) -> None:
        """Order ``compute`` after every owner's pushes of this step."""
        _lib.flags_wait(self.flags.data_ptr(), self.n_regions * self.world, -1, self.epoch, self.timeout_s,
                        compute.cuda_stream)
        ev = torch.cuda.Event()
        ev.record(self.copy_stream)
        compute.wait_event(ev)
