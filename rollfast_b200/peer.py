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
