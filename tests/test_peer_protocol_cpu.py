"""Copy-engine gather protocol (rollfast_b200/peer.py) on CPU.

The library's peer calls are replaced by in-process equivalents over CPU
tensors: a push is a memmove between the ranks' buffers, a flag signal a
32-bit store, and a flag wait asserts that its condition already holds.  The
ranks then run their steps in lockstep phases (all pushes of a bucket before
any tail of it), which is one legal interleaving of the device-side protocol:
every wait must be satisfied and every gathered slot must hold its owner's
data."""

import ctypes

import pytest
import torch

from rollfast_b200 import peer
from rollfast_b200.distributed import make_plan, ns_flops
from rollfast_b200.peer import PeerGather, _Remote, ack_index, ce_layout, flag_index


class _Stream:
    cuda_stream = 0

    def __init__(self, *a, **k):
        pass

    def wait_event(self, ev):
        pass


class _Event:
    def record(self, *a):
        pass


def _u32(addr):
    return ctypes.c_uint32.from_address(addr).value


class _FakeLib:
    def __init__(self):
        self.copied = 0

    def peer_copy(self, dst, src, nbytes, stream):
        ctypes.memmove(dst, src, nbytes)
        self.copied += nbytes

    def flags_signal(self, addrs, value, stream):
        for a in addrs:
            ctypes.c_uint32.from_address(a).value = value & 0xFFFFFFFF

    def flags_wait(self, addr, n, skip, target, timeout_s, stream):
        for i in range(n):
            if i != skip:
                v = _u32(addr + 4 * i)
                if ((v - target) & 0xFFFFFFFF) >= 1 << 31:
                    raise AssertionError(f"flag {i} = {v} < {target}: wait would time out")


@pytest.fixture
def fake(monkeypatch):
    lib = _FakeLib()
    monkeypatch.setattr(torch.cuda, "Stream", _Stream)
    monkeypatch.setattr(torch.cuda, "Event", _Event)
    monkeypatch.setattr(peer, "_lib", lib)
    return lib


def _ranks(sizes, world, buckets):
    costs = [ns_flops(1, 8, s) for s in sizes]
    plan = make_plan(sizes, costs, world, buckets)
    gs = [PeerGather(plan, r, world, None, torch.float16, torch.device("cpu"), timeout_s=1.0) for r in range(world)]
    for r, g in enumerate(gs):
        for q, h in enumerate(gs):
            if q != r:
                g.remote[q] = _Remote(h.buf.data_ptr(), h.flags.data_ptr())
    return plan, gs


def _value(step, leaf, n):
    return (torch.arange(n, dtype=torch.float32) % 251 + 7 * leaf + 1000 * step).to(torch.float16)


def test_layout_is_aligned_and_flags_are_distinct():
    offs, total = ce_layout([10, 64, 0, 5], 3)
    assert offs == [0, 64, 256, 256] and total == 320
    assert all(o % 64 == 0 for o in offs)
    idx = {flag_index(k, s, 4) for k in range(3) for s in range(4)} | {ack_index(s, 3, 4) for s in range(4)}
    assert len(idx) == 3 * 4 + 4 == max(idx) + 1


@pytest.mark.parametrize("world,buckets", [(2, 1), (2, 3), (4, 2), (3, 4)])
def test_lockstep_steps_gather_every_slot(fake, world, buckets):
    sizes = [96, 40, 40, 96, 300, 300, 300, 17, 5, 128]
    plan, gs = _ranks(sizes, world, buckets)
    es = 2
    for step in range(1, 4):
        for g in gs:
            g.begin_step()
        for k, b in enumerate(plan.buckets):
            for r, g in enumerate(gs):  # owners write their slots, then push
                slot, _ = g.buffers[k]
                for i in b.leaves:
                    o, off = b.offsets[i]
                    if o == r:
                        slot[off: off + sizes[i]] = _value(step, i, sizes[i])
                g.push(k, _Event())
            for r, g in enumerate(gs):  # every receiver's wait holds, data landed
                g.wait_bucket(k, _Stream())
                _, region = g.buffers[k]
                for i in b.leaves:
                    o, off = b.offsets[i]
                    got = region[o * b.seg + off: o * b.seg + off + sizes[i]]
                    assert torch.equal(got, _value(step, i, sizes[i])), (step, k, r, i)
        for g in gs:
            g.end_step(_Stream(), _Stream())
        assert all(g.epoch == step for g in gs)
    # each rank pushed exactly its used elements to every peer, every step
    per_step = sum(b.used[r] for b in plan.buckets for r in range(world)) * (world - 1) * es
    assert fake.copied == 3 * per_step


def test_missing_ack_blocks_the_next_push(fake):
    sizes = [64, 64, 64, 64]
    plan, gs = _ranks(sizes, 2, 1)
    for g in gs:
        g.begin_step()
    for g in gs:
        g.push(0, _Event())
    for g in gs:
        g.wait_bucket(0, _Stream())
    gs[0].end_step(_Stream(), _Stream())  # rank 1 has not finished reading step 1
    with pytest.raises(AssertionError, match="wait would time out"):
        gs[0].begin_step()                # rank 0 must not push step 2 into rank 1 yet


def test_tail_wait_fails_before_peer_pushes(fake):
    plan, gs = _ranks([64, 64, 64, 64], 2, 1)
    for g in gs:
        g.begin_step()
    gs[0].push(0, _Event())
    with pytest.raises(AssertionError):
        gs[0].wait_bucket(0, _Stream())   # rank 1 has not pushed bucket 0
