"""Multi-GPU host logic on CPU: leaf ownership (LPT on NS FLOPs), bucket
layout, and the bucketed owner-computes / all-gather exchange over world-size-2
gloo process groups."""

import os
import socket

import pytest
import torch

from rollfast_b200.distributed import bucket_buffers, lpt_assign, make_plan, ns_flops, run_buckets


def llama_leaves():
    layer = [(4096, 4096), (4096, 1024), (4096, 1024), (4096, 4096), (4096, 14336), (4096, 14336), (14336, 4096)]
    return [s for _ in range(32) for s in layer]


def test_ns_flops_counts_the_smaller_side_as_m():
    assert ns_flops(1, 4096, 14336) == 4 * 4096 ** 2 * 14336 + 2 * 4096 ** 3
    assert ns_flops(2, 14336, 4096) == 2 * ns_flops(1, 4096, 14336)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_lpt_balances_llama_leaves_exactly(world):
    leaves = llama_leaves()
    costs = [ns_flops(1, *s) for s in leaves]
    owner = lpt_assign(costs, world)
    loads = [0] * world
    for c, r in zip(costs, owner):
        loads[r] += c
    assert max(loads) == min(loads)  # 96 / 64 / 64 leaves of three costs divide evenly
    assert sorted(set(owner)) == list(range(world))


def test_lpt_is_deterministic_and_bounded():
    costs = [7, 7, 5, 3, 3, 2, 1, 1]
    a = lpt_assign(costs, 3)
    assert a == lpt_assign(costs, 3)
    loads = [sum(c for c, r in zip(costs, a) if r == k) for k in range(3)]
    assert max(loads) <= sum(costs) / 3 + max(costs)


@pytest.mark.parametrize("world,buckets", [(2, 1), (2, 4), (8, 4), (3, 3)])
def test_bucket_layout_covers_every_leaf_once(world, buckets):
    leaves = llama_leaves()
    sizes = [a * b for a, b in leaves]
    costs = [ns_flops(1, *s) for s in leaves]
    plan = make_plan(sizes, costs, world, buckets)
    seen = [i for b in plan.buckets for i in b.leaves]
    assert [b.index for b in plan.buckets] == list(range(len(plan.buckets)))
    assert seen == list(range(len(leaves)))
    assert len(plan.buckets) <= buckets
    for b in plan.buckets:
        used = [0] * world
        for i in b.leaves:
            r, off = b.offsets[i]
            assert r == plan.owner[i] and off == used[r]
            used[r] += sizes[i]
        assert b.seg == -(-max(used) // 64) * 64 and b.used == used
    if len(plan.buckets) > 2:  # small last bucket: short exposed final gather
        bc = [sum(costs[i] for i in b.leaves) for b in plan.buckets]
        assert bc[-1] < max(bc)


def test_bucket_weights_shape():
    from rollfast_b200.distributed import bucket_weights

    assert bucket_weights(1) == [1.0]
    assert bucket_weights(4) == [8.0, 4.0, 2.0, 1.0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, sizes, costs, buckets, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = make_plan(sizes, costs, world, buckets)

        def compute_owned(ids, offsets, send):
            for i in ids:  # stand-in for the NS output of leaf i, computed by its owner
                send[offsets[i]: offsets[i] + sizes[i]] = torch.arange(sizes[i], dtype=torch.float32) + 1000.0 * i

        def exchange(bucket, send, recv):
            dist.all_gather_into_tensor(recv, send)

        buffers = bucket_buffers(plan, world, torch.float32, torch.device("cpu"))
        views = []
        for _ in range(2):  # persistent buffers reused on a second step
            views = run_buckets(plan, rank, world, sizes, compute_owned, exchange, buffers)
        ok = sorted(i for i, _ in views) == list(range(len(sizes)))
        for i, v in views:
            ok &= bool(torch.equal(v, torch.arange(sizes[i], dtype=torch.float32) + 1000.0 * i))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("buckets", [1, 3])
def test_gloo_world2_owner_compute_and_all_gather(buckets):
    import torch.multiprocessing as mp

    sizes = [96, 40, 40, 96, 300, 300, 300, 17, 5]
    costs = [ns_flops(1, 8, s // 8 if s % 8 == 0 else s) for s in sizes]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, sizes, costs, buckets, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}


def _configure_worker(rank, world, port, q):
    import torch.distributed as dist

    import rollfast_b200.distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = {}
        try:
            D.configure(transport="bogus")
            res["bad"] = "accepted"
        except ValueError:
            res["bad"] = "rejected"
        ctx = D.configure(transport="NCCL", buckets=3)
        res["ctx"] = (ctx.rank, ctx.world_size, ctx.transport, ctx.buckets, D.active_transport())
        prev = D.use(None)
        res["use"] = (prev is ctx, D.current() is None, D.active_transport())
        D.use(ctx)
        os.environ["ROLLFAST_DIST_GATHER"] = "ce"
        res["env"] = D.configure().transport
        D.clear()
        res["cleared"] = D.current() is None
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_configure_transport_selection():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_configure_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        res = results[r]
        assert res["bad"] == "rejected"
        assert res["ctx"] == (r, 2, "nccl", 3, "nccl")
        assert res["use"] == (True, True, "none")
        assert res["env"] == "ce" and res["cleared"]


def _consolidate_worker(rank, world, port, q):
    import torch.distributed as dist

    import rollfast_b200.distributed as D

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ctx = D.configure(transport="nccl")
        owners = [0, 1, 1, 0, 1]
        mus = [torch.full((3, 4), -1.0) for _ in owners]
        for i, (t, o) in enumerate(zip(mus, owners)):
            if o == rank:
                t.fill_(10.0 * i + o)   # only the owner's copy is current
        ctx.owned_state = list(zip(mus, owners))
        n = D.consolidate_momentum()
        ok = n == len(owners) and all(bool((t == 10.0 * i + o).all()) for i, (t, o) in enumerate(zip(mus, owners)))
        D.clear()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_consolidate_momentum_from_owners():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_consolidate_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}


def llama70b_meta_tree(layers=80):
    d, kv, ff = 8192, 1024, 28672
    mk = lambda *s: torch.empty(s, dtype=torch.bfloat16, device="meta")  # noqa: E731
    tree = {"final_norm": mk(d)}
    for i in range(layers):
        tree[f"l{i:02d}"] = {"q": mk(d, d), "k": mk(d, kv), "v": mk(d, kv), "o": mk(d, d), "gate": mk(d, ff),
                             "up": mk(d, ff), "down": mk(ff, d), "attn_norm": mk(d), "mlp_norm": mk(d)}
    return tree


def test_ownership_of_llama70b_is_flop_balanced_and_matches_the_update_planner():
    """updates="owned": the public ownership tree, from
    shapes alone (meta tensors), equals the assignment the sharded update
    makes, and balances the 80-layer tree exactly over 8 ranks
    (30 / 20 / 20 gate-up-down / q-o / k-v matrices per rank)."""
    import rollfast_b200 as rf
    from rollfast_b200.distributed import owner_ranks, ownership
    from rollfast_b200.tree import tree_leaves

    tree = llama70b_meta_tree()
    own = ownership(tree, world_size=8)
    owners = tree_leaves(own)
    flat = tree_leaves(tree)
    muon_shapes = [tuple([1, *x.shape]) for x in flat if x.ndim == 2]
    adam = [x.numel() for x in flat if x.ndim == 1]
    mo, ao = owner_ranks(muon_shapes, adam, 8)
    assert [r for r, x in zip(owners, flat) if x.ndim == 2] == mo
    assert [r for r, x in zip(owners, flat) if x.ndim == 1] == ao
    loads = [0] * 8
    for s, r in zip(muon_shapes, mo):
        loads[r] += ns_flops(*s)
    assert max(loads) == min(loads)
    counts = {}
    for s, r in zip(muon_shapes, mo):
        counts.setdefault(r, []).append(min(s[1:]) * max(s[1:]))
    assert all(len(v) == 70 for v in counts.values())
    # A meta tree initialises without allocating: the state of leaves a rank
    # does not own can stay meta.
    st = rf.muon(learning_rate=0.01).init({"w": torch.empty(64, 128, device="meta")})
    assert st.inner_states["muon"].inner_state[0][0].mu["w"].is_meta
