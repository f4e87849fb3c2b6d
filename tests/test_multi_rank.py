"""Multi-rank host logic on CPU (gloo, world size 2): the context slicing of one long sequence (BASELINE
config 4) - group ranges, region ownership, the all-gather of partial triples in rank order and their merge -
against attention over the whole context; and the max-over-ranks timing reduction bench.py uses."""
import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "sj-kvarn-codec_b200"))
import slices  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)                  # the same data on every rank
        rows, D, G, n_groups, sink, tail = 8, 64, 16, 12, 5, 9
        n = sink + n_groups * G + tail
        qv = rng.standard_normal((rows, D)).astype(np.float32)
        k = rng.standard_normal((n, D)).astype(np.float32)
        v = rng.standard_normal((n, D)).astype(np.float32)
        scale = 1.0 / np.sqrt(D)
        # this rank's positions: its group slice, the sink on rank 0, the ring on the last rank
        g0, g1 = slices.group_range(rank, world, n_groups)
        reg = slices.regions(rank, world)
        idx = list(range(sink + g0 * G, sink + g1 * G))
        if reg & slices.SJK_REGION_SINK:
            idx = list(range(sink)) + idx
        if reg & slices.SJK_REGION_RING:
            idx = idx + list(range(sink + n_groups * G, n))
        part = torch.from_numpy(slices.partial_np(qv, k[idx], v[idx], scale).astype(np.float32))
        allp = slices.gather(dist, part)
        out = slices.merge_partials_np(allp.numpy())
        s = (qv.astype(np.float64) @ k.astype(np.float64).T) * scale
        p = np.exp(s - s.max(axis=1, keepdims=True))
        ref = (p @ v.astype(np.float64)) / p.sum(axis=1, keepdims=True)
        err = float(np.abs(out - ref).max() / np.abs(ref).max())
        # timing reduction of bench.py: every rank reports its own time, the job time is the max over ranks
        t = torch.tensor([1.0 + rank, 2.0 - rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, err, len(idx), t.tolist()))
    finally:
        dist.destroy_process_group()


def test_context_slices_gloo():
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n_total = 5 + 12 * 16 + 9
    assert sum(r[2] for r in res) == n_total          # every position attended exactly once
    for rank, err, _, t in res:
        assert err < 1e-5, (rank, err)
        assert t == [2.0, 2.0]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_group_ranges_and_regions(world):
    n = 8192
    ranges = [slices.group_range(r, world, n) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    assert max(b - a for a, b in ranges) - min(b - a for a, b in ranges) <= 1
    # weighted by cost (config 4: one sink chunk on rank 0, 32 ring chunks on the last rank)
    w = slices.CHUNK_WEIGHT
    wr = [slices.group_range(r, world, n, sink_chunks=1, tail_chunks=32) for r in range(world)]
    assert wr[0][0] == 0 and wr[-1][1] == n and all(a[1] == b[0] for a, b in zip(wr, wr[1:]))
    cost = [b - a + (w if r == 0 else 0) + (32 * w if r == world - 1 else 0) for r, (a, b) in enumerate(wr)]
    assert max(cost) - min(cost) <= 1.0, cost
    if world > 1:
        assert wr[-1][1] - wr[-1][0] < n // world
    regs = [slices.regions(r, world) for r in range(world)]
    assert sum(1 for r in regs if r & slices.SJK_REGION_SINK) == 1 and regs[0] & slices.SJK_REGION_SINK
    assert sum(1 for r in regs if r & slices.SJK_REGION_RING) == 1 and regs[-1] & slices.SJK_REGION_RING
    assert all(r & slices.SJK_REGION_BODY for r in regs)


def _pool_worker(rank, world, port, q):
    """Config-3 partition on one rank: the LPT owner table of the 64 seeded contexts, gathered from every rank."""
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ctx = np.random.default_rng(3).integers(8192, 65536 + 1, size=64)
        owner = torch.tensor(slices.lpt_assign(ctx, world), dtype=torch.int64)
        allo = [torch.zeros_like(owner) for _ in range(world)]
        dist.all_gather(allo, owner)
        q.put((rank, [a.tolist() for a in allo]))
    finally:
        dist.destroy_process_group()


def test_pool_partition_lpt_two_ranks():
    """Every rank computes the same sequence-to-rank table (no exchange needed), each sequence has one owner,
    and the context loads of the ranks differ by at most the smallest context (the LPT bound for this case)."""
    import multiprocessing as mp
    ctx_ = mp.get_context("spawn")
    q = ctx_.Queue()
    port = _free_port()
    procs = [ctx_.Process(target=_pool_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    tables = [t for _, ts in res for t in ts]
    assert all(t == tables[0] for t in tables)
    ctx = np.random.default_rng(3).integers(8192, 65536 + 1, size=64)
    owner = np.array(tables[0])
    loads = [int(ctx[owner == r].sum()) for r in range(2)]
    assert set(owner.tolist()) == {0, 1} and abs(loads[0] - loads[1]) <= int(ctx.min())


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_lpt_assign_balance(world):
    ctx = np.random.default_rng(3).integers(8192, 65536 + 1, size=64)
    owner = np.array(slices.lpt_assign(ctx, world))
    loads = np.array([ctx[owner == r].sum() for r in range(world)])
    assert owner.min() >= 0 and owner.max() < world
    assert loads.max() - loads.min() <= ctx.max()
    assert slices.lpt_assign(ctx, world) == owner.tolist()
