"""The product allocator makes the reference's decisions (CPU, incl. a 2-rank gloo run)."""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from kvcompress_b200.compressor.allocator import Cell, JointAllocator


def test_matches_golden(golden):
    for entry in golden.meta["allocator"]:
        shapes = entry.get("shapes") or [entry["shape"], entry["shape"]]
        alloc = JointAllocator(target_ratio=entry["ratio"], bits_grid=tuple(entry["bits"]))
        res = alloc.optimize([Cell(shape=tuple(s), candidate_bits=tuple(entry["bits"])) for s in shapes])
        got = [[a.r_token, a.r_feature, a.bits, a.cost_bytes, a.error] for a in res.allocations]
        assert got == entry["allocations"]
        assert res.total_bytes == entry["total_bytes"]
        assert res.target_bytes == entry["target_bytes"]
        assert res.achieved_ratio == entry["achieved_ratio"]
        assert res.lambda_star == entry["lambda_star"]
        # memoised second call returns an equal, independent result
        res2 = alloc.optimize([Cell(shape=tuple(s)) for s in shapes])
        assert [a.tuple for a in res2.allocations] == [a.tuple for a in res.allocations]
        res2.allocations[0].r_token = -1
        assert alloc.optimize([Cell(shape=tuple(s)) for s in shapes]).allocations[0].r_token != -1


@pytest.mark.parametrize("shape", [(3, 100, 48), (1, 33, 32), (2, 700, 80)])
@pytest.mark.parametrize("ratio", [1.5, 3.7, 9.0])
def test_matches_oracle_off_grid(shape, ratio):
    res = JointAllocator(target_ratio=ratio).optimize([Cell(shape=shape), Cell(shape=shape)])
    ref = oracle.allocate([shape, shape], ratio)
    assert [list(a.tuple) + [a.cost_bytes, a.error] for a in res.allocations] == \
        [list(a) for a in ref["allocations"]]
    assert res.lambda_star == ref["lambda_star"]


def test_tau_table_and_overrides():
    cells = [Cell(shape=(4, 64, 32), candidate_token_ranks=(1, 2, 4, 8)),
             Cell(shape=(4, 64, 32), epsilon_squared={0: 1.0, 2: 0.5, 4: 0.2, 8: 0.01})]
    tau = {0: [0.5] * (64 * 32 + 64)}
    res = JointAllocator(target_ratio=3.0).optimize(cells, tau_table=tau)
    assert res.allocations[0].r_token in (1, 2, 4, 8)
    assert JointAllocator(target_ratio=3.0).optimize([]).allocations == []
    with pytest.raises(ValueError):
        JointAllocator(target_ratio=1.0)


def _dist_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shapes = [(8, 8192, 128), (8, 8192, 128), (4, 2048, 64), (64, 4096, 128)]
        mine = [Cell(shape=s) for i, s in enumerate(shapes) if i % world == rank]
        res, idx = JointAllocator(target_ratio=4.0).optimize_distributed(mine)
        q.put((rank, [a.tuple for a in res.allocations], idx, res.lambda_star))
    finally:
        dist.destroy_process_group()


def test_distributed_allocation_gloo():
    """A global allocation over cells held by two ranks equals the one-process result."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_dist_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shapes = [(8, 8192, 128), (4, 2048, 64), (8, 8192, 128), (64, 4096, 128)]  # rank 0 cells, rank 1 cells
    ref = JointAllocator(target_ratio=4.0).optimize([Cell(shape=s) for s in shapes])
    for rank, allocs, idx, lam in outs:
        assert allocs == [a.tuple for a in ref.allocations]
        assert lam == ref.lambda_star
        assert idx == ([0, 1] if rank == 0 else [2, 3])


def _shard_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        shape, n_layers = (64, 32768, 128), 32
        layers = bench.my_layers(n_layers, world, rank)
        mine = [Cell(shape=shape, kind=kind) for _ in layers for kind in ("key", "value")]
        res, idx = JointAllocator(target_ratio=4.0).optimize_distributed(mine)
        q.put((rank, layers, [a.tuple for a in res.allocations], [a.cost_bytes for a in res.allocations], idx,
               res.total_bytes))
    finally:
        dist.destroy_process_group()


def test_cell_sharded_cache_allocation_gloo():
    """The benchmark's sharding of one 8 x 32k Llama-3-8B cache over two ranks
    (contiguous layer blocks, K and V cells): the allocation agreed over the
    ranks equals the one-process allocation of all 64 cells and the per-layer
    allocation every compress call uses, and the payload bytes add up to the
    same total."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + ((os.getpid() + 1000) % 2000)
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shape = (64, 32768, 128)
    assert outs[0][1] == list(range(16)) and outs[1][1] == list(range(16, 32))
    one = JointAllocator(target_ratio=4.0).optimize([Cell(shape=shape, kind=k) for _ in range(32)
                                                     for k in ("key", "value")])
    per_layer = JointAllocator(target_ratio=4.0).optimize([Cell(shape=shape, kind="key"),
                                                           Cell(shape=shape, kind="value")])
    for rank, _layers, allocs, costs, idx, total in outs:
        assert allocs == [a.tuple for a in one.allocations]
        assert allocs == [a.tuple for a in per_layer.allocations] * 32
        assert costs == [a.cost_bytes for a in one.allocations]
        assert total == one.total_bytes == 32 * per_layer.total_bytes
        assert idx == list(range(32 * rank, 32 * rank + 32))
