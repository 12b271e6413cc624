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
