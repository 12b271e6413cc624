"""Joint Lagrangian allocator (same decisions as kvcompress/compressor/allocator.py).

The reference scans 180 values of the multiplier, brackets and bisects,
evaluating ``error + lambda * cost`` over every (r_token, r_feature, bits)
candidate of every cell in pure Python (allocator.py:169-303, ~25 ms per
compress call).  Here each cell's candidate grid is a pair of numpy arrays
built once per shape and the per-cell argmin is vectorised; the
floating-point operations are the same (``lam * cost`` then ``+ error`` in
float64, first minimum wins), so the decisions are identical.  Results are
memoised by the cells' shapes: the allocation depends on nothing else.

:meth:`JointAllocator.optimize_distributed` runs the same search when the
cells are spread over several ranks: each rank builds the grids of its own
cells, the (cost, error) tables are all-gathered once, and every rank then
runs the identical deterministic search over the global set of cells.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from functools import lru_cache
from typing import Sequence

import numpy as np

__all__ = [
    "Allocation",
    "AllocationResult",
    "Cell",
    "DEFAULT_EPSILON_SQUARED",
    "JointAllocator",
    "bytes_original",
    "candidate_feature_ranks",
    "candidate_token_ranks",
]

# epsilon^2(b) calibration (allocator.py:53)
DEFAULT_EPSILON_SQUARED = {0: 1.0, 2: 0.30, 4: 0.10, 8: 0.04}


@dataclass
class Cell:
    """One (layer group, K/V) allocation target (allocator.py:56-80)."""

    shape: tuple[int, int, int]
    kind: str = "key"
    layer_group: int = 0
    epsilon_squared: dict[int, float] | None = None
    candidate_bits: tuple[int, ...] = (0, 2, 4, 8)
    candidate_token_ranks: tuple[int, ...] | None = None


@dataclass
class Allocation:
    """Per-cell decision (allocator.py:83-104)."""

    r_token: int
    r_feature: int
    bits: int
    cost_bytes: int
    error: float

    @property
    def tuple(self) -> tuple[int, int, int]:
        return (self.r_token, self.r_feature, self.bits)


@dataclass
class AllocationResult:
    """Output of :meth:`JointAllocator.optimize` (allocator.py:107-122)."""

    allocations: list[Allocation] = field(default_factory=list)
    total_bytes: int = 0
    target_bytes: int = 0
    achieved_ratio: float = 1.0
    target_ratio: float = 1.0
    lambda_star: float = 0.0

    def __iter__(self):
        return iter(self.allocations)

    def __len__(self) -> int:
        return len(self.allocations)


def bytes_original(shape: Sequence[int], element_size_bytes: int = 2) -> int:
    """Uncompressed bytes of a cell (allocator.py:613-633)."""
    n = 1
    for s in shape:
        n *= int(s)
    return n * int(element_size_bytes)


def candidate_feature_ranks(d: int) -> list[int]:
    """All ranks up to 32, else a log-spaced subset (allocator.py:636-645)."""
    if d <= 32:
        return list(range(1, d + 1))
    return [c for c in sorted({1, 2, 4, 8, 16, 32, 64, 96, 128, 192, 256, d}) if c <= d]


def candidate_token_ranks(t_max: int) -> list[int]:
    """1..32 then log-spaced up to ``t_max`` (allocator.py:648-654)."""
    if t_max <= 32:
        return list(range(1, t_max + 1))
    extras = sorted({48, 64, 96, 128, 192, 256, 384, 512, t_max})
    return list(range(1, 33)) + [e for e in extras if e <= t_max]


class _Grid:
    """Candidate arrays of one cell, in the reference's enumeration order."""

    __slots__ = ("rt", "rd", "bits", "cost", "err")

    def __init__(self, rt, rd, bits, cost, err):
        self.rt, self.rd, self.bits, self.cost, self.err = rt, rd, bits, cost, err

    def argmin(self, lam: float) -> int:
        return int(np.argmin(self.err + lam * self.costf))

    @property
    def costf(self) -> np.ndarray:
        return self.cost.astype(np.float64)

    def alloc(self, i: int) -> Allocation:
        return Allocation(int(self.rt[i]), int(self.rd[i]), int(self.bits[i]), int(self.cost[i]),
                          float(self.err[i]))


@lru_cache(maxsize=256)
def _default_grid(shape, bits_grid, eps_items, factor_bytes, max_token_rank, token_ranks):
    m, t, d = shape
    eps = dict(eps_items)
    rts = (sorted({int(r) for r in token_ranks}) if token_ranks is not None
           else candidate_token_ranks(min(t, max_token_rank)))
    rds = candidate_feature_ranks(d)
    rt_l, rd_l, b_l, c_l, e_l = [], [], [], [], []
    for rt0 in rts:
        for rd0 in rds:
            rt = min(rt0, t)
            rd = min(rd0, d)
            tucker_bytes = (m * rt * rd + t * rt + d * rd) * factor_bytes
            tau = max(0.0, max(1.0 - rt / max(t, 1), 1.0 - rd / max(d, 1)))
            for b in bits_grid:
                rt_l.append(rt)
                rd_l.append(rd)
                b_l.append(b)
                c_l.append(tucker_bytes + (b // 8) * m * t * d)
                e_l.append(eps.get(b, 1.0) * tau)
    g = _Grid(np.array(rt_l, np.int64), np.array(rd_l, np.int64), np.array(b_l, np.int64),
              np.array(c_l, np.int64), np.array(e_l, np.float64))
    g.err.setflags(write=False)
    return g


class JointAllocator:
    """Per-(layer group, K/V) Lagrangian allocator (allocator.py:125-466)."""

    def __init__(self, target_ratio: float, *, epsilon_squared: dict[int, float] | None = None,
                 factor_dtype_bytes: int = 2, element_size_bytes: int = 2,
                 max_token_rank: int = 512, bits_grid: tuple[int, ...] = (0, 2, 4, 8)) -> None:
        if target_ratio <= 1.0:
            raise ValueError(f"target_ratio must be > 1.0, got {target_ratio}")
        self.target_ratio = float(target_ratio)
        self.epsilon_squared = dict(epsilon_squared or DEFAULT_EPSILON_SQUARED)
        self.factor_dtype_bytes = int(factor_dtype_bytes)
        self.element_size_bytes = int(element_size_bytes)
        self.max_token_rank = int(max_token_rank)
        self.bits_grid = tuple(bits_grid)
        self._memo: dict = {}

    # -- grids ---------------------------------------------------------------

    def build_cell_grid(self, cell: Cell, tau_table=None, idx: int = 0) -> _Grid:
        """Candidate grid of one cell (cost Eq. 1, error Eq. 2; allocator.py:309-375)."""
        eps = cell.epsilon_squared or self.epsilon_squared
        shape = tuple(int(s) for s in cell.shape)
        tr = tuple(cell.candidate_token_ranks) if cell.candidate_token_ranks is not None else None
        g = _default_grid(shape, self.bits_grid, tuple(sorted(eps.items())), self.factor_dtype_bytes,
                          self.max_token_rank, tr)
        if tau_table is None or idx not in tau_table:
            return g
        # empirical tau lookup (allocator.py:401-405), defaulting per entry
        m, t, d = shape
        err = g.err.copy()
        nb = len(self.bits_grid)
        for i in range(0, len(err), nb):
            rt, rd = int(g.rt[i]), int(g.rd[i])
            try:
                tau = float(tau_table[idx][rt * d + rd])
            except (IndexError, TypeError):
                continue
            for j, b in enumerate(self.bits_grid):
                err[i + j] = eps.get(b, 1.0) * tau
        return _Grid(g.rt, g.rd, g.bits, g.cost, err)

    # -- search ----------------------------------------------------------------

    def optimize(self, cells: Sequence[Cell], *, tau_table=None,
                 original_bytes: int | None = None) -> AllocationResult:
        """Allocate ranks and bits across ``cells`` to hit the target ratio."""
        if not cells:
            return AllocationResult(allocations=[], total_bytes=0, target_bytes=0,
                                    achieved_ratio=1.0, target_ratio=self.target_ratio)
        key = None
        if tau_table is None:
            key = (tuple((tuple(c.shape), tuple(sorted((c.epsilon_squared or {}).items())),
                          c.candidate_token_ranks) for c in cells), original_bytes)
            hit = self._memo.get(key)
            if hit is not None:
                return _copy_result(hit)
        grids = [self.build_cell_grid(c, tau_table, i) for i, c in enumerate(cells)]
        per_cell = [bytes_original(c.shape, self.element_size_bytes) for c in cells]
        res = self._search(grids, per_cell, original_bytes)
        if key is not None:
            self._memo[key] = res
        return _copy_result(res)

    def optimize_distributed(self, local_cells: Sequence[Cell], *, group=None) -> tuple[AllocationResult, list[int]]:
        """Global allocation over the cells of every rank.

        Each rank passes its own cells; their candidate tables are
        all-gathered over ``group`` (NCCL on GPUs, gloo on CPU), then every
        rank runs the same search over the concatenated cells.  Returns the
        global result and the indices of this rank's cells in it.
        """
        import torch
        import torch.distributed as dist

        grids = [self.build_cell_grid(c) for c in local_cells]
        per_cell = [bytes_original(c.shape, self.element_size_bytes) for c in local_cells]
        # one flat float64 table: [n, (len, orig, rt.., rd.., bits.., cost.., err..)*]
        parts = [float(len(grids))]
        for g, o in zip(grids, per_cell):
            parts += [float(len(g.err)), float(o)]
            parts += g.rt.astype(np.float64).tolist() + g.rd.astype(np.float64).tolist()
            parts += g.bits.astype(np.float64).tolist() + g.cost.astype(np.float64).tolist()
            parts += g.err.tolist()
        world = dist.get_world_size(group)
        backend = dist.get_backend(group)
        dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
        local = torch.tensor(parts, dtype=torch.float64, device=dev)
        n_local = torch.tensor([local.numel()], dtype=torch.int64, device=dev)
        sizes = [torch.zeros_like(n_local) for _ in range(world)]
        dist.all_gather(sizes, n_local, group=group)
        maxn = int(max(int(s.item()) for s in sizes))
        padded = torch.zeros(maxn, dtype=torch.float64, device=dev)
        padded[: local.numel()] = local
        bufs = [torch.zeros(maxn, dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(bufs, padded, group=group)
        all_grids, all_orig, mine = [], [], []
        me = dist.get_rank(group)
        for r, b in enumerate(bufs):
            v = b.cpu().numpy()
            pos = 1
            for _ in range(int(v[0])):
                n, o = int(v[pos]), int(v[pos + 1])
                pos += 2
                arr = [v[pos + i * n: pos + (i + 1) * n] for i in range(5)]
                pos += 5 * n
                if r == me:
                    mine.append(len(all_grids))
                all_grids.append(_Grid(arr[0].astype(np.int64), arr[1].astype(np.int64),
                                       arr[2].astype(np.int64), arr[3].astype(np.int64),
                                       arr[4].astype(np.float64)))
                all_orig.append(o)
        return self._search(all_grids, all_orig, None), mine

    def _search(self, grids: list[_Grid], per_cell: list[int], original_bytes) -> AllocationResult:
        original = sum(per_cell) if original_bytes is None else int(original_bytes)
        target_bytes = max(1, int(round(original / self.target_ratio)))
        costf = [g.cost.astype(np.float64) for g in grids]

        def argmin(lam):
            return [int(np.argmin(g.err + lam * c)) for g, c in zip(grids, costf)]

        def total(idx):
            return sum(int(g.cost[i]) for g, i in zip(grids, idx))

        log_target = math.log(self.target_ratio)
        cands = []
        for i in range(180):
            lam = 10.0 ** (-12 + 0.1 * i)
            idx = argmin(lam)
            tot = total(idx)
            if tot <= 0:
                continue
            cands.append((abs(math.log(original / tot) - log_target), tot, idx, lam))
        cands.sort(key=lambda c: c[0])
        best_score, _, best_idx, best_lam = cands[0]

        lo = best_lam / 10 if best_lam > 0 else 1e-12
        hi = best_lam * 10 if best_lam > 0 else 1e-6
        cost_lo, cost_hi = total(argmin(lo)), total(argmin(hi))
        if cost_lo > cost_hi:
            lo, hi, cost_lo, cost_hi = hi, lo, cost_hi, cost_lo
        for _ in range(60):
            if cost_lo > target_bytes and cost_hi < target_bytes:
                break
            if cost_lo < target_bytes:
                lo /= 10
                cost_lo = total(argmin(lo))
            elif cost_hi > target_bytes:
                hi *= 10
                cost_hi = total(argmin(hi))
            else:
                break
        for _ in range(40):
            mid = (lo + hi) / 2
            cost_mid = total(argmin(mid))
            if cost_mid > target_bytes:
                lo, cost_lo = mid, cost_mid
            else:
                hi, cost_hi = mid, cost_mid
        idx_mid = argmin((lo + hi) / 2)
        cost_mid = total(idx_mid)
        if cost_mid > 0:
            score_mid = abs(math.log(original / cost_mid) - log_target)
            if score_mid < best_score:
                best_idx, best_lam = idx_mid, (lo + hi) / 2
        allocs = [g.alloc(i) for g, i in zip(grids, best_idx)]
        tot = sum(a.cost_bytes for a in allocs)
        return AllocationResult(allocations=allocs, total_bytes=tot, target_bytes=target_bytes,
                                achieved_ratio=(sum(per_cell) / tot) if tot > 0 else 1.0,
                                target_ratio=self.target_ratio, lambda_star=best_lam)


def _copy_result(r: AllocationResult) -> AllocationResult:
    return AllocationResult(
        allocations=[Allocation(a.r_token, a.r_feature, a.bits, a.cost_bytes, a.error)
                     for a in r.allocations],
        total_bytes=r.total_bytes, target_bytes=r.target_bytes, achieved_ratio=r.achieved_ratio,
        target_ratio=r.target_ratio, lambda_star=r.lambda_star)
