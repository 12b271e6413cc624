"""Truncated SVD of the Tucker unfoldings, computed from Gram matrices.

``SVD`` keeps the reference's configuration surface
(kvcompress/compressor/svd.py:123-179: ``oversampling``, ``n_power``,
``seed``, ``method``) and its dispatch rules; the arithmetic runs in the
sm_100a kernels: one streaming pass builds ``A A^T`` (or ``A^T A``) and the
sketch product, then a per-matrix fp64 solver finds the Ritz pairs
(``kvc_gram`` + ``kvc_sketch_solve``).

The Gaussian sketch is the reference's: ``torch.manual_seed(seed)`` followed
by ``torch.randn(n, k)`` on the matrix's device (svd.py:259-260).  It is the
same matrix on every call with the same (n, k, seed, device), so it is drawn
once and cached; on later calls the global generator is reseeded and its
state set to where the reference's draw would leave it, so the RNG side
effects of a compress call match the reference's.
"""

from __future__ import annotations

import threading
from collections import OrderedDict
from dataclasses import dataclass
from typing import Literal

import torch

from kvcompress_b200._native import KVC

__all__ = ["SVD", "SVDResult", "sketch_omega", "sketch_width", "clear_sketch_cache"]


def sketch_width(rows: int, cols: int, rank: int, oversampling: int = 10, cap: int | None = None):
    """Clipped rank and sketch width ``k`` of ``SVD.randomise`` (svd.py:447-455)."""
    max_rank = min(rows, cols)
    rank = max(1, min(int(rank), max_rank))
    k = rank + int(oversampling)
    if cap is not None:
        k = min(k, int(cap))
    k = max(k, rank + 1)
    k = min(k, max_rank)
    return rank, k


_SKETCH: "OrderedDict[tuple, tuple[torch.Tensor, torch.Tensor | None]]" = OrderedDict()
_SKETCH_LOCK = threading.Lock()
_SKETCH_MAX = 8


def _seed_generators(seed: int) -> None:
    """``torch.manual_seed(seed)`` for the CPU and CUDA generators.

    Seeds the same generators as ``torch.manual_seed`` on a CUDA host without
    its deferred-initialisation bookkeeping for other device types (a stack
    capture per call, the largest host cost of a compress call)."""
    torch.random.default_generator.manual_seed(seed)
    if torch.cuda.is_initialized():
        for g in torch.cuda.default_generators:
            g.manual_seed(seed)
    else:
        torch.cuda.manual_seed_all(seed)


def sketch_omega(n: int, k: int, seed: int, device: torch.device) -> torch.Tensor:
    """The reference's sketch ``torch.manual_seed(seed); torch.randn(n, k)`` on ``device``."""
    device = torch.device(device)
    key = (int(n), int(k), int(seed), str(device))
    _seed_generators(int(seed))
    with _SKETCH_LOCK:
        hit = _SKETCH.get(key)
        if hit is not None:
            _SKETCH.move_to_end(key)
            om, state = hit
            if state is not None:
                torch.cuda.set_rng_state(state, device)
            return om
        om = torch.randn(int(n), int(k), dtype=torch.float32, device=device)
        state = torch.cuda.get_rng_state(device) if device.type == "cuda" else None
        _SKETCH[key] = (om, state)
        while len(_SKETCH) > _SKETCH_MAX:
            _SKETCH.popitem(last=False)
        return om


def clear_sketch_cache() -> None:
    with _SKETCH_LOCK:
        _SKETCH.clear()


@dataclass
class SVDResult:
    """Leading left singular vectors, squared singular values and tail mass."""

    u: torch.Tensor
    s: torch.Tensor
    tail_mass: torch.Tensor  # float64, one value per matrix (device)
    method: Literal["exact", "randomised"]


class SVD:
    """Exact / randomised SVD configuration (svd.py:123-179).

    ``method``: ``"auto"`` picks randomised when ``rank < min(shape) // 2``;
    ``"exact"`` and ``"randomised"`` force a path.
    """

    def __init__(self, *, oversampling: int = 10, n_power: int = 2, seed: int = 0,
                 method: Literal["auto", "exact", "randomised"] = "auto") -> None:
        self.oversampling = int(oversampling)
        self.n_power = int(n_power)
        self.seed = int(seed)
        self.method = method

    def resolve(self, rows: int, cols: int, rank: int | None, cap: int | None, forced_randomised=False):
        """Mode, clipped rank and sketch width the reference would use.

        ``forced_randomised`` mirrors FlashJoLT's CapWrapper, which always
        calls ``randomise`` (flashjolt.py:188-192).
        """
        max_rank = min(rows, cols)
        if rank is None:
            return KVC.SVD_EXACT, max_rank, 0
        r = max(1, min(int(rank), max_rank))
        if forced_randomised or self.method == "randomised" or (
                self.method == "auto" and r < max_rank // 2):
            r, k = sketch_width(rows, cols, r, self.oversampling, cap)
            return KVC.SVD_RANDOMISED, r, k
        return KVC.SVD_EXACT, r, 0

    def __call__(self, a: torch.Tensor, *, rank: int | None = None, cap: int | None = None) -> SVDResult:
        """Truncated SVD of a CUDA matrix (one matrix; the compressors batch cells)."""
        from kvcompress_b200 import ops

        if a.dim() != 2:
            raise ValueError(f"SVD expects a 2-D matrix, got shape {tuple(a.shape)}")
        rows, cols = a.shape
        mode, r, k = self.resolve(rows, cols, rank, cap)
        a = a.contiguous()
        dt = a.dtype if a.dtype in (torch.float32, torch.float16, torch.bfloat16) else torch.float32
        if a.dtype != dt:
            a = a.to(dt)
        if rows <= cols:
            # left side: Gram of the (cols x rows) transpose view
            at = a.t().contiguous()
            om = sketch_omega(cols, k, self.seed, a.device) if mode == KVC.SVD_RANDOMISED else None
            g = ops.gram([at], om)
            u, tail, sv2 = ops.sketch_solve(g, mode=mode, side=KVC.SIDE_LEFT, p=rows, n_other=cols,
                                            k=k, rank=r, n_power=self.n_power, omega=None,
                                            basis_dtype=dt)
            u = u[0]
        else:
            om = sketch_omega(cols, k, self.seed, a.device) if mode == KVC.SVD_RANDOMISED else None
            g = ops.gram([a], None)
            mat, tail, sv2 = ops.sketch_solve(g, mode=mode, side=KVC.SIDE_RIGHT, p=cols, n_other=rows,
                                              k=k, rank=r, n_power=self.n_power, omega=om,
                                              basis_dtype=torch.float64)
            u = ops.apply_basis([a], mat)[0]
        return SVDResult(u=u, s=sv2[0].clamp_min(0).sqrt(), tail_mass=tail[0],
                         method="exact" if mode == KVC.SVD_EXACT else "randomised")
