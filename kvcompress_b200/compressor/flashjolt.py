"""FlashJoLT: JoLT with a capped randomised SVD on both Tucker modes
(API of kvcompress/compressor/flashjolt.py:49-210).

The cap policy is ``q_cap = min(max(q_min(R), ceil(T / 32)), 512)`` with
``q_min = 64`` for ``R >= 5`` else 32; the sketch width of a rank-r mode is
``max(min(r + oversampling, q_cap), r + 1)`` clipped to the matrix
(svd.py:447-455), so it reaches 513 when r = 512.  As in the reference's
CapWrapper, the randomised path is used whatever the SVD's ``method``.
"""

from __future__ import annotations

import math
from typing import Any

import torch

from kvcompress_b200.compressor.cells import compress_cells
from kvcompress_b200.compressor.jolt import JoLTCompressor
from kvcompress_b200.compressor.svd import SVD

__all__ = ["FlashJoLTCompressor", "flashjolt_cap"]


def flashjolt_cap(context_length: int, target_ratio: float) -> int:
    """Cap on the randomised sketch (flashjolt.py:49-66)."""
    q_min = 64 if target_ratio >= 5.0 else 32
    return min(max(q_min, math.ceil(context_length / 32)), 512)


class FlashJoLTCompressor(JoLTCompressor):
    """Randomised-SVD variant of JoLT (flashjolt.py:69-169)."""

    name = "flashjolt"

    def __init__(self, *, compression_ratio: float = 3.0, bits: tuple[int, ...] = (0, 2, 4, 8),
                 cap: int | None = None, seed: int = 0, svd: SVD | None = None, **kwargs: Any) -> None:
        kwargs.setdefault("seed", seed)
        effective_svd = svd if svd is not None else SVD(seed=seed, method="randomised")
        super().__init__(compression_ratio=compression_ratio, bits=bits, svd=effective_svd, **kwargs)
        self.auto_cap: int | None = cap

    def _compress_cells(self, xs, rt, rd, bits, t):
        cap = self.auto_cap if self.auto_cap is not None else flashjolt_cap(t, self.compression_ratio)
        cap = cap if isinstance(cap, int) else 32
        return compress_cells(xs, r_token=rt, r_feature=rd, bits=bits, svd=self.svd, cap=cap,
                              forced_randomised=True, seed=self.seed,
                              jl_distribution=self.jl_distribution, symmetric=self.symmetric_quant,
                              per_channel=self.per_channel_quant, group_size=self.group_size,
                              factor_dtype=self.factor_dtype)
