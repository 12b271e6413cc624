"""The matrix-SVD ablation baseline of the reference (compressor/lowrank.py)
is not part of the B200 hot path; constructing it fails loudly."""

from __future__ import annotations

from typing import Any

__all__ = ["LowRankCompressor"]


class LowRankCompressor:
    def __init__(self, **kwargs: Any) -> None:
        raise NotImplementedError("the 'lowrank' ablation baseline is not implemented by kvcompress_b200; "
                                  "use 'jolt' or 'flashjolt'")
