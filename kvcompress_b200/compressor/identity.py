"""Cast-only baselines: fp16 / bf16 / float8_e4m3fn storage
(API of kvcompress/compressor/identity.py:31-117).

The casts run in ``kvc_cast``; float8_e4m3fn does not saturate (values that
round past 448 become NaN), as with torch's ``Tensor.to``.
"""

from __future__ import annotations

from typing import Any

import torch

from kvcompress_b200 import ops
from kvcompress_b200.compressor.base import CompressedPayload, CompressorStats, KVCompressor

__all__ = ["IdentityCompressor"]


class IdentityCompressor(KVCompressor):
    """Store K/V in ``factor_dtype`` (fp16 by default)."""

    name = "identity"

    def __init__(self, *, factor_dtype: torch.dtype = torch.float16, **unused: Any) -> None:
        super().__init__()
        self.factor_dtype = factor_dtype

    def _one(self, x: torch.Tensor) -> CompressedPayload:
        stored = ops.cast(x, self.factor_dtype) if x.dtype != self.factor_dtype else x.contiguous().clone()
        return CompressedPayload(
            method="identity", shape=tuple(x.shape), dtype=x.dtype,
            metadata={"r_token": 0, "r_feature": 0, "bits": 0}, data={"value": stored},
            stats=CompressorStats(bytes_original=x.numel() * x.element_size(),
                                  bytes_compressed=x.numel() * self.factor_dtype.itemsize))

    def compress(self, key: torch.Tensor, value: torch.Tensor) -> tuple[CompressedPayload, CompressedPayload]:
        return self._one(key), self._one(value)

    def decompress(self, key_payload: CompressedPayload,
                   value_payload: CompressedPayload) -> tuple[torch.Tensor, torch.Tensor]:
        def back(p):
            v = p.data["value"]
            return ops.cast(v, p.dtype) if v.dtype != p.dtype else v
        return back(key_payload), back(value_payload)
