"""Quantise-only baseline: int2/4/8 per channel over head_dim
(API of kvcompress/compressor/quantization_only.py:56-198).

As in the reference, ``group_size`` is accepted and ignored, and the
statistics and scale arithmetic run in the cache dtype.  K and V are
quantised in one launch per stage and decoded in one launch.
"""

from __future__ import annotations

from typing import Any

import torch

from kvcompress_b200.compressor.base import CompressedPayload, CompressorStats, KVCompressor
from kvcompress_b200.compressor.quantization import IntQuantizer

__all__ = ["IntQuantOnlyCompressor"]


class IntQuantOnlyCompressor(KVCompressor):
    """Integer quantisation, no Tucker, no rotation."""

    name = "int-quant-only"

    def __init__(self, *, bits: int = 4, per_channel: bool = True, symmetric: bool = True,
                 **unused: Any) -> None:
        super().__init__()
        self.bits = int(bits)
        self.per_channel = per_channel
        self.symmetric = symmetric
        self.quantizer = IntQuantizer(bits=bits, symmetric=symmetric, per_channel=per_channel)

    def compress(self, key: torch.Tensor, value: torch.Tensor) -> tuple[CompressedPayload, CompressedPayload]:
        if key.shape == value.shape and key.dtype == value.dtype:
            d = key.shape[-1]
            codes, scales, zps = self.quantizer.quantize_many([key.reshape(-1, d), value.reshape(-1, d)])
            return (self._payload(key, codes[0], scales[0], zps[0]),
                    self._payload(value, codes[1], scales[1], zps[1]))
        return self.compress_one(key), self.compress_one(value)

    def decompress(self, key_payload: CompressedPayload,
                   value_payload: CompressedPayload) -> tuple[torch.Tensor, torch.Tensor]:
        return self.decompress_one(key_payload), self.decompress_one(value_payload)

    def compress_one(self, x: torch.Tensor) -> CompressedPayload:
        d = x.shape[-1]
        q, s, z = self.quantizer.quantize(x.reshape(-1, d))
        return self._payload(x, q, s, z)

    def _payload(self, x, q, s, z) -> CompressedPayload:
        d = int(x.shape[-1])
        return CompressedPayload(
            method=f"int{self.bits}-only", shape=tuple(x.shape), dtype=x.dtype,
            metadata={"bits": self.bits, "symmetric": self.symmetric,
                      "per_channel": self.per_channel, "original_last": d},
            data={"q": q, "scale": s, "zero_point": z,
                  "original_last": torch.tensor(d, dtype=torch.int32)},
            stats=CompressorStats(bytes_original=x.numel() * x.element_size(),
                                  bytes_compressed=q.numel() * q.element_size()
                                  + s.numel() * s.element_size() + z.numel() * z.element_size()))

    def decompress_one(self, payload: CompressedPayload) -> torch.Tensor:
        md = payload.metadata
        qz = IntQuantizer(bits=int(md["bits"]), symmetric=bool(md["symmetric"]),
                          per_channel=bool(md["per_channel"]))
        flat = qz.dequantize(payload.data["q"], payload.data["scale"], payload.data["zero_point"],
                             original_last=int(md.get("original_last", payload.shape[-1])),
                             output_dtype=payload.dtype)
        return flat.reshape(payload.shape)
