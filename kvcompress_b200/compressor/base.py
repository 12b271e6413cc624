"""Compressor contract and self-describing payload.

Same interface as the reference (kvcompress/compressor/base.py:37-208):
``compress(K, V) -> (key_payload, value_payload)`` and
``decompress(key_payload, value_payload) -> (K, V)``; a payload's byte count
is the sum of the tensors in ``data`` (base.py:113-128).
"""

from __future__ import annotations

import abc
from dataclasses import dataclass, field
from typing import Any

import torch

__all__ = ["CompressorStats", "CompressedPayload", "KVCompressor"]


@dataclass
class CompressorStats:
    """Per-call statistics (fields as in base.py:37-83)."""

    compress_time_ms: float = 0.0
    decompress_time_ms: float = 0.0
    bytes_original: int = 0
    bytes_compressed: int = 0
    reconstruction_error: float | None = None
    extra: dict[str, Any] = field(default_factory=dict)

    def to_dict(self) -> dict[str, Any]:
        """Flat dict with the derived ``compression_ratio``."""
        return {
            "compress_time_ms": self.compress_time_ms,
            "decompress_time_ms": self.decompress_time_ms,
            "bytes_original": self.bytes_original,
            "bytes_compressed": self.bytes_compressed,
            "compression_ratio": self.compression_ratio,
            "reconstruction_error": self.reconstruction_error,
            **self.extra,
        }

    @property
    def compression_ratio(self) -> float:
        """``bytes_original / bytes_compressed``; 1.0 when nothing was stored."""
        if self.bytes_compressed == 0:
            return 1.0
        return self.bytes_original / self.bytes_compressed


@dataclass
class CompressedPayload:
    """Container for one compressed tensor (fields as in base.py:86-140)."""

    method: str
    shape: tuple[int, ...] | torch.Size
    dtype: torch.dtype
    metadata: dict[str, Any]
    data: dict[str, Any]
    stats: CompressorStats = field(default_factory=CompressorStats)

    @property
    def bytes_compressed(self) -> int:
        """Bytes of every tensor in ``data`` (one level of nested dicts)."""
        total = 0
        for v in self.data.values():
            if isinstance(v, torch.Tensor):
                total += v.numel() * v.element_size()
            elif isinstance(v, dict):
                for vv in v.values():
                    if isinstance(vv, torch.Tensor):
                        total += vv.numel() * vv.element_size()
        return total

    @property
    def bytes_original(self) -> int:
        """``prod(shape) * itemsize(dtype)``."""
        n = 1
        for s in self.shape:
            n *= int(s)
        return n * torch.empty((), dtype=self.dtype).element_size()


class KVCompressor(abc.ABC):
    """Abstract compressor: ``compress`` / ``decompress`` are inverses."""

    name: str = "base"

    def __init__(self, **kwargs: Any) -> None:
        for k, v in kwargs.items():
            setattr(self, k, v)

    @abc.abstractmethod
    def compress(self, key: torch.Tensor, value: torch.Tensor) -> tuple[CompressedPayload, CompressedPayload]:
        """Compress one layer's ``(m, T, dh)`` K and V."""
        raise NotImplementedError

    @abc.abstractmethod
    def decompress(self, key_payload: CompressedPayload,
                   value_payload: CompressedPayload) -> tuple[torch.Tensor, torch.Tensor]:
        """Inverse of :meth:`compress`."""
        raise NotImplementedError

    def estimate_size(self, payload: CompressedPayload) -> int:
        """Bytes occupied by ``payload``."""
        return payload.bytes_compressed

    def stats(self) -> dict[str, Any]:
        """Aggregated statistics; subclasses override."""
        return {}

    def __repr__(self) -> str:
        return f"{type(self).__name__}(name={self.name!r})"
