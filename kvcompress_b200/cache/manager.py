"""Cache facade used by model adapters (API of kvcompress/cache/manager.py:35-137)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Iterator, Sequence

import torch

from kvcompress_b200.cache.compress import CompressedKVCache
from kvcompress_b200.cache.metadata import CompressionMetadata
from kvcompress_b200.compressor.base import KVCompressor

__all__ = ["CacheManager"]


@dataclass
class CacheManager:
    compressor: KVCompressor
    max_layers: int | None = None
    device: torch.device | str | None = None
    cache: CompressedKVCache = field(init=False)
    live_layers: list[int] = field(default_factory=list, init=False)

    def __post_init__(self) -> None:
        self.cache = CompressedKVCache(compressor=self.compressor, max_layers=self.max_layers,
                                       device=self.device)

    def store(self, layer: int, key: torch.Tensor, value: torch.Tensor, **kwargs: Any) -> None:
        self.cache.store(layer, key, value, **kwargs)
        if layer not in self.live_layers:
            self.live_layers.append(layer)

    def store_layers(self, layers: Sequence[int], keys: Sequence[torch.Tensor], values: Sequence[torch.Tensor],
                     **kwargs: Any) -> None:
        """``store`` of several layers as one batched compress."""
        self.cache.store_layers(layers, keys, values, **kwargs)
        for layer in layers:
            if layer not in self.live_layers:
                self.live_layers.append(layer)

    def retrieve(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.cache.retrieve(layer)

    def clear(self) -> None:
        self.cache.clear()
        self.live_layers.clear()

    def evict(self, layer: int) -> None:
        self.cache.evict_layer(layer)
        self.live_layers = [e for e in self.live_layers if e != layer]

    def memory_used(self) -> int:
        return self.cache.memory_used()

    def memory_original(self) -> int:
        return self.cache.memory_original()

    def compression_ratio(self) -> float:
        return self.cache.compression_ratio()

    def stats(self) -> dict[str, Any]:
        s = self.cache.stats()
        s["live_layers"] = list(self.live_layers)
        return s

    def metadata(self) -> CompressionMetadata:
        return self.cache.metadata()

    def layers(self) -> Iterator[int]:
        return self.cache.layers()

    def __len__(self) -> int:
        return len(self.cache)

    def __contains__(self, layer: int) -> bool:
        return layer in self.cache
