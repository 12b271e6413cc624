"""Layer-indexed compressed KV cache (API of kvcompress/cache/compress.py).

``store`` normalises ``(B, n_kv, T, dh)`` to ``(B*n_kv, T, dh)`` cells and
compresses them; ``retrieve`` decompresses.  ``store_layers`` /
``retrieve_layers`` do many layers per call, batching every layer's K and V
into the same kernel launches when the compressor supports it.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Iterator, Sequence

import torch

from kvcompress_b200.cache.metadata import CompressionMetadata, LayerCompression
from kvcompress_b200.compressor.base import CompressedPayload, KVCompressor

__all__ = ["CompressedKVCache", "LayerEntry", "normalize_kv", "payload_to_meta"]


@dataclass
class LayerEntry:
    layer: int
    key: CompressedPayload | None = None
    value: CompressedPayload | None = None
    extras: dict[str, Any] = field(default_factory=dict)


class CompressedKVCache:
    """In-memory compressed cache with optional LRU eviction (compress.py:79-300)."""

    def __init__(self, compressor: KVCompressor, metadata: CompressionMetadata | None = None,
                 max_layers: int | None = None, device: torch.device | str | None = None) -> None:
        self.compressor = compressor
        self.metadata_ = metadata or CompressionMetadata(method=compressor.name, dtype="unknown")
        self.max_layers = max_layers
        self.device = torch.device(device) if device is not None else None
        self.entries: OrderedDict[int, LayerEntry] = OrderedDict()

    def store(self, layer: int, key: torch.Tensor, value: torch.Tensor, *, group_id: int = 0,
              group_size: int = 1, bits: tuple[int, ...] = (0, 2, 4, 8), seed: int = 0) -> None:
        """Compress and store one layer."""
        self.store_layers([layer], [key], [value], group_id=group_id, group_size=group_size, seed=seed)

    def store_layers(self, layers: Sequence[int], keys: Sequence[torch.Tensor],
                     values: Sequence[torch.Tensor], *, group_id: int = 0, group_size: int = 1,
                     seed: int = 0) -> None:
        """Compress and store several layers in batched launches."""
        pairs = [normalize_kv(k, v) for k, v in zip(keys, values)]
        many = getattr(self.compressor, "compress_many", None)
        if many is not None:
            payloads = many(pairs)
        else:
            payloads = [self.compressor.compress(k, v) for k, v in pairs]
        for layer, (k, v), (kp, vp) in zip(layers, pairs, payloads):
            self.entries[layer] = LayerEntry(layer=layer, key=kp, value=vp)
            self.entries.move_to_end(layer)
            self.metadata_.add_layer(payload_to_meta(layer, "key", k, kp, seed, group_id, group_size))
            self.metadata_.add_layer(payload_to_meta(layer, "value", v, vp, seed, group_id, group_size))
        self.enforce_eviction()

    def retrieve(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Reconstruct one layer's K and V."""
        return self.retrieve_layers([layer])[0]

    def retrieve_layers(self, layers: Sequence[int]) -> list[tuple[torch.Tensor, torch.Tensor]]:
        entries = []
        for layer in layers:
            entry = self.entries.get(layer)
            if entry is None:
                raise KeyError(f"layer {layer} not in cache")
            if entry.key is None or entry.value is None:
                raise KeyError(f"layer {layer} is not fully populated")
            entries.append((entry.key, entry.value))
        many = getattr(self.compressor, "decompress_many", None)
        out = many(entries) if many is not None else [self.compressor.decompress(k, v) for k, v in entries]
        if self.device is not None:
            out = [(k.to(self.device), v.to(self.device)) for k, v in out]
        return out

    def payload(self, layer: int, kind: str) -> CompressedPayload:
        entry = self.entries[layer]
        if kind == "key":
            return entry.key  # type: ignore[return-value]
        if kind == "value":
            return entry.value  # type: ignore[return-value]
        raise ValueError(f"kind must be 'key' or 'value', got {kind!r}")

    def has_layer(self, layer: int) -> bool:
        return layer in self.entries

    def clear(self) -> None:
        self.entries.clear()
        self.metadata_.layers.clear()
        self.metadata_.rebuild_index()

    def evict_layer(self, layer: int) -> None:
        self.entries.pop(layer, None)
        self.metadata_.layers = [e for e in self.metadata_.layers if e.layer != layer]
        self.metadata_.rebuild_index()

    def memory_used(self) -> int:
        return sum(p.bytes_compressed for p in self.all_payloads())

    def memory_original(self) -> int:
        return sum(p.bytes_original for p in self.all_payloads())

    def compression_ratio(self) -> float:
        o, c = self.memory_original(), self.memory_used()
        return o / c if c else 1.0

    def stats(self) -> dict[str, Any]:
        return {"n_layers": len(self.entries), "bytes_original": self.memory_original(),
                "bytes_compressed": self.memory_used(), "compression_ratio": self.compression_ratio(),
                "method": self.compressor.name}

    def metadata(self) -> CompressionMetadata:
        return self.metadata_

    def layers(self) -> Iterator[int]:
        return iter(list(self.entries.keys()))

    def __len__(self) -> int:
        return len(self.entries)

    def __contains__(self, layer: int) -> bool:
        return layer in self.entries

    def all_payloads(self) -> list[CompressedPayload]:
        out: list[CompressedPayload] = []
        for e in self.entries.values():
            if e.key is not None:
                out.append(e.key)
            if e.value is not None:
                out.append(e.value)
        return out

    def enforce_eviction(self) -> None:
        if self.max_layers is None:
            return
        while len(self.entries) > self.max_layers:
            evicted, _ = self.entries.popitem(last=False)
            self.metadata_.layers = [e for e in self.metadata_.layers if e.layer != evicted]
            self.metadata_.rebuild_index()


def normalize_kv(key: torch.Tensor, value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``(B, n_kv, T, dh)`` or ``(n_kv, T, dh)`` -> ``(B*n_kv, T, dh)`` (compress.py:308-333)."""
    if key.shape != value.shape:
        raise ValueError(f"K/V shape mismatch: {key.shape} vs {value.shape}")
    if key.dim() == 4:
        b, h, t, d = key.shape
        return key.reshape(b * h, t, d), value.reshape(b * h, t, d)
    if key.dim() == 3:
        return key, value
    raise ValueError(f"unsupported K/V rank: {key.dim()}")


def payload_to_meta(layer: int, kind: str, original: torch.Tensor, payload: CompressedPayload, seed: int,
                    group_id: int = 0, group_size: int = 1) -> LayerCompression:
    """Metadata entry of one stored payload (compress.py:336-381)."""
    return LayerCompression(
        layer=layer, kind=kind, m=payload.shape[0], tokens=payload.shape[1], dh=payload.shape[2],
        r_token=int(payload.metadata.get("r_token", 0)), r_feature=int(payload.metadata.get("r_feature", 0)),
        bits=int(payload.metadata.get("bits", 0)), core_dtype=str(payload.metadata.get("core_dtype", "fp16")),
        seed=seed, bytes_original=payload.bytes_original, bytes_compressed=payload.bytes_compressed,
        group_id=group_id, group_size=group_size)
