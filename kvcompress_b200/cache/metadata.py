"""Per-layer compression metadata (schema of kvcompress/cache/metadata.py:32-189)."""

from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any

__all__ = ["CompressionMetadata", "LayerCompression"]


@dataclass
class LayerCompression:
    """One (layer, key|value) entry."""

    layer: int
    kind: str
    m: int
    tokens: int
    dh: int
    r_token: int
    r_feature: int
    bits: int
    core_dtype: str = "fp16"
    seed: int = 0
    bytes_original: int = 0
    bytes_compressed: int = 0
    group_id: int = 0
    group_size: int = 1

    @property
    def shape(self) -> tuple[int, int, int]:
        return (self.m, self.tokens, self.dh)

    @property
    def compression_ratio(self) -> float:
        return 1.0 if self.bytes_compressed == 0 else self.bytes_original / self.bytes_compressed

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "LayerCompression":
        return cls(**d)


@dataclass
class CompressionMetadata:
    """Metadata of one compressed cache; (layer, kind) entries are unique."""

    method: str
    dtype: str
    layers: list[LayerCompression] = field(default_factory=list)
    layer_groups: int = 1
    bits_allowed: tuple[int, ...] = (0, 2, 4, 8)
    extras: dict[str, Any] = field(default_factory=dict)
    index: dict[tuple[int, str], int] = field(default_factory=dict, init=False, repr=False, compare=False)

    def layer(self, idx: int) -> LayerCompression:
        for entry in self.layers:
            if entry.layer == idx:
                return entry
        raise KeyError(f"no metadata for layer {idx}")

    def add_layer(self, entry: LayerCompression) -> None:
        key = (entry.layer, entry.kind)
        if key in self.index:
            self.layers[self.index[key]] = entry
            return
        self.index[key] = len(self.layers)
        self.layers.append(entry)

    def rebuild_index(self) -> None:
        self.index = {(e.layer, e.kind): i for i, e in enumerate(self.layers)}

    def bytes_original(self) -> int:
        return sum(e.bytes_original for e in self.layers)

    def bytes_compressed(self) -> int:
        return sum(e.bytes_compressed for e in self.layers)

    def compression_ratio(self) -> float:
        o, c = self.bytes_original(), self.bytes_compressed()
        return o / c if c else 1.0

    def to_dict(self) -> dict[str, Any]:
        return {"method": self.method, "dtype": self.dtype,
                "layers": [e.to_dict() for e in self.layers], "layer_groups": self.layer_groups,
                "bits_allowed": list(self.bits_allowed), "extras": self.extras}

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "CompressionMetadata":
        meta = cls(method=d["method"], dtype=d["dtype"],
                   layers=[LayerCompression.from_dict(x) for x in d.get("layers", [])],
                   layer_groups=d.get("layer_groups", 1),
                   bits_allowed=tuple(d.get("bits_allowed", (0, 2, 4, 8))), extras=d.get("extras", {}))
        meta.rebuild_index()
        return meta
