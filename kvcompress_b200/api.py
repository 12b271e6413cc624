"""Public model-level API (kvcompress/api.py): ``enable_compression`` patches a
Hugging Face model so its KV cache goes through a compressor, and returns a
``CompressionHandle`` to read statistics and to disable it again."""

from __future__ import annotations

import logging
from dataclasses import dataclass, field
from typing import Any, Literal

from kvcompress_b200.adapters.vllm import parse_target_memory

__all__ = ["CompressionHandle", "CompressionStats", "disable_compression", "enable_compression",
           "parse_target_memory"]

log = logging.getLogger(__name__)

MethodName = Literal["jolt", "flashjolt", "lowrank", "int8", "int4", "int2", "fp8", "fp16", "identity"]


@dataclass
class CompressionStats:
    """Counters of one compression session (api.py:61-86)."""

    compress_calls: int = 0
    decompress_calls: int = 0
    bytes_original: int = 0
    bytes_compressed: int = 0

    @property
    def compression_ratio(self) -> float:
        """``bytes_original / bytes_compressed``; 1.0 before anything was compressed."""
        return self.bytes_original / self.bytes_compressed if self.bytes_compressed else 1.0

    @property
    def memory_saved_bytes(self) -> int:
        return max(0, self.bytes_original - self.bytes_compressed)


@dataclass
class CompressionHandle:
    """What ``enable_compression`` returns (api.py:89-120)."""

    adapter: Any
    model: Any
    stats: CompressionStats = field(default_factory=CompressionStats)

    @property
    def is_active(self) -> bool:
        return bool(self.adapter.enabled)

    def disable(self) -> None:
        """Remove the patches (idempotent)."""
        self.adapter.disable()

    def stats_dict(self) -> dict[str, float]:
        s = self.stats
        return {"compress_calls": s.compress_calls, "decompress_calls": s.decompress_calls,
                "bytes_original": s.bytes_original, "bytes_compressed": s.bytes_compressed,
                "compression_ratio": s.compression_ratio, "memory_saved_bytes": s.memory_saved_bytes}


def enable_compression(model: Any, *, method: MethodName = "flashjolt", target_memory: str | float | None = None,
                       compression_ratio: float | None = None, layer_groups: int = 1,
                       bits: tuple[int, ...] = (0, 2, 4, 8), cache_implementation: str = "kvcompress",
                       seed: int = 0, incremental_block: int | None = None, **kwargs: Any) -> CompressionHandle:
    """Compress ``model``'s KV cache during generation (api.py:123-205).

    Exactly one of ``target_memory`` (``"25%"`` or 0.25: a 4x ratio) and
    ``compression_ratio`` is required (``ValueError`` otherwise); a ratio of 1
    selects the identity compressor.  ``incremental_block=N`` compresses each
    layer in chunks of N tokens as they fill instead of recompressing the
    whole layer on every update (``HuggingFaceAdapter``).  Other keyword
    arguments go to the compressor; an unknown ``method`` raises
    ``NotImplementedError``, a second call on an enabled model
    ``RuntimeError``.
    """
    if (target_memory is None) == (compression_ratio is None):
        raise ValueError("Exactly one of `target_memory` or `compression_ratio` must be provided.")
    if target_memory is not None:
        compression_ratio = parse_target_memory(target_memory)
    extra = dict(kwargs)
    if compression_ratio == 1.0:
        method = "identity"
        extra.pop("rank", None)
    log.info("kvcompress: enabling method=%s ratio=%.2fx on %s", method, compression_ratio, type(model).__name__)
    from kvcompress_b200.adapters.huggingface import HuggingFaceAdapter

    adapter = HuggingFaceAdapter(model=model, method=method, compression_ratio=compression_ratio,
                                 layer_groups=layer_groups, bits=bits, cache_implementation=cache_implementation,
                                 seed=seed, incremental_block=incremental_block, **extra)
    handle = CompressionHandle(adapter=adapter, model=model)
    adapter.stats_ref = handle.stats
    adapter.enable()
    return handle


def disable_compression(handle: CompressionHandle) -> None:
    """``handle.disable()``."""
    handle.disable()
