"""Compressed KV cache containers."""

from kvcompress_b200.cache.compress import CompressedKVCache, LayerEntry, normalize_kv, payload_to_meta
from kvcompress_b200.cache.manager import CacheManager
from kvcompress_b200.cache.metadata import CompressionMetadata, LayerCompression

__all__ = ["CacheManager", "CompressedKVCache", "CompressionMetadata", "LayerCompression", "LayerEntry",
           "normalize_kv", "payload_to_meta"]
