"""B200-native (sm_100a) JoLT / FlashJoLT KV-cache compression.

Same Python API as the reference kvcompress package (compressors, payload
schema, cache); the arithmetic runs in the hand-written CUDA kernels of
``kvcompress_b200/_lib/libkvc_b200.so`` (C ABI: ``include/kvc_b200.h``).
"""

from kvcompress_b200.api import CompressionHandle, CompressionStats, disable_compression, enable_compression
from kvcompress_b200.cache import CacheManager, CompressedKVCache, CompressionMetadata
from kvcompress_b200.compressor import (CompressedPayload, CompressorStats, DecodeStream, FlashJoLTCompressor,
                                        IdentityCompressor, IntQuantOnlyCompressor, JoLTCompressor,
                                        JointAllocator, KVCompressor, build_compressor, flashjolt_cap,
                                        supported_methods)

__all__ = ["CacheManager", "CompressedKVCache", "CompressedPayload", "CompressionHandle", "CompressionMetadata",
           "CompressionStats", "disable_compression", "enable_compression",
           "CompressorStats", "DecodeStream", "FlashJoLTCompressor", "IdentityCompressor", "IntQuantOnlyCompressor",
           "JoLTCompressor", "JointAllocator", "KVCompressor", "build_compressor", "flashjolt_cap",
           "supported_methods"]
