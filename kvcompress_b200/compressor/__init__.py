"""Compressors with the reference's API, running on the sm_100a kernels."""

from kvcompress_b200.compressor.allocator import (Allocation, AllocationResult, Cell,
                                                   JointAllocator)
from kvcompress_b200.compressor.base import CompressedPayload, CompressorStats, KVCompressor
from kvcompress_b200.compressor.dispatch import METHODS, build_compressor, supported_methods
from kvcompress_b200.compressor.flashjolt import FlashJoLTCompressor, flashjolt_cap
from kvcompress_b200.compressor.identity import IdentityCompressor
from kvcompress_b200.compressor.jolt import JoLTCompressor
from kvcompress_b200.compressor.quantization_only import IntQuantOnlyCompressor
from kvcompress_b200.compressor.stream import DecodeStream

__all__ = ["Allocation", "AllocationResult", "Cell", "CompressedPayload", "CompressorStats",
           "DecodeStream", "FlashJoLTCompressor", "IdentityCompressor", "IntQuantOnlyCompressor", "JoLTCompressor",
           "JointAllocator", "KVCompressor", "METHODS", "build_compressor", "flashjolt_cap",
           "supported_methods"]
