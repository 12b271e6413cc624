"""Method name -> compressor, with the reference's kwarg allow-lists
(kvcompress/compressor/dispatch.py:44-177)."""

from __future__ import annotations

import importlib
from typing import Any

import torch

from kvcompress_b200.compressor.base import KVCompressor

__all__ = ["METHODS", "build_compressor", "supported_methods"]

INT_KWARGS = frozenset({"bits", "per_channel", "symmetric", "group_size", "factor_dtype"})
LOWRANK_KWARGS = frozenset({"rank", "factor_dtype", "seed"})
JOLT_KWARGS = frozenset({"compression_ratio", "bits", "factor_dtype", "jl_distribution",
                         "symmetric_quant", "per_channel_quant", "group_size", "layer_groups", "seed"})
IDENTITY_KWARGS = frozenset({"factor_dtype"})

_PKG = "kvcompress_b200.compressor"

METHODS: dict[str, dict[str, Any]] = {
    "jolt": {"class_path": (f"{_PKG}.jolt", "JoLTCompressor"), "allowed_kwargs": JOLT_KWARGS},
    "flashjolt": {"class_path": (f"{_PKG}.flashjolt", "FlashJoLTCompressor"),
                  "allowed_kwargs": JOLT_KWARGS},
    "lowrank": {"class_path": (f"{_PKG}.lowrank", "LowRankCompressor"), "allowed_kwargs": LOWRANK_KWARGS},
    "int2": {"class_path": (f"{_PKG}.quantization_only", "IntQuantOnlyCompressor"),
             "allowed_kwargs": INT_KWARGS, "bits_override": 2},
    "int4": {"class_path": (f"{_PKG}.quantization_only", "IntQuantOnlyCompressor"),
             "allowed_kwargs": INT_KWARGS, "bits_override": 4},
    "int8": {"class_path": (f"{_PKG}.quantization_only", "IntQuantOnlyCompressor"),
             "allowed_kwargs": INT_KWARGS, "bits_override": 8},
    "fp8": {"class_path": (f"{_PKG}.identity", "IdentityCompressor"), "allowed_kwargs": IDENTITY_KWARGS,
            "dtype_override": getattr(torch, "float8_e4m3fn", torch.float16)},
    "fp16": {"class_path": (f"{_PKG}.identity", "IdentityCompressor"), "allowed_kwargs": IDENTITY_KWARGS,
             "dtype_override": torch.float16},
    "bf16": {"class_path": (f"{_PKG}.identity", "IdentityCompressor"), "allowed_kwargs": IDENTITY_KWARGS,
             "dtype_override": torch.bfloat16},
    "identity": {"class_path": (f"{_PKG}.identity", "IdentityCompressor"),
                 "allowed_kwargs": IDENTITY_KWARGS},
}


def supported_methods() -> tuple[str, ...]:
    return tuple(METHODS.keys())


def build_compressor(method: str, **kwargs: Any) -> KVCompressor:
    """Construct a compressor by its public name; unknown kwargs raise ``ValueError``."""
    method = method.lower()
    spec = METHODS.get(method)
    if spec is None:
        supported = ", ".join(repr(m) for m in METHODS)
        raise NotImplementedError(f"compressor method {method!r} is not supported; supported methods: "
                                  f"{supported}.")
    allowed = spec["allowed_kwargs"]
    unknown = set(kwargs) - allowed - {"compression_ratio", "bits", "seed", "layer_groups"}
    if unknown:
        raise ValueError(f"compressor method {method!r} got unexpected kwargs: {sorted(unknown)!r}; "
                         f"supported: {sorted(allowed)!r}.")
    if "bits_override" in spec:
        kwargs.setdefault("bits", spec["bits_override"])
    if "dtype_override" in spec:
        kwargs.setdefault("factor_dtype", spec["dtype_override"])
    module_name, attr = spec["class_path"]
    cls = getattr(importlib.import_module(module_name), attr)
    result = cls(**kwargs)
    if not isinstance(result, KVCompressor):
        raise TypeError(f"{cls.__name__} did not return a KVCompressor")
    return result
