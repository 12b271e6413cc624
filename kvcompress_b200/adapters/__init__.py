"""Callers of the compressor API that move compressed caches in and out.

The vLLM offload handler (``JoLTOffloadHandler`` and friends) is imported on
first use, as in the reference (kvcompress/adapters/__init__.py)."""

from typing import Any

from kvcompress_b200.adapters.vllm import export_kv, import_kv, read_payloads, resolve_cache, write_payloads

_OFFLOAD = ("JoLTOffloadHandler", "ThreadSafeEvictionPool", "is_vllm_kv_offload_available", "import_vllm_base")

__all__ = ["export_kv", "import_kv", "read_payloads", "resolve_cache", "write_payloads", *_OFFLOAD]


def __getattr__(name: str) -> Any:
    if name in _OFFLOAD:
        from kvcompress_b200.adapters import vllm_kv_offload

        return getattr(vllm_kv_offload, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
