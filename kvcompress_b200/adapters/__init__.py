"""Callers of the compressor API that move compressed caches in and out."""

from kvcompress_b200.adapters.vllm import export_kv, import_kv, read_payloads, resolve_cache, write_payloads

__all__ = ["export_kv", "import_kv", "read_payloads", "resolve_cache", "write_payloads"]
