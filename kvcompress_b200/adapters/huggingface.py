"""Hugging Face adapter: a ``DynamicCache`` subclass that compresses the cache
(API of kvcompress/adapters/huggingface.py).

``HuggingFaceAdapter.enable`` replaces ``DynamicCache`` in
``transformers.cache_utils`` and in every loaded ``transformers.*`` module
that imported it by name, so the model's generation instantiates
``KvCompressCache``; ``disable`` puts the original class back and restores
the model's ``generation_config.cache_implementation``.

``KvCompressCache.update`` calls the parent's update (which concatenates the
new tokens) and then mirrors the layer into the adapter's compressed store;
``__getitem__`` replaces the layer's K / V by their reconstruction before
returning them.  Two store modes:

* ``incremental_block=None`` (the reference's behaviour,
  huggingface.py:330-372): every update compresses the layer's whole
  current K / V (``CacheManager.store``), so a decode step costs a compress
  of all T tokens of the layer.
* ``incremental_block=N``: the layer's tokens are compressed in chunks of N
  as the chunks fill up, each chunk once (``(B * n_kv, N, dh)`` cells; all
  chunks completed by one update, e.g. a long prefill, go through one
  batched compress).  Tokens past the last full chunk stay as they are.
  A decode step then compresses nothing until a chunk completes, and a
  read decodes only the chunks added since the previous read (earlier
  chunks' reconstructions are kept).  The reconstruction is the chunks'
  decodes followed by the uncompressed tail, so it differs from the
  whole-layer mode (bases per chunk, an exact tail).
"""

from __future__ import annotations

import logging
import sys
import weakref
from dataclasses import dataclass, field
from typing import Any

import torch

from kvcompress_b200.adapters.registry import install as registry_install
from kvcompress_b200.cache.compress import normalize_kv
from kvcompress_b200.cache.manager import CacheManager
from kvcompress_b200.compressor.base import CompressedPayload, KVCompressor
from kvcompress_b200.compressor.dispatch import build_compressor as _build_compressor

__all__ = ["ChunkedLayer", "HuggingFaceAdapter", "build_compressor", "generic_install", "is_compression_active"]

log = logging.getLogger(__name__)

# adapters installed per model (id(model)); entries go away with the adapter
INSTALLED_ADAPTERS: "weakref.WeakValueDictionary[int, HuggingFaceAdapter]" = weakref.WeakValueDictionary()


def is_compression_active(model: object) -> bool:
    """True when an enabled adapter is installed on ``model``."""
    adapter = INSTALLED_ADAPTERS.get(id(model))
    return adapter is not None and adapter.enabled


def build_compressor(method: str, **kwargs: Any) -> KVCompressor:
    """``kvcompress_b200.compressor.dispatch.build_compressor`` (re-exported)."""
    return _build_compressor(method, **kwargs)


@dataclass
class ChunkedLayer:
    """Compressed chunks of one layer in incremental mode.

    ``chunks[i]`` holds the K / V payloads of tokens ``[i * N, (i + 1) * N)``;
    ``done = len(chunks) * N`` tokens are compressed; ``decoded`` is the
    ``(B, n_kv, decoded_tokens, dh)`` reconstruction of the first chunks."""

    owner: int  # id() of the cache object the chunks belong to
    heads: tuple[int, int]  # (B, n_kv)
    chunks: list[tuple[CompressedPayload, CompressedPayload]] = field(default_factory=list)
    done: int = 0
    decoded: tuple[torch.Tensor, torch.Tensor] | None = None
    decoded_chunks: int = 0

    def bytes(self) -> tuple[int, int]:
        orig = sum(p.bytes_original for pair in self.chunks for p in pair)
        comp = sum(p.bytes_compressed for pair in self.chunks for p in pair)
        return orig, comp


class HuggingFaceAdapter:
    """Wire a compressor into an HF model's ``DynamicCache``
    (huggingface.py:90-432; arguments as there, plus ``incremental_block``).

    ``cache_implementation`` other than ``"dynamic"`` / ``"dynamic_full"`` is
    replaced by ``"dynamic"``; ``device`` defaults to the model's first
    parameter's device; extra keyword arguments go to the compressor.
    """

    def __init__(self, *, model: Any, method: str, compression_ratio: float, layer_groups: int = 1,
                 bits: tuple[int, ...] = (0, 2, 4, 8), cache_implementation: str = "dynamic", seed: int = 0,
                 device: torch.device | str | None = None, incremental_block: int | None = None,
                 **kwargs: Any) -> None:
        self.model = model
        self.method = method
        self.compression_ratio = float(compression_ratio)
        self.layer_groups = int(layer_groups)
        self.bits = tuple(bits)
        if cache_implementation not in ("dynamic", "dynamic_full"):
            log.debug("kvcompress: ignoring cache_implementation=%r; using 'dynamic'", cache_implementation)
            cache_implementation = "dynamic"
        self.cache_implementation = cache_implementation
        self.seed = int(seed)
        if incremental_block is not None and int(incremental_block) <= 0:
            raise ValueError(f"incremental_block must be positive, got {incremental_block}")
        self.incremental_block = None if incremental_block is None else int(incremental_block)
        if device is None:
            try:
                param = next(model.parameters(), None)
                device = param.device if param is not None else None
            except (StopIteration, AttributeError, TypeError):
                device = None
        self.device = torch.device(device) if isinstance(device, str) else device
        self.compressor = _build_compressor(method, compression_ratio=compression_ratio, bits=bits, seed=seed,
                                            layer_groups=layer_groups, **kwargs)
        self.manager: CacheManager | None = None
        self.chunked: dict[int, ChunkedLayer] = {}
        self.enabled = False
        self.enable_rolled_back = False
        self.original_cache_implementation: str | None = None
        self.cache_implementation_existed = False
        self.original_dynamic_cache_cls: type | None = None
        self.patched_cache_cls: type | None = None
        self.patched_modules: dict[str, type] = {}
        self.family_install: Any = None
        self.stats_ref: Any = None

    # ---- lifecycle -----------------------------------------------------

    def enable(self) -> None:
        """Install the patches; a second call, or another enabled adapter on
        the model, raises ``RuntimeError``.  A failure part-way is rolled back."""
        if self.enabled:
            raise RuntimeError("kvcompress: enable() called twice on the same adapter; "
                               "call handle.disable() first.")
        if is_compression_active(self.model):
            raise RuntimeError("kvcompress: a different adapter is already installed on this model; "
                               "call its handle.disable() first.")
        log.info("kvcompress: enabling %s on %s", self.method, type(self.model).__name__)
        try:
            self.enable_inner()
        except BaseException:
            self.rollback_partial_enable()
            raise

    def enable_inner(self) -> None:
        self.manager = CacheManager(compressor=self.compressor, device=self.device)
        self.chunked = {}
        gc = getattr(self.model, "generation_config", None)
        if gc is not None:
            self.cache_implementation_existed = hasattr(gc, "cache_implementation")
            self.original_cache_implementation = getattr(gc, "cache_implementation", None)
            gc.cache_implementation = self.cache_implementation
        from transformers.cache_utils import DynamicCache

        self.original_dynamic_cache_cls = DynamicCache
        self.install_dynamic_cache(DynamicCache)
        model_type = getattr(getattr(self.model, "config", None), "model_type", None)
        if model_type is not None:
            self.family_install = registry_install(model_type=model_type, model=self.model,
                                                   cache_manager=self.manager)
        self.enabled = True
        INSTALLED_ADAPTERS[id(self.model)] = self

    def _restore_generation_config(self) -> None:
        gc = getattr(self.model, "generation_config", None)
        if gc is None:
            return
        if self.cache_implementation_existed:
            gc.cache_implementation = self.original_cache_implementation
        elif hasattr(gc, "cache_implementation"):
            try:
                delattr(gc, "cache_implementation")
            except AttributeError:
                pass

    def rollback_partial_enable(self) -> None:
        """Undo what a failed ``enable`` changed (once)."""
        if self.enable_rolled_back:
            return
        self.enable_rolled_back = True
        if self.original_dynamic_cache_cls is not None:
            try:
                self.uninstall_dynamic_cache()
            except Exception:  # noqa: BLE001 - best effort
                log.exception("kvcompress: rollback failed during uninstall_dynamic_cache")
        try:
            self._restore_generation_config()
        except Exception:  # noqa: BLE001
            log.exception("kvcompress: rollback failed for cache_implementation")
        self.manager = None

    def disable(self) -> None:
        """Restore ``DynamicCache`` and the generation config (no-op when not enabled)."""
        if not self.enabled:
            return
        self._restore_generation_config()
        self.uninstall_dynamic_cache()
        self.enabled = False
        INSTALLED_ADAPTERS.pop(id(self.model), None)
        log.info("kvcompress: disabled compression on %s", type(self.model).__name__)

    # ---- store -----------------------------------------------------------

    def mirror(self, cache_obj: Any, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Bring the compressed store of ``layer_idx`` up to the layer's K / V."""
        if self.incremental_block is None:
            self.manager.store(layer_idx, k, v)
            return
        n = self.incremental_block
        b, h, t = int(k.shape[0]), int(k.shape[1]), int(k.shape[-2])
        st = self.chunked.get(layer_idx)
        if st is None or st.owner != id(cache_obj) or st.heads != (b, h) or t < st.done:
            st = self.chunked[layer_idx] = ChunkedLayer(owner=id(cache_obj), heads=(b, h))
        new = [(k[:, :, a:a + n, :], v[:, :, a:a + n, :]) for a in range(st.done, t - n + 1, n)]
        if not new:
            return
        pairs = [normalize_kv(kc.contiguous(), vc.contiguous()) for kc, vc in new]
        many = getattr(self.compressor, "compress_many", None)
        st.chunks += many(pairs) if many is not None else [self.compressor.compress(kc, vc) for kc, vc in pairs]
        st.done += n * len(new)

    def reconstruct(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """The layer's K / V as the store gives them back."""
        if self.incremental_block is None:
            # the store holds (B * n_kv, T, dh) cells; the layer keeps its 4-D shape
            kd, vd = self.manager.retrieve(layer_idx)
            return kd.reshape(k.shape), vd.reshape(v.shape)
        st = self.chunked[layer_idx]
        if st.decoded_chunks < len(st.chunks):
            fresh = st.chunks[st.decoded_chunks:]
            many = getattr(self.compressor, "decompress_many", None)
            outs = many(fresh) if many is not None else [self.compressor.decompress(kp, vp) for kp, vp in fresh]
            b, h = st.heads
            n = self.incremental_block
            parts = [(kd.reshape(b, h, n, kd.shape[-1]), vd.reshape(b, h, n, vd.shape[-1])) for kd, vd in outs]
            if st.decoded is not None:
                parts.insert(0, st.decoded)
            st.decoded = (torch.cat([p[0] for p in parts], dim=2), torch.cat([p[1] for p in parts], dim=2))
            st.decoded_chunks = len(st.chunks)
        if st.decoded is None:
            return k, v
        kd, vd = st.decoded
        if st.done == k.shape[-2]:
            return kd, vd
        return (torch.cat([kd, k[:, :, st.done:, :].to(kd.dtype)], dim=2),
                torch.cat([vd, v[:, :, st.done:, :].to(vd.dtype)], dim=2))

    def has_layer(self, layer_idx: int) -> bool:
        if self.manager is None:
            return False
        if self.incremental_block is None:
            return layer_idx in self.manager
        return layer_idx in self.chunked

    def memory(self) -> tuple[int, int]:
        """(original bytes, compressed bytes) of what the store holds; in
        incremental mode the uncompressed tails count at their size in both."""
        if self.incremental_block is None:
            return self.manager.memory_original(), self.manager.memory_used()
        orig = comp = 0
        for st in self.chunked.values():
            o, c = st.bytes()
            orig, comp = orig + o, comp + c
        return orig, comp

    # ---- DynamicCache patching ------------------------------------------

    def install_dynamic_cache(self, dynamic_cache_cls: type) -> None:
        """Replace ``DynamicCache`` in every loaded ``transformers`` module
        with a subclass whose ``update`` / ``__getitem__`` go through the store."""
        adapter = self

        class KvCompressCache(dynamic_cache_cls):  # type: ignore[misc, valid-type]
            """DynamicCache whose layers are mirrored into a compressed store."""

            def update(self, key_states, value_states, layer_idx, cache_kwargs=None):  # type: ignore[override]
                out = super().update(key_states, value_states, layer_idx, cache_kwargs)
                if adapter.manager is not None:
                    layer = self.layers[layer_idx]
                    adapter.mirror(self, layer_idx, layer.keys, layer.values)
                    if adapter.stats_ref is not None:
                        adapter.stats_ref.compress_calls += 1
                        adapter.stats_ref.bytes_original, adapter.stats_ref.bytes_compressed = adapter.memory()
                return out

            def __getitem__(self, layer_idx: int):  # type: ignore[override]
                layers = getattr(self, "layers", None)
                if adapter.has_layer(layer_idx) and layers is not None and layer_idx < len(layers):
                    layer = layers[layer_idx]
                    layer.keys, layer.values = adapter.reconstruct(layer_idx, layer.keys, layer.values)
                    if adapter.stats_ref is not None:
                        adapter.stats_ref.decompress_calls += 1
                parent = getattr(super(), "__getitem__", None)
                if parent is not None:
                    return parent(layer_idx)
                # caches without an indexer (transformers 5): the layer's K / V
                return layers[layer_idx].keys, layers[layer_idx].values

        self.patched_cache_cls = KvCompressCache
        import transformers.cache_utils as cu

        cu.DynamicCache = KvCompressCache
        import transformers.generation.utils as gu

        if hasattr(gu, "DynamicCache"):
            gu.DynamicCache = KvCompressCache
            self.patched_modules["transformers.generation.utils"] = KvCompressCache
        for name, mod in list(sys.modules.items()):
            if mod is None or not name.startswith("transformers"):
                continue
            if getattr(mod, "DynamicCache", None) is dynamic_cache_cls:
                mod.DynamicCache = KvCompressCache
                self.patched_modules[name] = KvCompressCache

    def uninstall_dynamic_cache(self) -> None:
        """Put the original ``DynamicCache`` back in every patched module."""
        import transformers.cache_utils as cu

        if self.original_dynamic_cache_cls is not None:
            cu.DynamicCache = self.original_dynamic_cache_cls
        for name in list(self.patched_modules):
            mod = sys.modules.get(name)
            if mod is not None:
                mod.DynamicCache = self.original_dynamic_cache_cls
        self.patched_modules.clear()


def generic_install(model: object, cache_manager: CacheManager) -> None:
    """Install for model types without a shim: nothing beyond the cache subclass."""
    return None
