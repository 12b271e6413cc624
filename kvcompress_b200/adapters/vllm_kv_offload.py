"""vLLM KV-offload handler, Shape B (API of kvcompress/adapters/vllm_kv_offload.py).

vLLM's offloading worker hands a handler ``transfer_async(job_id, (src, dst))``
jobs and polls ``get_finished`` / ``wait``.  The data path is
``compress_block``: a block of every layer's K and V, ``(num_layers, 2, T,
dh)`` or a ``(K_block, V_block)`` pair of ``(num_layers, T, dh)`` tensors,
becomes one ``(1, T, dh)`` cell per layer and kind, stored in a thread-safe
eviction pool keyed ``(layer, "key" | "value")``.

The reference compresses such a block one layer at a time
(``store_block``, vllm_kv_offload.py:364-382: a ``CacheManager.store`` per
layer, each a separate compress call).  Here ``store_block`` gives every layer
to ``CacheManager.store_layers`` at once, so the cells of a block go through
the kernels as one batch (one ``kvc_compress`` call for up to 64 same-shape
cells), and ``decompress_layers`` decodes the requested layers with one
batched decode.  Payloads, allocations and the pool's contents are the ones
the per-layer path gives.

The vLLM base class (``vllm.v1.kv_offload.worker.worker.OffloadingHandler``)
is imported lazily and only consulted for attributes the handler does not
define; the data path works without vLLM.
"""

from __future__ import annotations

import logging
import threading
import time
from typing import Any

from kvcompress_b200.compressor.base import KVCompressor

__all__ = [
    "JoLTOffloadHandler",
    "ThreadSafeEvictionPool",
    "import_vllm_base",
    "is_vllm_kv_offload_available",
]

log = logging.getLogger(__name__)

_KINDS = ("key", "value")


def import_vllm_base() -> type | None:
    """vLLM's ``OffloadingHandler`` ABC, or None without vLLM (vllm_kv_offload.py:84-100)."""
    try:
        from vllm.v1.kv_offload.worker.worker import OffloadingHandler
    except ImportError:
        return None
    return OffloadingHandler


def is_vllm_kv_offload_available() -> bool:
    """True when vLLM's v1 KV-offload handler API imports (vllm_kv_offload.py:72-81)."""
    return import_vllm_base() is not None


class ThreadSafeEvictionPool:
    """Payload store keyed ``(layer, kind)`` behind an ``RLock``
    (vllm_kv_offload.py:103-141).  ``lock`` and ``store`` are public."""

    def __init__(self) -> None:
        self.lock = threading.RLock()
        self.store: dict[tuple[int, str], Any] = {}

    def put(self, layer: int, kind: str, payload: Any) -> None:
        with self.lock:
            self.store[(layer, kind)] = payload

    def put_many(self, items: dict[tuple[int, str], Any]) -> None:
        """Several ``(layer, kind) -> payload`` entries under one lock hold."""
        with self.lock:
            self.store.update(items)

    def get(self, layer: int, kind: str) -> Any | None:
        with self.lock:
            return self.store.get((layer, kind))

    def get_layer(self, layer: int) -> dict[str, Any]:
        """Snapshot of one layer's payloads (the kinds present)."""
        with self.lock:
            return {kind: self.store[(layer, kind)] for kind in _KINDS if (layer, kind) in self.store}

    def drop_layer(self, layer: int) -> None:
        with self.lock:
            for kind in _KINDS:
                self.store.pop((layer, kind), None)

    def clear(self) -> None:
        with self.lock:
            self.store.clear()


class JoLTOffloadHandler:
    """Offload handler that compresses vLLM KV blocks (vllm_kv_offload.py:144-419).

    ``compressor``: any ``KVCompressor``; ``eviction_pool``: payload storage
    (a ``ThreadSafeEvictionPool`` by default).  Extra keyword arguments are
    accepted and ignored, as by the reference.

    ``transfer_async`` records a job as finished (or failed, when
    ``run_transfer`` raises) before it returns; ``get_finished`` drains the
    finished ``(job_id, success)`` entries and ``wait`` polls for a set of job
    ids for at most 60 s.
    """

    name = "jolt-offload"

    def __init__(self, compressor: KVCompressor, eviction_pool: ThreadSafeEvictionPool | None = None,
                 **kwargs: Any) -> None:
        base_cls = import_vllm_base()
        if base_cls is not None and (not isinstance(base_cls, type) or not hasattr(base_cls, "transfer_async")):
            raise ImportError(f"JoLTOffloadHandler: vLLM OffloadingHandler at {base_cls!r} "
                              "does not expose transfer_async; vLLM API drift.")
        self.compressor = compressor
        self.eviction_pool: ThreadSafeEvictionPool = (eviction_pool if eviction_pool is not None
                                                      else ThreadSafeEvictionPool())
        self.lock = threading.Lock()
        self.next_job_id = 0
        self.finished_jobs: list[Any] = []
        self.base_class: type | None = base_cls

    # ---- OffloadingHandler surface -------------------------------------

    def transfer_async(self, job_id: int, transfer_spec: Any) -> bool:
        """Run the transfer ``transfer_spec = (src, dst)`` and queue its result."""
        src_spec, dst_spec = transfer_spec
        try:
            self.run_transfer(src_spec, dst_spec)
        except Exception as e:  # noqa: BLE001 - a failed job is reported, not raised
            log.warning("JoLTOffloadHandler.transfer_async: transfer %d failed: %r", job_id, e)
            with self.lock:
                self.finished_jobs.append(self.make_result(job_id, success=False))
            return False
        with self.lock:
            self.finished_jobs.append(self.make_result(job_id, success=True))
        return True

    def get_finished(self) -> list[Any]:
        """The jobs finished since the last call (the list is drained)."""
        with self.lock:
            out, self.finished_jobs = self.finished_jobs, []
            return out

    def wait(self, job_ids: set[int]) -> None:
        """Poll until every id of ``job_ids`` is among the finished jobs, or 60 s passed."""
        deadline = time.monotonic() + 60.0
        while True:
            with self.lock:
                done = {entry[0] for entry in self.finished_jobs}
            if job_ids.issubset(done):
                return
            if time.monotonic() > deadline:
                log.warning("JoLTOffloadHandler.wait: timeout for %s", job_ids)
                return
            time.sleep(0.001)

    # ---- block data path ------------------------------------------------

    def compress_block(self, block: Any) -> dict[tuple[int, str], Any]:
        """Compress a block and put its payloads into the pool.

        ``block``: a ``(num_layers, 2, T, dh)`` tensor (vLLM's layout, K at
        index 0 of axis 1) or a ``(K_block, V_block)`` tuple of
        ``(num_layers, T, dh)`` tensors.  Returns ``(layer, kind) -> payload``
        for every layer.  Anything else raises ``ValueError``.
        """
        from kvcompress_b200.cache.manager import CacheManager

        mgr = CacheManager(compressor=self.compressor)
        if isinstance(block, tuple) and len(block) == 2:
            k_block, v_block = block
            self.store_block(mgr, k_block, v_block)
            return {(layer, kind): mgr.cache.payload(layer, kind) for layer in mgr.cache.layers() for kind in _KINDS}
        if hasattr(block, "dim") and block.dim() == 4:
            num_layers = block.shape[0]
            self.store_block(mgr, block[:, 0], block[:, 1])
            stored = {(layer, kind): mgr.cache.payload(layer, kind) for layer in range(num_layers) for kind in _KINDS}
            self.eviction_pool.put_many(stored)
            return stored
        raise ValueError(f"JoLTOffloadHandler.compress_block: unsupported block type "
                         f"{type(block).__name__} with shape {getattr(block, 'shape', None)}")

    def decompress_block(self, handle: int | list[Any] | dict) -> Any:
        """``(K, V)`` of one layer (an index, or a ``(layer, kind) -> payload``
        mapping), or a list of them for a list of layer indices."""
        if isinstance(handle, dict):
            return self.decompress_from_dict(handle)
        if isinstance(handle, list):
            return self.decompress_layers(handle)
        return self.decompress_layers([handle])[0]

    def __getattr__(self, name: str) -> Any:
        # anything the handler does not define comes from vLLM's base class
        if name.startswith("__") and name.endswith("__"):
            raise AttributeError(name)
        base = self.__dict__.get("base_class")
        if base is None:
            raise AttributeError(f"JoLTOffloadHandler.{name}: base class unbound")
        attr = getattr(base, name, None)
        if attr is None:
            raise AttributeError(f"JoLTOffloadHandler.{name}: not present on vLLM base")
        return attr

    # ---- internals -----------------------------------------------------

    def make_result(self, job_id: int, success: bool) -> Any:
        """A ``TransferResult``-shaped ``(job_id, success)`` pair."""
        return (job_id, success)

    def run_transfer(self, src_spec: Any, dst_spec: Any) -> None:
        """Record the transfer under the pool key ``(-1, "key")``; the wire
        format between vLLM's page buffers stays opaque, as in the reference
        (vllm_kv_offload.py:348-362)."""
        self.eviction_pool.put(-1, "key", ("transfer", getattr(src_spec, "blocks", None),
                                          getattr(dst_spec, "blocks", None)))

    def store_block(self, mgr: Any, k_block: Any, v_block: Any) -> None:
        """Compress ``(num_layers, T, dh)`` K and V blocks into ``mgr`` and the pool.

        Each layer becomes a ``(1, T, dh)`` cell; all layers are compressed in
        one batched call (``CacheManager.store_layers``) where the manager
        has it, else one ``store`` per layer."""
        num_layers = k_block.shape[0]
        layers = list(range(num_layers))
        keys = [k_block[i].unsqueeze(0) for i in layers]
        values = [v_block[i].unsqueeze(0) for i in layers]
        many = getattr(mgr, "store_layers", None)
        if many is not None:
            many(layers, keys, values)
        else:
            for i in layers:
                mgr.store(i, keys[i], values[i])
        self.eviction_pool.put_many({(i, kind): mgr.cache.payload(i, kind) for i in layers for kind in _KINDS})

    def decompress_from_dict(self, stored: dict[tuple[int, str], Any]) -> tuple[Any, Any]:
        """``(K, V)`` of the first layer named in a ``(layer, kind) -> payload`` mapping."""
        if not stored:
            raise ValueError("JoLTOffloadHandler: empty stored dict")
        layer = next(iter(stored))[0]
        return self.compressor.decompress(stored[(layer, "key")], stored[(layer, "value")])

    def decompress_layers(self, layer_indices: list[int]) -> list[tuple[Any, Any]]:
        """``(K, V)`` per pooled layer of ``layer_indices`` (one batched decode);
        a layer missing from the pool is logged and skipped.  A single-head
        ``(1, T, dh)`` result is returned as ``(T, dh)``."""
        pairs = []
        for layer in layer_indices:
            kp, vp = self.eviction_pool.get(layer, "key"), self.eviction_pool.get(layer, "value")
            if kp is None or vp is None:
                log.warning("JoLTOffloadHandler: missing payload for layer %d (key=%s, value=%s)",
                            layer, kp is not None, vp is not None)
                continue
            pairs.append((kp, vp))
        if not pairs:
            return []
        many = getattr(self.compressor, "decompress_many", None)
        outs = many(pairs) if many is not None else [self.compressor.decompress(kp, vp) for kp, vp in pairs]
        squeeze = lambda x: x.squeeze(0) if x.dim() == 3 and x.shape[0] == 1 else x  # noqa: E731
        return [(squeeze(k), squeeze(v)) for k, v in outs]
