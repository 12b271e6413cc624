"""Hugging Face adapter (enable_compression / HuggingFaceAdapter / registry).

CPU: the adapter lifecycle as the reference's unit tests exercise it
(tests/unit/adapter_test.py there), and the patched ``DynamicCache`` with the
fp32 identity compressor in both store modes.  GPU: FlashJoLT through the
patched cache; the whole-layer mode stores exactly ``compress`` of the
layer's current K / V after every update (the reference's behaviour), the
incremental mode compresses each chunk once and reads back the chunks'
decodes followed by the uncompressed tail.
"""

from __future__ import annotations

import pytest
import torch

from kvcompress_b200 import CompressionHandle, build_compressor, enable_compression
from kvcompress_b200.adapters import huggingface as hf_module
from kvcompress_b200.adapters.huggingface import HuggingFaceAdapter
from kvcompress_b200.adapters.registry import REGISTRY, install, known_model_types, register, resolve
from kvcompress_b200.api import parse_target_memory


class FakeModel:
    def __init__(self, model_type: str = "llama", has_cache_impl: bool = True) -> None:
        self.config = type("Config", (), {})()
        self.config.model_type = model_type
        self.generation_config = type("GenConfig", (), {})()
        if has_cache_impl:
            self.generation_config.cache_implementation = None


def _dynamic_cache():
    import transformers.cache_utils as cu

    return cu.DynamicCache


def test_registry():
    assert {"llama", "mistral", "qwen2"} <= set(known_model_types())
    assert resolve("llama") is not None and resolve("unknown-type") is None
    register("custom-test", resolve("llama"))
    try:
        assert resolve("custom-test") == resolve("llama")
    finally:
        REGISTRY.pop("custom-test", None)
    with pytest.raises(ValueError, match="already registered"):
        register("llama", "x")
    assert install(model=FakeModel("llama"), cache_manager=None, model_type="llama") is None
    assert install(model=FakeModel("nope"), cache_manager=None, model_type="nonexistent") is None


def test_enable_disable_lifecycle():
    model = FakeModel("llama")
    original = _dynamic_cache()
    handle = enable_compression(model, method="flashjolt", compression_ratio=2.0)
    try:
        assert isinstance(handle, CompressionHandle) and handle.model is model and handle.is_active
        assert _dynamic_cache() is not original and issubclass(_dynamic_cache(), original)
        import transformers.generation.utils as gu

        if hasattr(gu, "DynamicCache"):
            assert gu.DynamicCache is _dynamic_cache()
        with pytest.raises(RuntimeError, match="already"):
            enable_compression(model, method="jolt", compression_ratio=3.0)
        d = handle.stats_dict()
        assert {"compress_calls", "decompress_calls", "compression_ratio", "memory_saved_bytes"} <= set(d)
    finally:
        handle.disable()
    assert not handle.is_active and _dynamic_cache() is original
    handle.disable()  # idempotent


def test_enable_arguments():
    model = FakeModel("llama")
    with pytest.raises(ValueError, match="target_memory"):
        enable_compression(model, method="jolt")
    with pytest.raises(ValueError, match="target_memory"):
        enable_compression(model, method="jolt", target_memory="25%", compression_ratio=4.0)
    with pytest.raises(NotImplementedError, match="not supported"):
        enable_compression(model, method="not-a-method", compression_ratio=2.0)
    with pytest.raises(ValueError, match="incremental_block"):
        enable_compression(model, method="flashjolt", compression_ratio=2.0, incremental_block=0)
    assert parse_target_memory("25%") == 4.0 and parse_target_memory(0.25) == 4.0
    for bad in ("abc", 0, "150%"):
        with pytest.raises(ValueError):
            parse_target_memory(bad)
    h = enable_compression(model, method="flashjolt", target_memory="100%")
    try:
        assert h.adapter.compressor.name == "identity"
    finally:
        h.disable()


def test_generation_config_restored():
    model = FakeModel("llama", has_cache_impl=False)
    h = enable_compression(model, method="flashjolt", compression_ratio=2.0)
    assert model.generation_config.cache_implementation == "dynamic"
    h.disable()
    assert not hasattr(model.generation_config, "cache_implementation")

    class Model:
        config = type("C", (), {"model_type": "llama"})()
        generation_config = type("G", (), {"cache_implementation": "static"})()

    m = Model()
    h = enable_compression(m, method="flashjolt", compression_ratio=2.0)
    assert m.generation_config.cache_implementation == "dynamic"
    h.disable()
    assert m.generation_config.cache_implementation == "static"


def test_enable_rolls_back_on_failure(monkeypatch):
    original = _dynamic_cache()

    def boom(**_kwargs):
        raise RuntimeError("simulated family-shim install failure")

    monkeypatch.setattr(hf_module, "registry_install", boom)
    model = FakeModel("llama", has_cache_impl=False)
    adapter = HuggingFaceAdapter(model=model, method="flashjolt", compression_ratio=2.0)
    with pytest.raises(RuntimeError, match="simulated"):
        adapter.enable()
    assert not hasattr(model.generation_config, "cache_implementation")
    assert _dynamic_cache() is original and adapter.enabled is False


def _updates(cache, k, v, steps):
    """Prefill with ``k[..., :steps[0], :]`` then one update per further step size."""
    t = 0
    for s in steps:
        cache.update(k[:, :, t:t + s], v[:, :, t:t + s], 0)
        t += s
    return t


def test_patched_cache_whole_layer_mode_identity():
    model = FakeModel("llama")
    h = enable_compression(model, method="fp16", compression_ratio=2.0, factor_dtype=torch.float32)
    try:
        cache = _dynamic_cache()()
        k, v = torch.randn(1, 2, 12, 8), torch.randn(1, 2, 12, 8)
        t = _updates(cache, k, v, [9, 1, 1])
        assert h.stats.compress_calls == 3 and h.adapter.has_layer(0)
        kd, vd = cache[0]
        assert kd.shape == (1, 2, t, 8) and torch.equal(kd, k[:, :, :t]) and torch.equal(vd, v[:, :, :t])
        assert h.stats.decompress_calls == 1
    finally:
        h.disable()


def test_patched_cache_incremental_mode_identity():
    model = FakeModel("llama")
    h = enable_compression(model, method="fp16", compression_ratio=2.0, factor_dtype=torch.float32,
                           incremental_block=4)
    try:
        cache = _dynamic_cache()()
        k, v = torch.randn(1, 2, 20, 8), torch.randn(1, 2, 20, 8)
        _updates(cache, k, v, [10])
        st = h.adapter.chunked[0]
        assert st.done == 8 and len(st.chunks) == 2
        first = st.chunks[0]
        kd, vd = cache[0]
        assert torch.equal(kd, k[:, :, :10]) and torch.equal(vd, v[:, :, :10])
        _updates(cache, k[:, :, 10:], v[:, :, 10:], [1, 1, 1])  # 13 tokens: a third chunk
        assert st.done == 12 and len(st.chunks) == 3 and st.chunks[0] is first
        kd, vd = cache[0]
        assert st.decoded_chunks == 3 and torch.equal(kd, k[:, :, :13]) and torch.equal(vd, v[:, :, :13])
        orig, comp = h.adapter.memory()
        assert orig == 3 * 2 * 2 * 4 * 8 * 4 and comp == orig  # three chunks of K and V, fp32 stored
        # a new cache (new generation) starts the layer again
        other = _dynamic_cache()()
        other.update(k[:, :, :5], v[:, :, :5], 0)
        assert h.adapter.chunked[0] is not st and h.adapter.chunked[0].done == 4
    finally:
        h.disable()


# ---------------------------------------------------------------------------
# GPU: FlashJoLT through the patched cache


def _kv(tokens, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    base = torch.randn(1, 8, tokens, 16, generator=g, device="cuda") @ torch.randn(16, 128, generator=g,
                                                                                   device="cuda") / 4
    k = (base + 0.1 * torch.randn(1, 8, tokens, 128, generator=g, device="cuda")).bfloat16()
    v = (base.flip(-1) + 0.1 * torch.randn(1, 8, tokens, 128, generator=g, device="cuda")).bfloat16()
    return k, v


def _same_payload(a, b):
    assert sorted(a.data) == sorted(b.data)
    for f in a.data:
        assert torch.equal(a.data[f], b.data[f]), f
    assert a.metadata == b.metadata


@pytest.mark.gpu
def test_whole_layer_mode_stores_compress_of_the_current_layer():
    model = FakeModel("llama")
    h = enable_compression(model, method="flashjolt", compression_ratio=4.0)
    comp = build_compressor("flashjolt", compression_ratio=4.0)
    try:
        cache = _dynamic_cache()()
        k, v = _kv(514)
        _updates(cache, k, v, [512, 1, 1])
        kp, vp = comp.compress(k.reshape(8, 514, 128), v.reshape(8, 514, 128))
        _same_payload(h.adapter.manager.cache.payload(0, "key"), kp)
        _same_payload(h.adapter.manager.cache.payload(0, "value"), vp)
        kd, vd = cache[0]
        k_ref, v_ref = comp.decompress(kp, vp)
        assert kd.shape == k.shape and torch.equal(kd, k_ref.reshape(k.shape)) and torch.equal(vd, v_ref.reshape(v.shape))
        # bf16 cells with an 8-bit residual: at most 2x
        assert h.stats.compress_calls == 3 and 1.5 < h.stats.compression_ratio <= 2.0
    finally:
        h.disable()


@pytest.mark.gpu
def test_incremental_mode_compresses_each_chunk_once():
    model = FakeModel("llama")
    h = enable_compression(model, method="flashjolt", compression_ratio=4.0, incremental_block=128)
    comp = build_compressor("flashjolt", compression_ratio=4.0)
    try:
        cache = _dynamic_cache()()
        k, v = _kv(400, seed=1)
        _updates(cache, k, v, [300])
        st = h.adapter.chunked[0]
        assert st.done == 256 and len(st.chunks) == 2
        kept = list(st.chunks)
        _updates(cache, k[:, :, 300:], v[:, :, 300:], [1] * 90)  # 390 tokens: one more chunk
        assert st.done == 384 and len(st.chunks) == 3 and all(a is b for a, b in zip(st.chunks, kept))
        kd, vd = cache[0]
        parts_k, parts_v = [], []
        for i, (kp, vp) in enumerate(st.chunks):
            a = i * 128
            want_k, want_v = comp.compress(k[0, :, a:a + 128].contiguous(), v[0, :, a:a + 128].contiguous())
            _same_payload(kp, want_k)
            _same_payload(vp, want_v)
            dk, dv = comp.decompress(kp, vp)
            parts_k.append(dk)
            parts_v.append(dv)
        want_k = torch.cat(parts_k + [k[0, :, 384:390]], dim=1).unsqueeze(0)
        want_v = torch.cat(parts_v + [v[0, :, 384:390]], dim=1).unsqueeze(0)
        assert torch.equal(kd, want_k) and torch.equal(vd, want_v)
        err = float((kd.float() - k[:, :, :390].float()).norm() / k[:, :, :390].float().norm())
        assert 0.0 < err < 1.0
    finally:
        h.disable()
