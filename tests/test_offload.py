"""vLLM offload handler, Shape B (kvcompress_b200.adapters.vllm_kv_offload).

CPU: the handler surface as the reference's own unit tests exercise it
(tests/unit/vllm_kv_offload_test.py there), with the fp32 identity
compressor.  GPU: a bf16 block through FlashJoLT against the reference's
handler run on the same block (tests/golden/make_offload_fixture.py): same
allocations, payload layout and byte counts, decode of the reference's own
payloads equal to its decode, and the batched block path equal bit for bit
to per-layer compress calls.
"""

from __future__ import annotations

import json
import os
import threading

import numpy as np
import pytest
import torch

from kvcompress_b200 import IdentityCompressor, JoLTCompressor, build_compressor
from kvcompress_b200.adapters import vllm_kv_offload as mod
from kvcompress_b200.adapters.vllm_kv_offload import (
    JoLTOffloadHandler,
    ThreadSafeEvictionPool,
    is_vllm_kv_offload_available,
)
from kvcompress_b200.compressor.base import CompressedPayload
from kvcompress_b200.synthetic import WORKLOADS, make_kv_layer

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _identity():
    return IdentityCompressor(factor_dtype=torch.float32)


def test_availability_probe_and_lazy_exports():
    assert isinstance(is_vllm_kv_offload_available(), bool)
    import kvcompress_b200.adapters as adapters

    assert adapters.JoLTOffloadHandler is JoLTOffloadHandler
    with pytest.raises(AttributeError):
        adapters.not_a_name  # noqa: B018


def test_handler_attributes_and_base_class():
    h = JoLTOffloadHandler(compressor=JoLTCompressor(compression_ratio=3.0), block_shape=(4, 2, 16, 8))
    assert h.name == "jolt-offload"
    for attr in ("compress_block", "decompress_block", "transfer_async", "get_finished", "wait"):
        assert hasattr(h, attr)
    assert isinstance(h.eviction_pool, ThreadSafeEvictionPool)
    if is_vllm_kv_offload_available():
        assert h.base_class is mod.import_vllm_base()
        assert callable(h.shutdown)  # forwarded from vLLM's base class
    with pytest.raises(AttributeError):
        h.no_such_method_anywhere()


def test_handler_without_vllm(monkeypatch):
    monkeypatch.setattr(mod, "import_vllm_base", lambda: None)
    h = JoLTOffloadHandler(compressor=_identity())
    assert h.base_class is None
    with pytest.raises(AttributeError, match="base class unbound"):
        h.some_vllm_only_method()


def test_handler_rejects_a_drifted_base(monkeypatch):
    monkeypatch.setattr(mod, "import_vllm_base", lambda: type("Drifted", (), {}))
    with pytest.raises(ImportError, match="API drift"):
        JoLTOffloadHandler(compressor=_identity())


def test_thread_safe_pool_round_trip():
    pool = ThreadSafeEvictionPool()
    n_threads, n_layers = 16, 32
    barrier = threading.Barrier(n_threads)

    def worker(tid):
        barrier.wait()
        for layer in range(n_layers):
            pool.put(layer, "key", (tid, layer))
            pool.put(layer, "value", (tid, layer + 1000))
            assert pool.get(layer, "key") is not None and pool.get(layer, "value") is not None

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(n_threads)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for layer in range(n_layers):
        assert set(pool.get_layer(layer)) == {"key", "value"}
    pool.drop_layer(3)
    assert pool.get_layer(3) == {} and pool.get(3, "key") is None
    pool.clear()
    assert pool.store == {}


def test_compress_block_separates_k_and_v():
    h = JoLTOffloadHandler(compressor=_identity())
    torch.manual_seed(0)
    k, v = torch.randn(2, 4, 8), torch.randn(2, 4, 8)
    stored = h.compress_block(torch.stack([k, v], dim=1))
    assert len(stored) == 4
    for layer in range(2):
        assert not torch.equal(stored[(layer, "key")].data["value"], stored[(layer, "value")].data["value"])
        assert h.eviction_pool.get(layer, "key") is stored[(layer, "key")]
        kd, vd = h.decompress_block(layer)
        assert torch.equal(kd, k[layer]) and torch.equal(vd, v[layer])


def test_compress_block_tuple_list_and_dict_handles():
    h = JoLTOffloadHandler(compressor=_identity())
    torch.manual_seed(0)
    k, v = torch.randn(3, 4, 8), torch.randn(3, 4, 8)
    stored = h.compress_block((k, v))
    assert sorted(stored) == [(i, kind) for i in range(3) for kind in ("key", "value")]
    out = h.decompress_block([0, 2])
    assert len(out) == 2
    assert torch.equal(out[0][0], k[0]) and torch.equal(out[1][1], v[2])
    kd, vd = h.decompress_block({(1, "key"): stored[(1, "key")], (1, "value"): stored[(1, "value")]})
    assert kd.shape == (1, 4, 8) and torch.equal(kd[0], k[1]) and torch.equal(vd[0], v[1])
    with pytest.raises(ValueError, match="empty stored dict"):
        h.decompress_block({})
    assert h.decompress_block([7]) == []  # missing layers are skipped
    with pytest.raises(IndexError):
        h.decompress_block(7)


def test_compress_block_rejects_unknown_layouts():
    h = JoLTOffloadHandler(compressor=_identity())
    for bad in (torch.randn(2, 4, 8), [torch.randn(1, 4, 8)] * 2):
        with pytest.raises(ValueError, match="unsupported block type"):
            h.compress_block(bad)


def test_jolt_block_needs_cuda_tensors():
    """No CPU path: a CPU block fails loudly in the compressor."""
    h = JoLTOffloadHandler(compressor=build_compressor("flashjolt", compression_ratio=4.0))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        h.compress_block(torch.randn(2, 2, 64, 64).bfloat16())


def test_transfer_jobs_success_failure_and_wait(monkeypatch):
    h = JoLTOffloadHandler(compressor=_identity())

    class Spec:
        def __init__(self, blocks):
            self.blocks = blocks

    assert h.transfer_async(7, (Spec([0, 1]), Spec([2, 3]))) is True
    assert h.eviction_pool.get(-1, "key") == ("transfer", [0, 1], [2, 3])
    assert h.get_finished() == [(7, True)]
    assert h.get_finished() == []

    def boom(self, src, dst):
        raise RuntimeError("simulated failure")

    monkeypatch.setattr(JoLTOffloadHandler, "run_transfer", boom)
    assert h.transfer_async(99, (None, None)) is False
    assert h.get_finished() == [(99, False)]
    h.finished_jobs += [(1, True), (2, True)]
    h.wait({1, 2})  # returns at once
    clock = {"t": 0.0}

    def fast_clock():
        clock["t"] += 1000.0
        return clock["t"]

    monkeypatch.setattr(mod.time, "monotonic", fast_clock)
    monkeypatch.setattr(mod.time, "sleep", lambda s: None)
    h.wait({999})  # times out instead of looping forever


# ---------------------------------------------------------------------------
# GPU: FlashJoLT blocks against the reference's handler


def _fixture():
    arrays = np.load(os.path.join(GOLD, "ref_offload.npz"))
    with open(os.path.join(GOLD, "ref_offload.json")) as f:
        cells = json.load(f)
    return arrays, cells


def _tensor(a: np.ndarray, dtype: str) -> torch.Tensor:
    dt = getattr(torch, dtype)
    if dt == torch.bfloat16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.copy()).to(dt)


def _block(arrays) -> torch.Tensor:
    return _tensor(arrays["block"], "bfloat16")


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.mark.gpu
def test_block_matches_the_reference_handler():
    arrays, cells = _fixture()
    block = _block(arrays).cuda()
    h = JoLTOffloadHandler(compressor=build_compressor("flashjolt", compression_ratio=4.0, seed=0))
    stored = h.compress_block(block)
    assert sorted(f"{layer}/{kind}" for layer, kind in stored) == sorted(cells)
    for (layer, kind), p in stored.items():
        ref = cells[f"{layer}/{kind}"]
        assert p.method == ref["method"] and list(p.shape) == ref["shape"]
        assert p.bytes_compressed == ref["bytes_compressed"]
        assert {f: str(t.dtype).replace("torch.", "") for f, t in p.data.items()} == ref["dtypes"]
        for key in ("r_token", "r_feature", "bits", "core_dtype", "residual_seed", "residual_symmetric",
                    "residual_per_channel", "residual_group_size"):
            assert p.metadata[key] == ref["metadata"][key], key
    # end-to-end error of every layer within 2% of the reference's on the same block
    for layer, (kd, vd) in enumerate(h.decompress_block(list(range(block.shape[0])))):
        for kind, got, idx in (("key", kd, 0), ("value", vd, 1)):
            x = block[layer, idx]
            ref = _tensor(arrays[f"dec{layer}_{kind}"], "bfloat16").cuda()
            assert got.shape == x.shape and got.dtype == torch.bfloat16
            err, err_ref = _rel(got, x), _rel(ref, x)
            assert abs(err - err_ref) <= 0.02 * err_ref, (layer, kind, err, err_ref)


@pytest.mark.gpu
def test_decode_of_the_reference_payloads_matches_its_decode():
    arrays, cells = _fixture()
    h = JoLTOffloadHandler(compressor=build_compressor("flashjolt", compression_ratio=4.0, seed=0))
    layers = sorted({int(c.split("/")[0]) for c in cells})
    for cell, ref in cells.items():
        layer, kind = cell.split("/")
        data = {f: _tensor(arrays[f"c{layer}_{kind}/{f}"], dt).cuda() for f, dt in ref["dtypes"].items()}
        h.eviction_pool.put(int(layer), kind, CompressedPayload(
            method=ref["method"], shape=tuple(ref["shape"]), dtype=getattr(torch, ref["dtype"]),
            metadata=dict(ref["metadata"]), data=data))
    for layer, (kd, vd) in zip(layers, h.decompress_layers(layers)):
        for kind, got in (("key", kd), ("value", vd)):
            want = _tensor(arrays[f"dec{layer}_{kind}"], "bfloat16").cuda()
            assert got.shape == want.shape and got.dtype == want.dtype
            assert _rel(got, want) < 1e-2, (layer, kind)


@pytest.mark.gpu
def test_batched_block_equals_per_layer_compress():
    w = WORKLOADS["llama3-8b-kv-b1-t8192-bf16"]
    layers = []
    for li in range(5):
        k, v = make_kv_layer(w, li, seed=3, tokens=512)
        layers.append(torch.stack([k[0, 1], v[0, 1]]))
    block = torch.stack(layers).cuda()  # (5, 2, 512, 128)
    comp = build_compressor("flashjolt", compression_ratio=4.0, seed=0)
    h = JoLTOffloadHandler(compressor=comp)
    stored = h.compress_block(block)
    for layer in range(block.shape[0]):
        kp, vp = comp.compress(block[layer, 0].unsqueeze(0), block[layer, 1].unsqueeze(0))
        for kind, want in (("key", kp), ("value", vp)):
            got = stored[(layer, kind)]
            assert sorted(got.data) == sorted(want.data)
            for f in want.data:
                assert torch.equal(got.data[f], want.data[f]), (layer, kind, f)
            assert got.metadata == want.metadata
    outs = h.decompress_block(list(range(block.shape[0])))
    for layer, (kd, vd) in enumerate(outs):
        k_ref, v_ref = comp.decompress(stored[(layer, "key")], stored[(layer, "value")])
        assert torch.equal(kd, k_ref[0]) and torch.equal(vd, v_ref[0])
