"""Compressed-cache files (export_kv / import_kv) in the reference's format.

Fixtures from the reference's own export of a small cache
(tests/golden/make_export_fixture.py): its safetensors file and sidecar, the
float32 decode of its cells, and the file's tensor layout.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch
from safetensors.torch import load_file, save_file

from kvcompress_b200.adapters import export_kv, import_kv, read_payloads, write_payloads
from kvcompress_b200.synthetic import WORKLOADS, make_kv_layer

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
REF_FILE = os.path.join(GOLD, "ref_export.safetensors")


class _Layer:
    def __init__(self, k, v):
        self.keys, self.values = k, v


class _Cache:
    def __init__(self, layers):
        self.layers = layers

    def update(self, k, v, layer_idx):
        self.layers[layer_idx] = _Layer(k, v)


class _Model:
    def __init__(self, cache):
        self.past_key_values = cache


def _fixture_cache():
    """The reference fixture's cache (make_export_fixture.fixture_cache)."""
    w = WORKLOADS["llama3-8b-kv-b1-t8192-bf16"]
    layers = []
    for li in range(2):
        k, v = make_kv_layer(w, li, seed=5, tokens=256)
        layers.append((k[:, :2, :, :64].contiguous(), v[:, :2, :, :64].contiguous()))
    return layers


def test_file_round_trip_and_safetensors_compatibility(tmp_path):
    g = torch.Generator().manual_seed(1)
    tensors = {
        "0/key/core": torch.randn(4, 2, 3, generator=g).half(),
        "0/key/u_token": torch.randn(33, 2, generator=g).bfloat16(),
        "0/key/residual_packed": torch.randint(0, 256, (7, 5), generator=g, dtype=torch.int32).to(torch.uint8),
        "0/key/residual_scale": torch.rand(64, generator=g),
        "0/key/residual_zero_point": torch.zeros(64, dtype=torch.int32),
        "0/key/residual_dtype": torch.tensor(8, dtype=torch.int32),
        "1/value/tail": torch.randn(3, generator=g, dtype=torch.float64),
    }
    ours = str(tmp_path / "ours.safetensors")
    write_payloads(ours, tensors.items())
    for loaded in (load_file(ours), read_payloads(ours, "cpu")):
        assert set(loaded) == set(tensors)
        for k, t in tensors.items():
            assert loaded[k].dtype == t.dtype and loaded[k].shape == t.shape
            assert torch.equal(loaded[k], t)
    theirs = str(tmp_path / "theirs.safetensors")
    save_file(tensors, theirs)
    got = read_payloads(theirs, "cpu")
    for k, t in tensors.items():
        assert torch.equal(got[k], t)


def test_reads_the_reference_file_like_safetensors():
    ref = load_file(REF_FILE)
    got = read_payloads(REF_FILE, "cpu")
    assert set(got) == set(ref)
    for k in ref:
        assert got[k].dtype == ref[k].dtype and torch.equal(got[k], ref[k])


@pytest.mark.gpu
def test_import_of_the_reference_file_matches_the_reference_decode():
    """Import decodes the residual too: the reference's float32 decode of the
    file's cells (ref_decode.npz).  The reference's own import_kv keeps only
    the Tucker part (ref_import.npz; it reads the residual bit width from the
    cell metadata, where export_kv does not put it)."""
    want = np.load(os.path.join(GOLD, "ref_decode.npz"))
    model = _Model(_Cache([_Layer(None, None) for _ in range(2)]))
    import_kv(model, REF_FILE, target_memory=None, compression_ratio=4.0, method="flashjolt", seed=0)
    for li, layer in enumerate(model.past_key_values.layers):
        for kind, got in (("key", layer.keys), ("value", layer.values)):
            ref = want[f"l{li}_{kind}"]
            assert got.dtype == torch.float32 and tuple(got.shape) == ref.shape
            g = got.cpu().numpy()
            assert np.linalg.norm(g - ref) <= 1e-5 * np.linalg.norm(ref), (li, kind)


@pytest.mark.gpu
def test_export_matches_the_reference_layout_and_round_trips(tmp_path):
    layers = [(k.cuda(), v.cuda()) for k, v in _fixture_cache()]
    model = _Model(_Cache([_Layer(k, v) for k, v in layers]))
    path = str(tmp_path / "kv.safetensors")
    export_kv(model, path, method="flashjolt", compression_ratio=4.0, seed=0)
    with open(os.path.join(GOLD, "ref_export_layout.json")) as f:
        layout = json.load(f)
    ours = load_file(path)
    dt_name = {torch.float16: "F16", torch.float32: "F32", torch.int32: "I32", torch.uint8: "U8",
               torch.bfloat16: "BF16"}
    assert sorted(ours) == sorted(layout)
    for k, spec in layout.items():
        assert dt_name[ours[k].dtype] == spec["dtype"] and list(ours[k].shape) == spec["shape"], k
    with open(path + ".meta.json") as f:
        side = json.load(f)
    with open(REF_FILE + ".meta.json") as f:
        ref_side = json.load(f)
    assert set(side["cell_metadata"]) == set(ref_side["cell_metadata"])
    for cell, cm in ref_side["cell_metadata"].items():
        assert side["cell_metadata"][cell]["method"] == cm["method"]
        assert side["cell_metadata"][cell]["shape"] == cm["shape"]
        assert set(side["cell_metadata"][cell]["metadata"]) == set(cm["metadata"])
    # round trip: the end-to-end error of the imported cache is the
    # reference's on the same cache (its file decoded with the residual)
    ref = np.load(os.path.join(GOLD, "ref_decode.npz"))
    back = _Model(_Cache([_Layer(None, None) for _ in range(2)]))
    import_kv(back, path, target_memory=None, compression_ratio=4.0, method="flashjolt", seed=0)
    for li, ((k, v), layer) in enumerate(zip(layers, back.past_key_values.layers)):
        for kind, x, y in (("key", k, layer.keys), ("value", v, layer.values)):
            x3 = x.reshape(-1, x.shape[-2], x.shape[-1]).float()
            err = float((y - x3).norm() / x3.norm())
            err_ref = float(np.linalg.norm(ref[f"l{li}_{kind}"] - x3.cpu().numpy()) / x3.norm().item())
            assert abs(err - err_ref) <= 0.05 * err_ref, (li, kind, err, err_ref)
