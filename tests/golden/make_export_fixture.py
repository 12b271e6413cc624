"""Export / import fixture made by the reference itself (run on CPU).

    python tests/golden/make_export_fixture.py

Runs the reference's ``export_kv`` on a small seeded two-layer cache (bf16,
(B, n_kv, T, d) = (1, 2, 256, 64), FlashJoLT at ratio 4) and its
``import_kv`` on the file it wrote, and saves:

* ``ref_export.safetensors`` + ``ref_export.safetensors.meta.json``: the
  reference's file, to be read by ``kvcompress_b200.adapters.import_kv``;
* ``ref_import.npz``: the float32 K / V the reference's ``import_kv`` put into
  the cache, per layer.  That import takes the residual bit width from the
  cell metadata, where ``export_kv`` never writes it, so it decodes the
  residual as "int0" and keeps only the Tucker part;
* ``ref_decode.npz``: the same cells decoded in float32 with the residual,
  through the reference's own ``reconstruct_partial_tucker`` and
  ``decode_residual`` with the bit width of the payload (what
  ``import_kv``'s docstring describes, and what ``import_kv`` here returns);
* ``ref_export_layout.json``: tensor names, dtypes and shapes of the file,
  which ``export_kv`` here must reproduce for the same cache.

The reference is imported (never copied) from the source tree named by
``--reference PATH`` or ``$KVCOMPRESS_REFERENCE``.
"""

from __future__ import annotations

import json
import os
import struct
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from _reference import import_reference  # noqa: E402

REF = import_reference()

from kvcompress.adapters.vllm import export_kv, import_kv  # noqa: E402

from kvcompress_b200.synthetic import WORKLOADS, make_kv_layer  # noqa: E402


class _Layer:
    def __init__(self, k, v):
        self.keys, self.values = k, v


class _Cache:
    def __init__(self, layers):
        self.layers = layers

    def update(self, k, v, layer_idx):
        while len(self.layers) <= layer_idx:
            self.layers.append(_Layer(None, None))
        self.layers[layer_idx] = _Layer(k, v)


class _Model:
    def __init__(self, cache):
        self.past_key_values = cache


def fixture_cache():
    """The two-layer cache of the fixture (also built by the tests)."""
    w = WORKLOADS["llama3-8b-kv-b1-t8192-bf16"]
    layers = []
    for li in range(2):
        k, v = make_kv_layer(w, li, seed=5, tokens=256)
        layers.append((k[:, :2, :, :64].contiguous(), v[:, :2, :, :64].contiguous()))
    return layers


def main() -> None:
    torch.manual_seed(0)
    layers = fixture_cache()
    model = _Model(_Cache([_Layer(k, v) for k, v in layers]))
    path = os.path.join(HERE, "ref_export.safetensors")
    export_kv(model, path, method="flashjolt", compression_ratio=4.0, seed=0)
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    layout = {k: {"dtype": v["dtype"], "shape": v["shape"]} for k, v in sorted(header.items())}
    with open(os.path.join(HERE, "ref_export_layout.json"), "w") as f:
        json.dump(layout, f, indent=1, sort_keys=True)
    target = _Model(_Cache([_Layer(None, None) for _ in layers]))
    import_kv(target, path, target_memory=None, compression_ratio=4.0, method="flashjolt", seed=0)
    arrays = {}
    for li, layer in enumerate(target.past_key_values.layers):
        arrays[f"l{li}_key"] = layer.keys.float().numpy()
        arrays[f"l{li}_value"] = layer.values.float().numpy()
    np.savez_compressed(os.path.join(HERE, "ref_import.npz"), **arrays)
    np.savez_compressed(os.path.join(HERE, "ref_decode.npz"), **decode_with_residual(path))
    print("wrote", path, "and", len(arrays), "decoded tensors")


def decode_with_residual(path):
    """float32 decode of every cell of ``path`` by the reference's functions,
    the residual's bit width taken from the payload's ``residual_dtype``."""
    from safetensors.torch import load_file

    from kvcompress.compressor.residual import ResidualPayload, decode_residual
    from kvcompress.compressor.tucker import TuckerFactors, reconstruct_partial_tucker

    tensors = load_file(path)
    with open(path + ".meta.json") as f:
        cells = json.load(f)["cell_metadata"]
    out = {}
    for cell, cm in cells.items():
        layer, kind = cell.split("/")
        d = {k.split("/", 2)[2]: t for k, t in tensors.items() if k.startswith(cell + "/")}
        md = cm["metadata"]
        m, t, dh = cm["shape"]
        f = TuckerFactors(core=d["core"].float(), u_token=d["u_token"].float(), u_feature=d["u_feature"].float(),
                          token_sv=torch.empty(0), feature_sv=torch.empty(0), token_tail_mass=0.0,
                          feature_tail_mass=0.0)
        rec = reconstruct_partial_tucker(f, (m, t, dh))
        bits = int(d["residual_dtype"].item())
        if bits > 0:
            res = ResidualPayload(projection_seed=int(md["residual_seed"]),
                                  projection_distribution=md["residual_distribution"],
                                  projection_sparsity=float(md["residual_sparsity"]), quant_dtype=f"int{bits}",
                                  symmetric=bool(md["residual_symmetric"]), per_channel=bool(md["residual_per_channel"]),
                                  group_size=md["residual_group_size"], packed=d["residual_packed"],
                                  scale=d["residual_scale"], zero_point=d["residual_zero_point"],
                                  original_shape=tuple(int(x) for x in d["residual_original_shape"].tolist()),
                                  original_last=int(d["residual_original_last"].item()))
            rec = rec + decode_residual(res)
        out[f"l{layer}_{kind}"] = rec.float().numpy()
    return out


if __name__ == "__main__":
    main()
