"""Offload-block fixture made by the reference's own handler (run on CPU).

    python tests/golden/make_offload_fixture.py

Runs the reference's ``JoLTOffloadHandler.compress_block`` with a FlashJoLT
compressor (ratio 4) on a seeded bf16 block in vLLM's ``(num_layers, 2, T,
dh)`` layout, then its ``decompress_block`` on every layer, and saves:

* ``ref_offload.npz``: the block, every payload tensor of every
  ``(layer, kind)`` cell (``c{layer}_{kind}/{field}``), and the reference's
  decoded K / V per layer (``dec{layer}_{kind}``); bf16 arrays as raw uint16;
* ``ref_offload.json``: per cell the payload's method, shape, dtype,
  metadata and byte count.

The reference is imported (never copied) from the source tree named by
``--reference PATH`` or ``$KVCOMPRESS_REFERENCE``.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from _reference import import_reference  # noqa: E402

REF = import_reference()

from kvcompress import build_compressor  # noqa: E402
from kvcompress.adapters.vllm_kv_offload import JoLTOffloadHandler  # noqa: E402

from kvcompress_b200.synthetic import WORKLOADS, make_kv_layer  # noqa: E402

LAYERS, TOKENS = 2, 128


def raw(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def fixture_block() -> torch.Tensor:
    """``(LAYERS, 2, TOKENS, 128)`` bf16: head 0 of the Llama-3-8B workload's layers
    (also built by the tests)."""
    w = WORKLOADS["llama3-8b-kv-b1-t8192-bf16"]
    out = []
    for li in range(LAYERS):
        k, v = make_kv_layer(w, li, seed=7, tokens=TOKENS)
        out.append(torch.stack([k[0, 0], v[0, 0]]))
    return torch.stack(out).contiguous()


def main() -> None:
    block = fixture_block()
    comp = build_compressor("flashjolt", compression_ratio=4.0, seed=0)
    handler = JoLTOffloadHandler(compressor=comp)
    stored = handler.compress_block(block)
    arrays = {"block": raw(block)}
    cells = {}
    for (layer, kind), p in sorted(stored.items()):
        for field, t in p.data.items():
            arrays[f"c{layer}_{kind}/{field}"] = raw(t)
        cells[f"{layer}/{kind}"] = {
            "method": p.method, "shape": list(p.shape), "dtype": str(p.dtype).replace("torch.", ""),
            "metadata": p.metadata, "bytes_compressed": int(p.bytes_compressed),
            "dtypes": {field: str(t.dtype).replace("torch.", "") for field, t in p.data.items()},
        }
    for layer, (k, v) in enumerate(handler.decompress_block(list(range(LAYERS)))):
        arrays[f"dec{layer}_key"] = raw(k)
        arrays[f"dec{layer}_value"] = raw(v)
    np.savez_compressed(os.path.join(HERE, "ref_offload.npz"), **arrays)
    with open(os.path.join(HERE, "ref_offload.json"), "w") as f:
        json.dump(cells, f, indent=1, sort_keys=True)
    print("wrote", len(arrays), "arrays,", len(cells), "cells")


if __name__ == "__main__":
    main()
