"""Compressed-cache files: ``export_kv`` / ``import_kv`` with the reference's
format (kvcompress/adapters/vllm.py:87-395).

The file is a safetensors file with one tensor per payload field, named
``"{layer}/{kind}/{field}"``, plus a JSON sidecar ``path + ".meta.json"``
holding the cache metadata and, under ``"cell_metadata"``, each cell's
``method``, ``shape``, ``dtype`` and payload ``metadata``.  Files written here
load in the reference and the other way round.

The B200 side of it:

* export compresses every layer in one batched call (``store_layers``), then
  stages all payload tensors in one pinned host buffer with asynchronous
  device-to-host copies, one synchronisation, and writes header and data
  with two ``write`` calls;
* import reads the data section into pinned memory with one ``readinto``,
  copies it to the device in one transfer, and makes every payload tensor a
  view of that device buffer (tensors are ordered by element size, so every
  view is aligned); all JoLT cells of the file are then decoded in batched
  launches (``decompress_many``).

As in the reference, ``import_kv`` puts float32 ``(m, T, d)`` tensors into the
model's cache layers.
"""

from __future__ import annotations

import json
import struct
from typing import Any, Iterable

import numpy as np
import torch

from kvcompress_b200.cache.compress import CompressedKVCache
from kvcompress_b200.cache.metadata import CompressionMetadata
from kvcompress_b200.compressor.base import CompressedPayload, KVCompressor
from kvcompress_b200.compressor.cells import decompress_cells
from kvcompress_b200.compressor.dispatch import build_compressor
from kvcompress_b200.compressor.jolt import group_payloads

__all__ = ["export_kv", "import_kv", "is_vllm_available", "parse_target_memory", "read_payloads",
           "resolve_cache", "write_payloads"]

# safetensors dtype names (the format's own table)
_ST_NAME = {torch.float64: "F64", torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16",
            torch.int64: "I64", torch.int32: "I32", torch.int16: "I16", torch.int8: "I8",
            torch.uint8: "U8", torch.bool: "BOOL"}
if hasattr(torch, "float8_e4m3fn"):
    _ST_NAME[torch.float8_e4m3fn] = "F8_E4M3"
_ST_DTYPE = {v: k for k, v in _ST_NAME.items()}


def resolve_cache(model: Any) -> Any:
    """The model's live cache: ``past_key_values``, ``kv_cache`` or ``cache``
    (probed in that order, as the reference does)."""
    for attr in ("past_key_values", "kv_cache", "cache"):
        cache = getattr(model, attr, None)
        if cache is not None:
            return cache
    raise RuntimeError("could not locate a KV cache on the model; expected "
                       "model.past_key_values, model.kv_cache, or model.cache")


def parse_target_memory(value: str | float) -> float:
    """``"25%"`` / ``0.25`` -> compression ratio 4.0 (kvcompress/api.py:213-231)."""
    if isinstance(value, (int, float)):
        if not 0 < value <= 1:
            raise ValueError(f"target_memory fraction must be in (0, 1], got {value}")
        return 1.0 / value
    s = str(value).strip()
    if s.endswith("%"):
        pct = float(s[:-1])
        if not 0 < pct <= 100:
            raise ValueError(f"target_memory percent must be in (0, 100], got {pct}")
        return 100.0 / pct
    raise ValueError(f"target_memory must be a fraction or 'N%' string, got {value!r}")


def is_vllm_available() -> bool:
    try:
        import vllm  # noqa: F401
    except Exception:
        return False
    return True


# ---------------------------------------------------------------- file format

def write_payloads(path: str, tensors: Iterable[tuple[str, torch.Tensor]]) -> int:
    """Write named tensors (device or host) as one safetensors file.

    Tensors are laid out by decreasing element size, so every tensor starts
    at a multiple of its element size.  Device tensors are copied into one
    pinned host buffer (asynchronous copies, one synchronisation).  Returns
    the bytes of the data section."""
    items = [(name, t) for name, t in tensors]
    order = sorted(range(len(items)), key=lambda i: (-items[i][1].element_size(), i))
    header: dict[str, Any] = {}
    offsets = []
    off = 0
    for i in order:
        name, t = items[i]
        if t.dtype not in _ST_NAME:
            raise TypeError(f"write_payloads: dtype {t.dtype} of {name!r} has no safetensors name")
        n = t.numel() * t.element_size()
        header[name] = {"dtype": _ST_NAME[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + n]}
        offsets.append((i, off, n))
        off += n
    total = off
    staging = torch.empty(max(total, 1), dtype=torch.uint8, pin_memory=torch.cuda.is_available())
    any_device = False
    for i, o, n in offsets:
        t = items[i][1]
        if n == 0:
            continue
        dst = staging[o:o + n]
        src = t.contiguous().reshape(-1).view(torch.uint8) if t.dim() else t.reshape(1).view(torch.uint8)
        if src.is_cuda:
            any_device = True
            dst.copy_(src, non_blocking=True)
        else:
            dst.copy_(src)
    if any_device:
        torch.cuda.synchronize()
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        f.write(memoryview(staging.numpy())[:total])
    return total


def read_payloads(path: str, device: torch.device | str | None = None) -> dict[str, torch.Tensor]:
    """Read a safetensors file: the data section in one read, one copy to
    ``device`` (default: the current CUDA device when there is one), and
    every tensor a view of that buffer (a copy when a view would be
    misaligned)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
    device = torch.device(device)
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
        header.pop("__metadata__", None)
        total = max((int(v["data_offsets"][1]) for v in header.values()), default=0)
        host = torch.empty(max(total, 1), dtype=torch.uint8, pin_memory=device.type == "cuda")
        f.readinto(memoryview(host.numpy())[:total])
    buf = host.to(device, non_blocking=True) if device.type == "cuda" else host
    out: dict[str, torch.Tensor] = {}
    for name, spec in header.items():
        dt = _ST_DTYPE[spec["dtype"]]
        a, b = (int(x) for x in spec["data_offsets"])
        shape = [int(s) for s in spec["shape"]]
        es = torch.empty((), dtype=dt).element_size()
        raw = buf[a:b]
        if a % es == 0:
            t = raw.view(dt).view(shape) if b > a else torch.empty(shape, dtype=dt, device=buf.device)
        else:
            t = raw.clone().view(dt).view(shape)
        out[name] = t
    return out


# ---------------------------------------------------------------- export / import

def export_kv(model: Any, path: str, *, method: str = "flashjolt", compression_ratio: float = 3.0,
              bits: tuple[int, ...] = (0, 2, 4, 8), seed: int = 0,
              compressor: KVCompressor | None = None) -> CompressionMetadata:
    """Compress the model's live cache and write ``path`` + ``path.meta.json``
    (kvcompress/adapters/vllm.py:87-202)."""
    cache = resolve_cache(model)
    if compressor is None:
        compressor = build_compressor(method, compression_ratio=compression_ratio, bits=bits, seed=seed)
    tmp_cache = CompressedKVCache(compressor=compressor)
    n_layers = len(cache.layers)
    tmp_cache.store_layers(list(range(n_layers)), [cache.layers[i].keys for i in range(n_layers)],
                           [cache.layers[i].values for i in range(n_layers)])
    tensors: list[tuple[str, torch.Tensor]] = []
    cells: dict[str, dict[str, Any]] = {}
    for layer_idx in tmp_cache.layers():
        for kind in ("key", "value"):
            payload = tmp_cache.payload(layer_idx, kind)
            for name, t in payload.data.items():
                if isinstance(t, torch.Tensor):
                    tensors.append((f"{layer_idx}/{kind}/{name}", t))
            cells[f"{layer_idx}/{kind}"] = {
                "method": payload.method,
                "shape": list(payload.shape),
                "dtype": str(payload.dtype),
                "metadata": {k: (v.tolist() if hasattr(v, "tolist") else v) for k, v in payload.metadata.items()},
            }
    write_payloads(path, tensors)
    meta = tmp_cache.metadata()
    meta_dict = meta.to_dict()
    meta_dict["cell_metadata"] = cells
    with open(path + ".meta.json", "w") as f:
        json.dump(meta_dict, f, indent=2, default=str)
    return meta


def _dtype_of(name: str) -> torch.dtype:
    s = str(name).replace("torch.", "")
    dt = getattr(torch, s, None)
    if not isinstance(dt, torch.dtype):
        raise ValueError(f"import_kv: unknown dtype {name!r}")
    return dt


def import_kv(model: Any, path: str, *, target_memory: str | None = "100%", compression_ratio: float | None = None,
              method: str = "flashjolt", bits: tuple[int, ...] = (0, 2, 4, 8), seed: int = 0,
              device: torch.device | str | None = None) -> CompressionMetadata:
    """Load ``path`` (+ sidecar) and put the decoded K / V into the model's
    cache layers (kvcompress/adapters/vllm.py:205-382)."""
    cache = resolve_cache(model)
    tensors = read_payloads(path, device)
    with open(path + ".meta.json") as f:
        meta_dict = json.load(f)
    cell_meta = meta_dict.get("cell_metadata", {})
    ratio = compression_ratio
    if ratio is None and target_memory is not None:
        ratio = parse_target_memory(target_memory)
    if ratio == 1.0:
        method = "identity"
    compressor = build_compressor(method, compression_ratio=ratio or 3.0, bits=bits, seed=seed)
    tmp_cache = CompressedKVCache(compressor=compressor)

    by_cell: dict[tuple[int, str], dict[str, torch.Tensor]] = {}
    for key, t in tensors.items():
        parts = key.split("/", 2)
        if len(parts) != 3 or parts[1] not in ("key", "value"):
            continue
        try:
            layer_idx = int(parts[0])
        except ValueError:
            continue
        by_cell.setdefault((layer_idx, parts[1]), {})[parts[2]] = t

    decoded: dict[tuple[int, str], torch.Tensor] = {}
    jolt_cells, jolt_payloads = [], []
    for (layer_idx, kind), data in sorted(by_cell.items()):
        cm = cell_meta.get(f"{layer_idx}/{kind}", {})
        md = dict(cm.get("metadata", {}))
        if "core" in data and "u_token" in data and "u_feature" in data:
            m = int(data["core"].shape[0])
            t = int(data["u_token"].shape[0])
            d = int(data["u_feature"].shape[0])
            shape = tuple(cm.get("shape", (m, t, d)))
            dt = _dtype_of(cm.get("dtype", "float32"))
            fields = dict(data)
            for small in ("residual_original_shape", "residual_original_last", "residual_dtype"):
                if small in fields:
                    fields[small] = fields[small].cpu()
            if "bits" not in md and "residual_dtype" in md:
                md["bits"] = int(md["residual_dtype"])
            md.setdefault("bits", int(fields["residual_dtype"].item()) if "residual_dtype" in fields else 0)
            jolt_cells.append((layer_idx, kind))
            jolt_payloads.append(CompressedPayload(method="jolt", shape=shape, dtype=dt, metadata=md, data=fields))
        elif "value" in data:
            decoded[(layer_idx, kind)] = data["value"]
        elif "u" in data and "s" in data and "vh" in data:
            u, s, vh = data["u"].float(), data["s"].float(), data["vh"].float()
            m = int(md.get("m", u.shape[0]))
            decoded[(layer_idx, kind)] = ((u * s) @ vh).reshape(m, int(md.get("T", 1)), -1)
    # every JoLT cell of the file in batched launches, decoded straight to
    # float32 (the reference's reconstruction dtype)
    for members in group_payloads(jolt_payloads):
        rec = decompress_cells([jolt_payloads[i] for i in members], out_dtype=torch.float32)
        for i, x in zip(members, rec):
            decoded[jolt_cells[i]] = x
    layers_attr = getattr(cache, "layers", None)
    for layer_idx in sorted({layer for layer, _ in decoded}):
        k, v = decoded.get((layer_idx, "key")), decoded.get((layer_idx, "value"))
        if k is None or v is None:
            continue
        if layers_attr is not None and layer_idx < len(layers_attr):
            layers_attr[layer_idx].keys = k
            layers_attr[layer_idx].values = v
        else:
            cache.update(k, v, layer_idx)
    return tmp_cache.metadata()
