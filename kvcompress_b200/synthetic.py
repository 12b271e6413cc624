"""Seeded synthetic KV caches with the shapes of real models.

No public dataset is involved: each (layer, K|V) tensor of shape
``(batch, n_kv, T, head_dim)`` is a latent low-rank signal plus noise.

* Every (batch, head) slice is ``A @ B + sigma * N``, with ``A ~ N(0, 1)``
  of shape ``(T, r)``, ``B ~ N(0, 1/r)`` of shape ``(r, head_dim)`` and
  ``N ~ N(0, 1)``.  The generator for tensor (layer, kind) is seeded with
  ``seed * 1_000_003 + 2 * layer + kind`` (kind 0 = K, 1 = V).
* K only: ``n_outliers`` channels, drawn once per model from ``seed``, are
  scaled by 8; then rotary position embedding (rotate-half convention,
  ``theta_i = base ** (-2 i / head_dim)``, positions ``0..T-1``).
* The result is cast to the requested dtype.

``WORKLOADS`` names the model-shaped caches the benchmark and the tests use.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

__all__ = ["KVWorkload", "WORKLOADS", "make_kv_layer", "outlier_channels", "layer_sigma"]


@dataclass(frozen=True)
class KVWorkload:
    """A model-shaped KV cache and the compressor settings applied to it."""

    name: str
    layers: int
    n_kv: int
    head_dim: int
    batch: int
    tokens: int
    dtype: torch.dtype
    latent_rank: int
    sigma: float
    n_outliers: int
    rope_base: float
    method: str
    compression_ratio: float
    bits: tuple = (0, 2, 4, 8)
    sigma_range: tuple | None = None  # per-layer sigma ~ U[lo, hi] when set
    layer_groups: int = 1

    @property
    def cell_shape(self) -> tuple[int, int, int]:
        """``(m, T, d)`` with ``m = batch * n_kv``: one compressor cell."""
        return (self.batch * self.n_kv, self.tokens, self.head_dim)

    @property
    def tensor_bytes(self) -> int:
        """Bytes of one layer's K (or V)."""
        m, t, d = self.cell_shape
        return m * t * d * torch.tensor([], dtype=self.dtype).element_size()


WORKLOADS = {
    # TinyLlama-1.1B-shaped, fp32, FlashJoLT 4x.
    "tinyllama-1.1b-kv-t2048-fp32": KVWorkload(
        "tinyllama-1.1b-kv-t2048-fp32", 22, 4, 64, 1, 2048, torch.float32,
        16, 0.1, 4, 10000.0, "flashjolt", 4.0),
    # Llama-3-8B-shaped, one sequence of 8192 tokens, FlashJoLT at 25 % memory.
    "llama3-8b-kv-b1-t8192-bf16": KVWorkload(
        "llama3-8b-kv-b1-t8192-bf16", 32, 8, 128, 1, 8192, torch.bfloat16,
        32, 0.1, 8, 500000.0, "flashjolt", 4.0),
    # Llama-3-8B-shaped, batch 8 x 32k, FlashJoLT 4x: the cache of the
    # previous entry compressed the FlashJoLT way (randomised SVDs), the
    # target workload for 1 / 2 / 4 / 8 GPUs.
    "llama3-8b-kv-b8-t32768-bf16": KVWorkload(
        "llama3-8b-kv-b8-t32768-bf16", 32, 8, 128, 8, 32768, torch.bfloat16,
        16, 0.1, 4, 10000.0, "flashjolt", 4.0),
    # One layer of the batch 8 cache at 4k tokens, FlashJoLT 4x with residual
    # bits (0, 2, 4): the allocator picks (512, 16, 4), so the token sketch
    # meets the q cap (513 wide).
    "llama3-8b-kv-b8-t4096-bf16-qcap": KVWorkload(
        "llama3-8b-kv-b8-t4096-bf16-qcap", 1, 8, 128, 8, 4096, torch.bfloat16,
        16, 0.1, 4, 10000.0, "flashjolt", 4.0, bits=(0, 2, 4)),
    # Llama-3-8B-shaped, batch 8 x 32k, exact JoLT 3x.
    "llama3-8b-kv-b8-t32768-bf16-jolt": KVWorkload(
        "llama3-8b-kv-b8-t32768-bf16-jolt", 32, 8, 128, 8, 32768, torch.bfloat16,
        16, 0.1, 4, 10000.0, "jolt", 3.0),
    # Qwen2-7B-shaped decode stream, batch 4 x 128k, FlashJoLT 4x.
    "qwen2-7b-kv-b4-t131072-bf16": KVWorkload(
        "qwen2-7b-kv-b4-t131072-bf16", 28, 4, 128, 4, 131072, torch.bfloat16,
        48, 0.1, 4, 10000.0, "flashjolt", 4.0),
    # Llama-3-70B-shaped, batch 8 x 32k, FlashJoLT at 20 % memory.
    "llama3-70b-kv-b8-t32768-bf16": KVWorkload(
        "llama3-70b-kv-b8-t32768-bf16", 80, 8, 128, 8, 32768, torch.bfloat16,
        64, 0.1, 4, 10000.0, "flashjolt", 5.0, sigma_range=(0.05, 0.3), layer_groups=4),
}


def outlier_channels(head_dim: int, n_outliers: int, seed: int = 0) -> torch.Tensor:
    """The model-wide K outlier channels: ``randperm(head_dim)[:n]`` from ``seed``."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    return torch.randperm(head_dim, generator=g)[:n_outliers]


def layer_sigma(w: KVWorkload, layer: int, seed: int = 0) -> float:
    """Noise level of ``layer``: fixed, or drawn from ``U[lo, hi]`` per layer."""
    if w.sigma_range is None:
        return float(w.sigma)
    g = torch.Generator(device="cpu").manual_seed(int(seed) * 7919 + 17)
    u = torch.rand(w.layers, generator=g, dtype=torch.float64)[layer].item()
    lo, hi = w.sigma_range
    return float(lo + (hi - lo) * u)


def _rope(x: torch.Tensor, base: float) -> torch.Tensor:
    """Rotate-half RoPE over the last axis at positions ``0..T-1``."""
    t, d = x.shape[-2], x.shape[-1]
    half = d // 2
    inv = base ** (-2.0 * torch.arange(half, dtype=torch.float64, device=x.device) / d)
    ang = torch.arange(t, dtype=torch.float64, device=x.device)[:, None] * inv[None, :]
    cos = torch.cos(ang).to(x.dtype)
    sin = torch.sin(ang).to(x.dtype)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def make_kv_layer(
    w: KVWorkload,
    layer: int,
    *,
    seed: int = 0,
    device: str | torch.device = "cpu",
    tokens: int | None = None,
    batch: int | None = None,
    precise: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """K and V of one layer, shape ``(batch, n_kv, T, head_dim)`` in ``w.dtype``.

    ``tokens`` / ``batch`` override the workload's sizes (small parity cases
    keep the value distribution of the full workload).  ``precise`` does the
    arithmetic in float64 before the final cast, so the same bytes come out on
    any CPU whatever its BLAS (the parity fixtures of large caches regenerate
    their inputs this way instead of storing them).
    """
    t = int(tokens or w.tokens)
    b = int(batch or w.batch)
    d, r = w.head_dim, w.latent_rank
    sigma = layer_sigma(w, layer, seed)
    fdt = torch.float64 if precise else torch.float32
    out = []
    for kind in (0, 1):
        g = torch.Generator(device=device).manual_seed(int(seed) * 1_000_003 + 2 * int(layer) + kind)
        s = b * w.n_kv
        a = torch.randn(s, t, r, generator=g, device=device, dtype=fdt)
        bm = torch.randn(s, r, d, generator=g, device=device, dtype=fdt) / math.sqrt(r)
        x = torch.bmm(a, bm)
        del a, bm
        x.add_(torch.randn(s, t, d, generator=g, device=device, dtype=fdt), alpha=sigma)
        if kind == 0:
            ch = outlier_channels(d, w.n_outliers, seed).to(device)
            x[..., ch] *= 8.0
            x = _rope(x, w.rope_base)
        out.append(x.to(w.dtype).reshape(b, w.n_kv, t, d))
        del x
    return out[0], out[1]
