"""Square Johnson-Lindenstrauss rotation of the residual.

The JL matrix is generated on the host exactly as the reference generates
it (kvcompress/compressor/jl.py:108-174: a fresh CPU ``torch.Generator``
seeded with ``seed``, N(0, 1)/sqrt(d) or Rademacher entries), so it is
bit-identical; it is then copied once to the device and cached per
(shape, distribution, seed, device) like ``cached_projection``
(jl.py:185-235).  The kernels apply it as ``R @ Pi^T`` on encode and
``Rt @ Pi`` on decode (the reference's "cheap inverse", jl.py:90-105).
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Literal

import torch

__all__ = ["JLDistribution", "JLProjection", "cached_projection", "clear_projection_cache",
           "gaussian_projection", "rademacher_projection"]

JLDistribution = Literal["gaussian", "rademacher"]


@dataclass
class JLProjection:
    """A JL matrix (``output_dim x input_dim``) and how it was drawn."""

    matrix: torch.Tensor
    distribution: JLDistribution
    seed: int

    @property
    def device(self) -> torch.device:
        return self.matrix.device

    @property
    def dtype(self) -> torch.dtype:
        return self.matrix.dtype

    def apply(self, x: torch.Tensor) -> torch.Tensor:
        """``x @ matrix.T`` along the last axis."""
        if x.shape[-1] != self.matrix.shape[-1]:
            raise ValueError(f"JL apply: trailing dim mismatch: x.shape[-1]={x.shape[-1]}, "
                             f"matrix.shape[-1]={self.matrix.shape[-1]}")
        return x @ self.matrix.t()

    def apply_inverse(self, x: torch.Tensor) -> torch.Tensor:
        """``x @ matrix`` (the decode-side map, not the matrix inverse)."""
        return x @ self.matrix


def gaussian_projection(output_dim: int, input_dim: int, *, seed: int,
                        device: torch.device | str = "cpu",
                        dtype: torch.dtype = torch.float32) -> JLProjection:
    """N(0, 1/input_dim) entries drawn on a seeded CPU generator."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(int(seed))
    mat = torch.randn(output_dim, input_dim, generator=gen, dtype=torch.float32)
    mat = mat / (input_dim ** 0.5)
    return JLProjection(matrix=mat.to(device=device, dtype=dtype), distribution="gaussian",
                        seed=int(seed))


def rademacher_projection(output_dim: int, input_dim: int, *, seed: int,
                          device: torch.device | str = "cpu", dtype: torch.dtype = torch.float32,
                          sparsity: float = 1.0) -> JLProjection:
    """+-1/sqrt(input_dim) entries (sparse Achlioptas form when sparsity < 1)."""
    if not 0 < sparsity <= 1:
        raise ValueError(f"sparsity must be in (0, 1], got {sparsity}")
    gen = torch.Generator(device="cpu")
    gen.manual_seed(int(seed))
    if sparsity == 1.0:
        mat = (torch.randint(0, 2, (output_dim, input_dim), generator=gen) * 2 - 1).to(torch.float32)
    else:
        keep = (torch.rand(output_dim, input_dim, generator=gen) < sparsity).to(torch.float32)
        signs = (torch.randint(0, 2, (output_dim, input_dim), generator=gen) * 2 - 1).to(torch.float32)
        mat = keep * signs / (sparsity ** 0.5)
    mat = mat / (input_dim ** 0.5)
    return JLProjection(matrix=mat.to(device=device, dtype=dtype), distribution="rademacher",
                        seed=int(seed))


_CACHE: dict[tuple, JLProjection] = {}
_CACHE_LOCK = threading.Lock()


def cached_projection(output_dim: int, input_dim: int, *, distribution: JLDistribution = "gaussian",
                      seed: int = 0, device: torch.device | str = "cpu",
                      dtype: torch.dtype = torch.float32, sparsity: float = 1.0) -> JLProjection:
    """Process-wide cache of JL matrices keyed by (shape, distribution, seed, device)."""
    key = (output_dim, input_dim, distribution, int(seed), str(torch.device(device)), float(sparsity),
           dtype)
    with _CACHE_LOCK:
        proj = _CACHE.get(key)
        if proj is None:
            if distribution == "gaussian":
                proj = gaussian_projection(output_dim, input_dim, seed=seed, device=device, dtype=dtype)
            elif distribution == "rademacher":
                proj = rademacher_projection(output_dim, input_dim, seed=seed, device=device,
                                             dtype=dtype, sparsity=sparsity)
            else:
                raise ValueError(f"unknown JL distribution {distribution!r}")
            _CACHE[key] = proj
    return proj


def clear_projection_cache() -> None:
    """Drop every cached JL matrix."""
    with _CACHE_LOCK:
        _CACHE.clear()
