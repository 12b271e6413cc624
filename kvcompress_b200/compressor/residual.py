"""JL-rotated residual payload (API of kvcompress/compressor/residual.py:51-315).

``encode_residual`` rotates ``R`` (any of fp32/fp16/bf16, shape
``(..., d)``) by the seeded JL matrix and quantises it
(``kvc_residual_stats`` + ``kvc_residual_quant`` with no Tucker term);
``decode_residual`` dequantises and applies ``@ Pi`` (``kvc_decompress``),
returning float32.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from kvcompress_b200 import ops
from kvcompress_b200._native import KVC
from kvcompress_b200.compressor.cells import scale_mode_of
from kvcompress_b200.compressor.jl import cached_projection

__all__ = ["ResidualPayload", "decode_residual", "encode_residual", "estimate_residual_bytes"]


@dataclass
class ResidualPayload:
    """Serialized JL-rotated residual (fields as in residual.py:51-85)."""

    projection_seed: int
    projection_distribution: str
    projection_sparsity: float
    quant_dtype: str
    symmetric: bool
    per_channel: bool
    group_size: int | None
    packed: torch.Tensor
    scale: torch.Tensor
    zero_point: torch.Tensor
    original_shape: tuple[int, ...]
    original_last: int

    @property
    def bits(self) -> int:
        return int(self.quant_dtype[3:])

    @property
    def bytes_compressed(self) -> int:
        """Byte estimate with the reference's formula (residual.py:95-108)."""
        bits = self.bits
        elem = self.packed.numel() * self.packed.element_size()
        n_entries = self.packed.numel() * (8 // max(bits, 1))
        return n_entries * ((bits + 7) // 8) + elem + self.scale.numel() * 4 + self.zero_point.numel() * 4


def encode_residual(residual: torch.Tensor, *, bits: int, seed: int, distribution: str = "gaussian",
                    sparsity: float = 1.0, symmetric: bool = True, per_channel: bool = True,
                    group_size: int | None = None) -> ResidualPayload:
    """JL rotation + uniform quantisation of ``residual`` (residual.py:155-239)."""
    if bits not in (0, 2, 4, 8):
        raise ValueError(f"bits must be 0, 2, 4, or 8, got {bits}")
    shape = tuple(residual.shape)
    dev = residual.device
    d = shape[-1]
    if bits == 0:
        return ResidualPayload(seed, distribution, sparsity, "int0", symmetric, per_channel, group_size,
                               torch.zeros(0, dtype=torch.uint8, device=dev), torch.zeros(0, device=dev),
                               torch.zeros(0, dtype=torch.int32, device=dev), shape, d)
    rows = residual.numel() // d
    cell = residual.contiguous().view(1, rows, d)
    proj = cached_projection(d, d, distribution=distribution, seed=seed, device=dev,
                             dtype=torch.float32, sparsity=sparsity).matrix
    mode = scale_mode_of(per_channel, group_size, d)
    if mode == KVC.SCALE_GROUP:
        codes, scales, zps = ops.residual_quant([cell], None, proj, None, None, bits=bits,
                                                symmetric=symmetric, scale_mode=mode,
                                                group_size=group_size, stat_dtype=torch.float32,
                                                arith_dtype=torch.float32)
    else:
        scales, zps = ops.residual_stats([cell], None, proj, bits=bits, symmetric=symmetric,
                                         scale_mode=mode, stat_dtype=torch.float32)
        codes, _, _ = ops.residual_quant([cell], None, proj, scales, zps, bits=bits, symmetric=symmetric,
                                         scale_mode=mode, group_size=None, stat_dtype=torch.float32,
                                         arith_dtype=torch.float32)
    return ResidualPayload(seed, distribution, sparsity, f"int{bits}", symmetric, per_channel, group_size,
                           codes[0], scales[0], zps[0], shape, d)


def decode_residual(payload: ResidualPayload, device: torch.device | None = None) -> torch.Tensor:
    """Dequantise and apply ``@ Pi`` (residual.py:242-288); float32 result."""
    dev = device or payload.packed.device
    if payload.quant_dtype == "int0" or payload.packed.numel() == 0:
        return torch.zeros(payload.original_shape, dtype=torch.float32, device=dev)
    d = int(payload.original_last)
    rows = int(payload.packed.shape[0])
    proj = cached_projection(d, d, distribution=payload.projection_distribution,
                             seed=payload.projection_seed, device=dev, dtype=torch.float32,
                             sparsity=payload.projection_sparsity).matrix
    mode = scale_mode_of(payload.per_channel, payload.group_size, d)
    if payload.scale.dim() == 0:
        mode = KVC.SCALE_TENSOR
    out = ops.decompress((1, rows, d), torch.float32, codes=[payload.packed.to(dev)],
                         scales=[payload.scale.to(dev)], zps=[payload.zero_point.to(dev)],
                         bits=payload.bits, symmetric=payload.symmetric, scale_mode=mode,
                         group_size=payload.group_size, proj=proj, device=dev)[0]
    return out.reshape(payload.original_shape)


def estimate_residual_bytes(shape, bits: int, per_channel: bool = True, group_size: int | None = None) -> int:
    """The reference's byte estimate (residual.py:291-315)."""
    m, t, d = shape
    if bits == 0:
        return 0
    n = m * t * d
    packed_bytes = (n * bits + 7) // 8
    proj_bytes = d * d * 4
    if per_channel:
        scale_bytes = m * t * 4 + m * t * 4
    elif group_size is not None:
        scale_bytes = (m * t * d) // group_size * 8
    else:
        scale_bytes = 8
    return packed_bytes + proj_bytes + scale_bytes
