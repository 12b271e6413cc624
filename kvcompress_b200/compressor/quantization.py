"""Integer quantisers on sm_100a (API of kvcompress/compressor/quantization.py).

``quantize_tensor`` / ``dequantize_tensor`` keep the reference's payload
dict (``q``, ``scale``, ``zero_point``, ``original_last``) and semantics:
statistics and scale arithmetic in the input dtype
(``IntQuantizer.compute_params``, quantization.py:410-452), IEEE divide,
round half to even and clamp (quantization.py:340-357), sub-byte packing
with the first element in the high bits (quantization.py:181-238).  The
work runs in ``kvc_residual_stats`` / ``kvc_residual_quant`` /
``kvc_decompress`` with no Tucker term and no rotation.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from kvcompress_b200 import ops
from kvcompress_b200._native import KVC

__all__ = ["IntQuantizer", "dequantize_tensor", "estimate_int_bytes", "quantize_tensor"]


def _mode(per_channel: bool, group_size: int | None, d: int) -> int:
    if per_channel:
        return KVC.SCALE_CHANNEL
    if group_size is not None:
        if d % int(group_size) != 0:
            raise ValueError(f"last dim {d} not divisible by group_size {group_size}")
        return KVC.SCALE_GROUP
    return KVC.SCALE_TENSOR


@dataclass
class IntQuantizer:
    """Symmetric / asymmetric 2-, 4- or 8-bit quantiser (quantization.py:278-309)."""

    bits: int
    symmetric: bool = True
    per_channel: bool = True
    group_size: int | None = None

    def __post_init__(self) -> None:
        if self.bits not in (2, 4, 8):
            raise ValueError(f"IntQuantizer bits must be 2/4/8, got {self.bits}")
        if self.symmetric:
            self.qmax = (1 << (self.bits - 1)) - 1
            self.qmin = -(1 << (self.bits - 1))
        else:
            self.qmax = (1 << self.bits) - 1
            self.qmin = 0

    @property
    def name(self) -> str:
        return f"int{self.bits}"

    def quantize_many(self, xs: list[torch.Tensor]):
        """Quantise same-shape 2-D tensors in one launch per stage."""
        x0 = xs[0]
        if x0.dim() != 2:
            xs = [x.reshape(-1, x.shape[-1]) for x in xs]
            x0 = xs[0]
        rows, d = x0.shape
        mode = _mode(self.per_channel, self.group_size, d)
        cells = [x.contiguous().view(1, rows, d) for x in xs]
        if mode == KVC.SCALE_GROUP:
            codes, scales, zps = ops.residual_quant(
                cells, None, None, None, None, bits=self.bits, symmetric=self.symmetric,
                scale_mode=mode, group_size=self.group_size, stat_dtype=x0.dtype,
                arith_dtype=torch.float32)
        else:
            scales, zps = ops.residual_stats(cells, None, None, bits=self.bits,
                                             symmetric=self.symmetric, scale_mode=mode,
                                             stat_dtype=x0.dtype)
            arith = x0.dtype if mode == KVC.SCALE_TENSOR else torch.float32
            codes, _, _ = ops.residual_quant(
                cells, None, None, scales, zps, bits=self.bits, symmetric=self.symmetric,
                scale_mode=mode, group_size=None, stat_dtype=x0.dtype, arith_dtype=arith)
        return codes, scales, zps

    def quantize(self, x: torch.Tensor):
        """``(packed, scale, zero_point)`` of one tensor."""
        codes, scales, zps = self.quantize_many([x])
        return codes[0], scales[0], zps[0]

    def dequantize_many(self, qs, scales, zps, *, original_last: int,
                        output_dtype: torch.dtype | None = None):
        rows = int(qs[0].shape[0])
        d = int(original_last)
        mode = _mode(self.per_channel, self.group_size, d) if scales[0].dim() != 0 else KVC.SCALE_TENSOR
        outs = ops.decompress((1, rows, d), output_dtype or torch.float32, codes=list(qs),
                              scales=list(scales), zps=list(zps), bits=self.bits,
                              symmetric=self.symmetric, scale_mode=mode, group_size=self.group_size,
                              n_cells=len(qs), device=qs[0].device)
        return [o.view(rows, d) for o in outs]

    def dequantize(self, q, scale, zero_point, *, original_last: int | None = None,
                   output_dtype: torch.dtype | None = None) -> torch.Tensor:
        if original_last is None:
            original_last = int(q.shape[-1])
        return self.dequantize_many([q], [scale], [zero_point], original_last=original_last,
                                    output_dtype=output_dtype)[0]


def _quantizer(dtype: str, symmetric: bool, per_channel: bool, group_size) -> IntQuantizer:
    if dtype not in ("int2", "int4", "int8"):
        raise ValueError(f"unknown quantizer name {dtype!r}")
    return IntQuantizer(bits=int(dtype[3:]), symmetric=symmetric, per_channel=per_channel,
                        group_size=group_size)


def quantize_tensor(x: torch.Tensor, *, dtype: str, symmetric: bool = True, per_channel: bool = True,
                    group_size: int | None = None) -> dict[str, torch.Tensor]:
    """Quantise ``x`` (quantization.py:518-554)."""
    q, s, z = _quantizer(dtype, symmetric, per_channel, group_size).quantize(x)
    return {"q": q, "scale": s, "zero_point": z,
            "original_last": torch.tensor(x.shape[-1], dtype=torch.int32)}


def dequantize_tensor(payload: dict[str, torch.Tensor], *, dtype: str, symmetric: bool = True,
                      per_channel: bool = True, group_size: int | None = None,
                      output_shape: tuple[int, ...] | None = None,
                      output_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Inverse of :func:`quantize_tensor` (quantization.py:557-597)."""
    qz = _quantizer(dtype, symmetric, per_channel, group_size)
    ol = payload["original_last"]
    original_last = int(ol.item()) if isinstance(ol, torch.Tensor) else int(ol)
    x = qz.dequantize(payload["q"], payload["scale"], payload["zero_point"],
                      original_last=original_last, output_dtype=output_dtype)
    return x.reshape(output_shape) if output_shape is not None else x


def estimate_int_bytes(numel: int, bits: int) -> int:
    """Bytes of ``numel`` packed ``bits``-wide integers."""
    return (numel * bits + 7) // 8
