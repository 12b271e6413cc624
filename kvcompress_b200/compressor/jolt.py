"""JoLT compressor on sm_100a (API of kvcompress/compressor/jolt.py:82-463).

``compress(K, V)`` allocates (r_token, r_feature, bits) for the two cells
with the joint Lagrangian allocator, runs the batched GPU pipeline
(:mod:`kvcompress_b200.compressor.cells`) on K and V together and emits the
reference's payload schema: fp16 ``core``/``u_token``/``u_feature`` and the
``residual_*`` tensors (jolt.py:331-399).  ``decompress`` reconstructs both
payloads in one fused kernel launch.

Beyond the reference API, :meth:`JoLTCompressor.compress_many` /
:meth:`decompress_many` take many layers at once: every stage is then one
launch for all cells, and the host synchronises once per call (to read the
tail masses that go into ``metadata``).
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Sequence

import torch

from kvcompress_b200 import ops
from kvcompress_b200.compressor.allocator import AllocationResult, Cell, JointAllocator
from kvcompress_b200.compressor.base import CompressedPayload, CompressorStats, KVCompressor
from kvcompress_b200.compressor.cells import CellResult, compress_cells, decompress_cells
from kvcompress_b200.compressor.svd import SVD

# metadata that must agree for payloads to share one decode launch
_GROUP_META = ("bits", "residual_seed", "residual_distribution", "residual_sparsity", "residual_symmetric",
               "residual_per_channel", "residual_group_size")

def group_payloads(flat) -> list[list[int]]:
    """Indices of payloads that can share one decode launch (same shape,
    dtype, ranks, factor dtype, device, bits and quantiser settings)."""
    groups: dict[tuple, list[int]] = {}
    for i, p in enumerate(flat):
        md = p.metadata
        core = p.data["core"]
        packed = p.data.get("residual_packed")
        gk = (tuple(p.shape), p.dtype, core.shape, core.dtype, core.get_device(),
              packed is not None and packed.numel() > 0, *(md.get(k) for k in _GROUP_META))
        groups.setdefault(gk, []).append(i)
    return list(groups.values())


_DESC: dict[tuple[int, int, int, int], tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}

__all__ = ["JoLTCompressor", "JoLTFactors"]

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


@dataclass
class JoLTFactors:
    """Per-cell factors, residual and allocation (jolt.py:67-79)."""

    tucker: CellResult
    residual: Any
    allocation: Any


class JoLTCompressor(KVCompressor):
    """Paper-faithful JoLT with exact SVDs by default (jolt.py:82-141)."""

    name = "jolt"

    def __init__(self, *, compression_ratio: float = 3.0, bits: tuple[int, ...] = (0, 2, 4, 8),
                 factor_dtype: torch.dtype = torch.float16, jl_distribution: str = "gaussian",
                 allocator: JointAllocator | None = None, svd: SVD | None = None,
                 symmetric_quant: bool = True, per_channel_quant: bool = True,
                 group_size: int | None = None, layer_groups: int = 1, seed: int = 0,
                 **unused: Any) -> None:
        super().__init__()
        if compression_ratio <= 1.0:
            raise ValueError(f"compression_ratio must be > 1.0, got {compression_ratio}")
        self.compression_ratio = float(compression_ratio)
        self.bits = tuple(bits)
        self.factor_dtype = factor_dtype
        self.jl_distribution = jl_distribution
        self.allocator = allocator or JointAllocator(target_ratio=compression_ratio,
                                                     bits_grid=self.bits,
                                                     factor_dtype_bytes=factor_dtype.itemsize)
        self.svd = svd or SVD(seed=seed, method="exact")
        self.symmetric_quant = symmetric_quant
        self.per_channel_quant = per_channel_quant
        self.group_size = group_size
        self.layer_groups = int(layer_groups)
        self.seed = int(seed)
        self.last_stats = CompressorStats()
        self.call_count = 0

    # ------------------------------------------------------------------ api

    def compress(self, key: torch.Tensor, value: torch.Tensor) -> tuple[CompressedPayload, CompressedPayload]:
        """Allocator-driven JoLT compression of one layer's ``(m, T, dh)`` K and V."""
        return self.compress_many([(key, value)])[0]

    def decompress(self, key_payload: CompressedPayload,
                   value_payload: CompressedPayload) -> tuple[torch.Tensor, torch.Tensor]:
        """Inverse of :meth:`compress` (jolt.py:228-253)."""
        t0 = time.perf_counter()
        out = self.decompress_many([(key_payload, value_payload)])[0]
        elapsed = (time.perf_counter() - t0) * 1000
        if self.last_stats.decompress_time_ms == 0.0:
            self.last_stats.decompress_time_ms = elapsed
        return out

    def stats(self) -> dict[str, Any]:
        return {"method": self.name, "call_count": self.call_count, **self.last_stats.to_dict()}

    # ------------------------------------------------------------- batched

    def compress_many(self, pairs: Sequence[tuple[torch.Tensor, torch.Tensor]]) -> list[tuple[CompressedPayload, CompressedPayload]]:
        """Compress several layers; cells of equal shape and allocation share launches."""
        t_start = time.perf_counter()
        plans = []
        # layers of one shape share the allocation: (result, (K allocation, V allocation))
        alloc_of: dict[torch.Size, tuple[AllocationResult, tuple]] = {}
        # group cells by (shape, dtype, device, allocation) so each group is one batch; every tensor
        # attribute is read once (a 64-cell call spends its host time on such reads)
        groups: dict[tuple, list[tuple[int, int]]] = {}
        for li, (key, value) in enumerate(pairs):
            ks, kdt, kdev = key.shape, key.dtype, key.device
            vs, vdt, vdev = value.shape, value.dtype, value.device
            if ks != vs:
                raise ValueError(f"K/V shape mismatch: {ks} vs {vs}")
            if len(ks) != 3:
                raise ValueError(f"JoLT expects 3-D (m, T, dh); got {tuple(ks)}")
            for dev, dt in ((kdev, kdt), (vdev, vdt)):
                if dev.type != "cuda":
                    raise RuntimeError(f"kvcompress_b200 compresses CUDA tensors only (got a {dev} tensor)")
                if dt not in _DTYPES:
                    raise TypeError(f"unsupported K/V dtype {dt}")
            hit = alloc_of.get(ks)
            if hit is None:
                m, t, d = ks
                res = self.allocator.optimize([
                    Cell(shape=(m, t, d), kind="key", layer_group=0, candidate_bits=self.bits),
                    Cell(shape=(m, t, d), kind="value", layer_group=0, candidate_bits=self.bits)])
                hit = alloc_of[ks] = (res, tuple(a.tuple for a in res.allocations))
            plans.append(hit[0])
            groups.setdefault((ks, kdt, kdev, hit[1][0]), []).append((li, 0))
            groups.setdefault((ks, vdt, vdev, hit[1][1]), []).append((li, 1))
        results: dict[tuple[int, int], CellResult] = {}
        order, tails_t = [], []
        for (shape, _, _, (rt, rd, b)), members in groups.items():
            # same shape, dtype and device by the grouping, CUDA and a K/V dtype by
            # the checks above: the batch goes to the kernels without re-checks
            xs = ops.Cells([pairs[li][side].contiguous() for li, side in members])
            cell_res = self._compress_cells(xs, rt, rd, b, shape[1])
            for (li, side), r in zip(members, cell_res):
                results[(li, side)] = r
            order += members
            tails_t.append(cell_res)
        # payloads first (host work that overlaps the kernels still running),
        # then one host sync for every tail mass (one small copy per batch)
        out = []
        for li, ((key, value), res) in enumerate(zip(pairs, plans)):
            k_alloc, v_alloc = res.allocations
            kp = self.build_payload(key, JoLTFactors(results[(li, 0)], None, k_alloc), (0.0, 0.0))
            vp = self.build_payload(value, JoLTFactors(results[(li, 1)], None, v_alloc), (0.0, 0.0))
            out.append((kp, vp))
        # the tail masses, copied to pinned host memory by kvc_compress as soon
        # as the solves were done: usually ready by now, while the residual
        # passes still run
        tt_all, tf_all = [], []
        for cell_res in tails_t:
            host, _, ready = cell_res[0].tails_host
            ready.synchronize()
            vals = host.tolist()
            k = len(cell_res)
            tt_all += vals[:k]
            tf_all += vals[k:2 * k]
        for (li, side), tt, tf in zip(order, tt_all, tf_all):
            md = out[li][side].metadata
            md["tail_token_mass"] = float(tt)
            md["tail_feature_mass"] = float(tf)
        elapsed = (time.perf_counter() - t_start) * 1000
        key, value = pairs[-1]
        kp, vp = out[-1]
        k_alloc, v_alloc = plans[-1].allocations
        self.last_stats = CompressorStats(
            compress_time_ms=elapsed,
            bytes_original=key.numel() * key.element_size() * 2,
            bytes_compressed=kp.bytes_compressed + vp.bytes_compressed,
            extra={
                "k_r_token": k_alloc.r_token, "k_r_feature": k_alloc.r_feature, "k_bits": k_alloc.bits,
                "v_r_token": v_alloc.r_token, "v_r_feature": v_alloc.r_feature, "v_bits": v_alloc.bits,
                "lambda_star": plans[-1].lambda_star, "achieved_ratio": plans[-1].achieved_ratio,
                "target_ratio": plans[-1].target_ratio,
            },
        )
        self.call_count += len(pairs)
        return out

    def decompress_many(self, pairs: Sequence[tuple[CompressedPayload, CompressedPayload]]) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """Reconstruct several layers; compatible payloads share one launch."""
        flat = [p for pair in pairs for p in pair]
        for p in flat:
            if p.method != "jolt":
                raise ValueError(f"JoLT cannot decode payload with method={p.method!r}")
        outs: list[torch.Tensor | None] = [None] * len(flat)
        for members in group_payloads(flat):
            rec = decompress_cells([flat[i] for i in members])
            for i, r in zip(members, rec):
                outs[i] = r
        return [(outs[2 * i], outs[2 * i + 1]) for i in range(len(pairs))]

    # ------------------------------------------------------------ internals

    def _compress_cells(self, xs, rt, rd, bits, t) -> list[CellResult]:
        return compress_cells(xs, r_token=rt, r_feature=rd, bits=bits, svd=self.svd, seed=self.seed,
                              jl_distribution=self.jl_distribution,
                              symmetric=self.symmetric_quant, per_channel=self.per_channel_quant,
                              group_size=self.group_size, factor_dtype=self.factor_dtype)

    def compress_cell(self, x: torch.Tensor, allocation: Any) -> JoLTFactors:
        """One cell at a given allocation (jolt.py:273-329)."""
        r = self._compress_cells([x.contiguous()], int(allocation.r_token), int(allocation.r_feature),
                                 int(allocation.bits), x.shape[1])[0]
        return JoLTFactors(tucker=r, residual=None, allocation=allocation)

    def build_payload(self, original: torch.Tensor, factors: JoLTFactors,
                      tails: Sequence[float] | None = None) -> CompressedPayload:
        """Payload with the reference's keys, dtypes and metadata (jolt.py:331-399)."""
        r: CellResult = factors.tucker
        if tails is None:
            tails = torch.stack([r.tail_token, r.tail_feature]).cpu().tolist()
        fdt = self.factor_dtype
        if r.factors_stored is not None and r.factors_stored[0].dtype == fdt:
            core, u_token, u_feature = r.factors_stored
        else:
            core = ops.cast(r.core, fdt) if r.core.dtype != fdt else r.core.contiguous()
            u_token = ops.cast(r.u_token, fdt) if r.u_token.dtype != fdt else r.u_token.contiguous()
            u_feature = ops.cast(r.u_feature, fdt) if r.u_feature.dtype != fdt else r.u_feature.contiguous()
        data: dict[str, Any] = {"core": core, "u_token": u_token, "u_feature": u_feature}
        meta: dict[str, Any] = {
            "method": "jolt",
            "r_token": int(u_token.shape[1]),
            "r_feature": int(u_feature.shape[1]),
            "bits": factors.allocation.bits,
            "core_dtype": "fp16" if fdt == torch.float16 else "fp32",
            "tail_token_mass": float(tails[0]),
            "tail_feature_mass": float(tails[1]),
        }
        dev = original.device
        m, t, d = original.shape
        meta["residual_seed"] = self.seed
        meta["residual_distribution"] = self.jl_distribution
        meta["residual_sparsity"] = 1.0
        meta["residual_symmetric"] = self.symmetric_quant
        meta["residual_per_channel"] = self.per_channel_quant
        meta["residual_group_size"] = self.group_size
        if r.bits == 0:
            data["residual_packed"] = torch.zeros(0, dtype=torch.uint8, device=dev)
            data["residual_scale"] = torch.zeros(0, device=dev)
            data["residual_zero_point"] = torch.zeros(0, dtype=torch.int32, device=dev)
        else:
            data["residual_packed"] = r.packed
            data["residual_scale"] = r.scale
            data["residual_zero_point"] = r.zero_point
        # small int32 descriptors live on the host, as in the reference; they
        # are read-only, so payloads of one shape share them
        tmpl = _DESC.get((m, t, d, r.bits))
        if tmpl is None:
            tmpl = (torch.tensor([m, t, d], dtype=torch.int32), torch.tensor(d, dtype=torch.int32),
                    torch.tensor(r.bits, dtype=torch.int32))
            _DESC[(m, t, d, r.bits)] = tmpl
        data["residual_original_shape"], data["residual_original_last"], data["residual_dtype"] = tmpl
        return CompressedPayload(
            method="jolt", shape=tuple(original.shape), dtype=original.dtype, metadata=meta, data=data,
            stats=CompressorStats(
                bytes_original=original.numel() * original.element_size(),
                bytes_compressed=core.numel() * core.element_size()
                + u_token.numel() * u_token.element_size()
                + u_feature.numel() * u_feature.element_size()))

    def reconstruct_payload(self, payload: CompressedPayload) -> torch.Tensor:
        """One payload back to ``payload.dtype`` / ``payload.shape`` (jolt.py:401-463)."""
        if payload.method != "jolt":
            raise ValueError(f"JoLT cannot decode payload with method={payload.method!r}")
        return decompress_cells([payload])[0]

    def decompress_tokens(self, payload: CompressedPayload, t0: int, t1: int) -> torch.Tensor:
        """Reconstruct only tokens ``[t0, t1)`` of one payload: ``(m, t1 - t0, d)``."""
        if payload.method != "jolt":
            raise ValueError(f"JoLT cannot decode payload with method={payload.method!r}")
        return decompress_cells([payload], t0=t0, t1=t1)[0]
