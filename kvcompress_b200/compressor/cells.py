"""Batched GPU pipeline for JoLT cells (one layer's K and V, or many layers).

``compress_cells`` is ``compress_cell`` of the reference
(kvcompress/compressor/jolt.py:273-329 and flashjolt.py:102-169) applied to
a batch of same-shape cells that share one allocation; every stage is one
launch for the whole batch:

  1. kvc_gram           x^T [x | Omega_f]          (feature Gram + sketch)
  2. kvc_sketch_solve   U_d (d x rd), feature tail  (svd.py:221-316 / 181-219)
  3. kvc_project_feature x_proj in (T, m*rd) layout (tucker.py:251-254)
  4. kvc_gram           H = x_proj^T x_proj         (token Gram)
  5. kvc_sketch_solve   M with U_T = x_proj M, token tail
  6. kvc_apply_basis    U_T (T x rt)                (svd.py:285, 507-510)
  7. kvc_core           core (m, rt, rd)            (tucker.py:261)
  8. kvc_residual_stats + kvc_residual_quant        (jolt.py:310-328, residual.py:155-239)

``decompress_cells`` is ``reconstruct_payload`` (jolt.py:401-463) in one
fused launch.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from kvcompress_b200 import ops
from kvcompress_b200._native import KVC
from kvcompress_b200.compressor.jl import cached_projection
from kvcompress_b200.compressor.svd import SVD, sketch_omega

__all__ = ["CellResult", "compress_cells", "decompress_cells", "scale_mode_of", "tucker_cells"]


@dataclass
class CellResult:
    """Factors and residual of one compressed cell (all on the cell's device)."""

    core: torch.Tensor          # (m, rt, rd), cell dtype
    u_token: torch.Tensor       # (T, rt), cell dtype
    u_feature: torch.Tensor     # (d, rd), cell dtype
    tail_token: torch.Tensor    # () float64
    tail_feature: torch.Tensor  # () float64
    bits: int
    packed: torch.Tensor | None
    scale: torch.Tensor | None
    zero_point: torch.Tensor | None
    factors_stored: tuple | None = None  # (core, u_token, u_feature) in the payload's factor dtype
    # (pinned host tensor [token tails | feature tails] of the cell's batch,
    # index of the cell, CUDA event recorded once the host copy is done)
    tails_host: tuple | None = None


def scale_mode_of(per_channel: bool, group_size: int | None, d: int) -> int:
    """Scale layout the reference's IntQuantizer ends up using."""
    if per_channel:
        if group_size not in (None, 1):
            # quantization.py:338-346 broadcasts a (d,) scale against a
            # (n, d/g, g) view, which torch rejects
            raise RuntimeError("per-channel scales cannot be combined with group_size > 1 "
                               f"(got group_size={group_size})")
        return KVC.SCALE_CHANNEL
    if group_size is not None:
        if d % int(group_size) != 0:
            raise ValueError(f"last dim {d} not divisible by group_size {group_size}")
        return KVC.SCALE_GROUP
    return KVC.SCALE_TENSOR


def tucker_cells(xs: list[torch.Tensor], *, r_token: int, r_feature: int, svd: SVD,
                 cap: int | None = None, forced_randomised: bool = False):
    """Partial Tucker ST-HOSVD of same-shape cells (tucker.py:192-279).

    Returns lists ``(core, u_token, u_feature)`` in the cell dtype and the
    per-cell token / feature tail masses as float64 device tensors.
    """
    xs = ops.cells(xs, "tucker")
    x0 = xs[0]
    m, t, d = (int(s) for s in x0.shape)
    dt = x0.dtype
    dev = x0.device
    # ranks clipped by the axis lengths (tucker.py:230-238)
    rt_req = max(1, min(int(r_token), t))
    rd_req = max(1, min(int(r_feature), d))

    # --- feature mode: A_f = (d, m*T) -------------------------------------
    n_f = m * t
    mode_f, rd, k_f = svd.resolve(d, n_f, rd_req, cap, forced_randomised)
    om_f = sketch_omega(n_f, k_f, svd.seed, dev) if mode_f == KVC.SVD_RANDOMISED else None
    flat = xs.reshape(n_f, d)
    g_f = ops.gram(flat, om_f)
    u_d, tail_f, _ = ops.sketch_solve(g_f, mode=mode_f, side=KVC.SIDE_LEFT, p=d, n_other=n_f, k=k_f,
                                      rank=rd, n_power=svd.n_power, omega=None, basis_dtype=dt, want_sv2=False)
    u_feature = ops.split(u_d)

    # --- projection to (T, m*rd) ------------------------------------------
    x_proj_t = ops.project_feature(xs, u_feature)

    # --- token mode: A_t = (T, m*rd) -------------------------------------
    c = m * rd
    mode_t, rt, k_t = svd.resolve(t, c, rt_req, cap, forced_randomised)
    om_t = sketch_omega(c, k_t, svd.seed, dev) if mode_t == KVC.SVD_RANDOMISED else None
    g_t = ops.gram(x_proj_t, None)
    mat, tail_t, _ = ops.sketch_solve(g_t, mode=mode_t, side=KVC.SIDE_RIGHT, p=c, n_other=t, k=k_t,
                                      rank=rt, n_power=svd.n_power, omega=om_t,
                                      basis_dtype=torch.float64, want_sv2=False)
    u_token = ops.apply_basis(x_proj_t, mat)
    core = ops.core(x_proj_t, u_token, m, rd)
    return core, u_token, u_feature, tail_t, tail_f


def compress_cells(
    xs: list[torch.Tensor],
    *,
    r_token: int,
    r_feature: int,
    bits: int,
    svd: SVD,
    cap: int | None = None,
    forced_randomised: bool = False,
    seed: int = 0,
    jl_distribution: str = "gaussian",
    sparsity: float = 1.0,
    symmetric: bool = True,
    per_channel: bool = True,
    group_size: int | None = None,
    factor_dtype: torch.dtype | None = None,
) -> list[CellResult]:
    """Compress same-shape cells ``(m, T, d)`` sharing one allocation.

    With ``factor_dtype`` the factors are also returned cast to it (one
    launch per factor kind for the whole batch), as the payload stores them.
    """
    if bits not in (0, 2, 4, 8):
        raise ValueError(f"bits must be 0, 2, 4, or 8, got {bits}")
    x0 = xs[0]
    m, t, d = (int(s) for s in x0.shape)
    dt = x0.dtype
    dev = x0.device
    n = len(xs)
    if n > KVC.MAX_CELLS:
        out: list[CellResult] = []
        for i in range(0, n, KVC.MAX_CELLS):
            out += compress_cells(xs[i:i + KVC.MAX_CELLS], r_token=r_token, r_feature=r_feature,
                                  bits=bits, svd=svd, cap=cap, forced_randomised=forced_randomised,
                                  seed=seed, jl_distribution=jl_distribution, sparsity=sparsity,
                                  symmetric=symmetric, per_channel=per_channel, group_size=group_size,
                                  factor_dtype=factor_dtype)
        return out
    xs = ops.cells(xs, "compress")
    mode_scale = scale_mode_of(per_channel, group_size, d) if bits > 0 else KVC.SCALE_CHANNEL
    # ranks clipped by the axis lengths and each side's SVD mode and sketch
    # (tucker.py:230-262, svd.py:221-316): the same decisions as tucker_cells
    rt_req = max(1, min(int(r_token), t))
    rd_req = max(1, min(int(r_feature), d))
    mode_f, rd, k_f = svd.resolve(d, m * t, rd_req, cap, forced_randomised)
    om_f = sketch_omega(m * t, k_f, svd.seed, dev) if mode_f == KVC.SVD_RANDOMISED else None
    c = m * rd
    mode_t, rt, k_t = svd.resolve(t, c, rt_req, cap, forced_randomised)
    om_t = sketch_omega(c, k_t, svd.seed, dev) if mode_t == KVC.SVD_RANDOMISED else None
    proj = cached_projection(d, d, distribution=jl_distribution, seed=seed, device=dev, dtype=torch.float32,
                             sparsity=sparsity).matrix if bits > 0 else None
    r = ops.compress(xs, rt=rt, rd=rd, mode_f=mode_f, k_f=k_f, omega_f=om_f, mode_t=mode_t, k_t=k_t,
                     omega_t=om_t, n_power=svd.n_power, proj=proj, bits=bits, symmetric=symmetric,
                     scale_mode=mode_scale, group_size=group_size, factor_dtype=factor_dtype)
    core, u_token, u_feature = ops.split(r["core"]), ops.split(r["u_token"]), ops.split(r["u_feature"])
    tail_t, tail_f = ops.split(r["tail_token"]), ops.split(r["tail_feature"])
    if bits > 0:
        packed, scale, zps = ops.split(r["codes"]), ops.split(r["scale"]), ops.split(r["zero_point"])
    else:
        packed = scale = zps = [None] * n
    stored = [None] * n
    if factor_dtype is not None:
        sc, su, sf = (r[k + "_stored"] if r[k + "_stored"] is not None else r[k]
                      for k in ("core", "u_token", "u_feature"))
        sc, su, sf = ops.split(sc), ops.split(su), ops.split(sf)
        stored = [(sc[i], su[i], sf[i]) for i in range(n)]
    th = r["tails_host"], r["tails_ready"]
    return [CellResult(core=core[i], u_token=u_token[i], u_feature=u_feature[i],
                       tail_token=tail_t[i], tail_feature=tail_f[i], bits=bits, packed=packed[i],
                       scale=scale[i], zero_point=zps[i], factors_stored=stored[i],
                       tails_host=(th[0], i, th[1])) for i in range(n)]


def _batch_of(views: list[torch.Tensor]) -> torch.Tensor:
    """The (n, ...) tensor a list of per-cell views was cut from."""
    if isinstance(views, ops.Cells) and views.batch is not None:
        return views.batch
    base = views[0]._base
    if (base is not None and base.dim() == views[0].dim() + 1 and base.shape[0] == len(views)
            and base.shape[1:] == views[0].shape and base[0].data_ptr() == views[0].data_ptr()
            and all(v._base is base for v in views)):
        return base
    return torch.stack(views)


def decode_args(payloads, out_dtype: torch.dtype | None = None):
    """``(shape, out dtype, device, keyword arguments of ops.decompress)`` of
    same-layout JoLT payloads (at most ``KVC.MAX_CELLS``)."""
    p0 = payloads[0]
    m, t, d = (int(s) for s in p0.shape)
    dev = p0.data["core"].device
    odt = out_dtype or p0.dtype
    kw: dict = {"factors": ([p.data["core"] for p in payloads], [p.data["u_token"] for p in payloads],
                            [p.data["u_feature"] for p in payloads])}
    bits = int(p0.metadata.get("bits", 0)) if "residual_packed" in p0.data else 0
    if bits and p0.data["residual_packed"].numel() == 0:
        bits = 0
    if bits > 0:
        meta = p0.metadata
        mode = scale_mode_of(bool(meta["residual_per_channel"]), meta.get("residual_group_size"), d)
        proj = cached_projection(d, d, distribution=meta["residual_distribution"],
                                 seed=int(meta["residual_seed"]), device=dev, dtype=torch.float32,
                                 sparsity=float(meta["residual_sparsity"])).matrix
        kw.update(codes=[p.data["residual_packed"] for p in payloads],
                  scales=[p.data["residual_scale"] for p in payloads],
                  zps=[p.data["residual_zero_point"] for p in payloads], bits=bits,
                  symmetric=bool(meta["residual_symmetric"]), scale_mode=mode,
                  group_size=meta.get("residual_group_size"), proj=proj)
    return (m, t, d), odt, dev, kw


def decompress_cells(payloads, out_dtype: torch.dtype | None = None, t0: int = 0,
                     t1: int | None = None) -> list[torch.Tensor]:
    """Reconstruct same-layout JoLT payloads in one fused launch per batch.

    ``payloads`` share shape, ranks, bits and quantiser settings; returns
    ``(m, t1 - t0, d)`` tensors in each payload's original dtype.
    """
    if len(payloads) > KVC.MAX_CELLS:
        out = []
        for i in range(0, len(payloads), KVC.MAX_CELLS):
            out += decompress_cells(payloads[i:i + KVC.MAX_CELLS], out_dtype, t0, t1)
        return out
    shape, odt, dev, kw = decode_args(payloads, out_dtype)
    return ops.decompress(shape, odt, t0=t0, t1=t1, n_cells=len(payloads), device=dev, **kw)
