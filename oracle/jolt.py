"""numpy restatement of the reference JoLT / FlashJoLT path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function
names the reference file:line it restates; paths are relative to the
reference project root (``kvcompress/compressor/...``).

Conventions
-----------
* Tensors are numpy ``float32`` arrays that hold values of the *logical*
  dtype ``dt`` ('f32', 'f16' or 'bf16'): after every operation the
  reference performs in bf16/fp16, the oracle rounds with :func:`round_to`.
* Matrix products accumulate in float32 (BLAS sgemm), as the reference's
  fp32 and bf16 torch matmuls do, and round once at the end.
* Random matrices are arguments: ``proj`` is the JL matrix Pi (d x d) and
  ``omega_fn(n, k)`` returns the randomised-SVD sketch for an (m x n)
  matrix, exactly as ``torch.manual_seed(seed); torch.randn(n, k)`` gives it
  to the reference (``svd.py:259-260``).
"""

from __future__ import annotations

import math
from typing import Callable

import numpy as np

__all__ = [
    "EPSILON_SQUARED",
    "allocate",
    "bytes_original",
    "candidate_feature_ranks",
    "candidate_token_ranks",
    "dequantize",
    "exact_svd",
    "flashjolt_cap",
    "fp8_e4m3fn_round",
    "jolt_compress_cell",
    "jolt_decompress_cell",
    "pack_codes",
    "partial_tucker",
    "quant_params",
    "quantize_codes",
    "randomised_svd",
    "reconstruct_tucker",
    "round_bf16",
    "round_to",
    "sketch_width",
    "unpack_codes",
]


# ---------------------------------------------------------------------------
# dtype rounding
# ---------------------------------------------------------------------------


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even).

    Same rule as torch's ``c10::BFloat16`` conversion: add ``0x7FFF`` plus
    the lowest kept bit, truncate the low 16 bits; NaN stays NaN.
    """
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32("nan")
    return out


def round_to(a: np.ndarray, dt: str) -> np.ndarray:
    """Round float32 values to the logical dtype ``dt`` and return float32."""
    a = np.asarray(a, dtype=np.float32)
    if dt == "f32":
        return a
    if dt == "f16":
        with np.errstate(over="ignore"):
            return a.astype(np.float16).astype(np.float32)
    if dt == "bf16":
        return round_bf16(a)
    raise ValueError(dt)


def dt_op(fn, dt: str, *args):
    """Elementwise op computed in float32 then rounded to ``dt``.

    torch's CPU bf16/fp16 kernels widen to float, compute, and round.
    """
    with np.errstate(all="ignore"):
        return round_to(fn(*[np.asarray(x, dtype=np.float32) for x in args]), dt)


def matmul_round(a: np.ndarray, b: np.ndarray, dt: str) -> np.ndarray:
    """fp32-accumulated product rounded once to ``dt``."""
    return round_to(np.matmul(a.astype(np.float32), b.astype(np.float32)), dt)


# ---------------------------------------------------------------------------
# Allocator -- allocator.py
# ---------------------------------------------------------------------------

# allocator.py:53
EPSILON_SQUARED = {0: 1.0, 2: 0.30, 4: 0.10, 8: 0.04}


def bytes_original(shape, element_size_bytes: int = 2) -> int:
    """allocator.py:613-633."""
    n = 1
    for s in shape:
        n *= int(s)
    return n * int(element_size_bytes)


def candidate_feature_ranks(d: int) -> list[int]:
    """allocator.py:636-645."""
    if d <= 32:
        return list(range(1, d + 1))
    c = sorted({1, 2, 4, 8, 16, 32, 64, 96, 128, 192, 256, d})
    return [x for x in c if x <= d]


def candidate_token_ranks(t_max: int) -> list[int]:
    """allocator.py:648-654."""
    if t_max <= 32:
        return list(range(1, t_max + 1))
    base = list(range(1, 33))
    extras = sorted({48, 64, 96, 128, 192, 256, 384, 512, t_max})
    return base + [e for e in extras if e <= t_max]


def _cell_grid(shape, bits_grid, eps, factor_bytes, max_token_rank):
    """allocator.py:309-375 (with tau_error's default model, 377-408)."""
    m, t, d = shape
    grid = []
    for rt in candidate_token_ranks(min(t, max_token_rank)):
        for rd in candidate_feature_ranks(d):
            rt = min(rt, t)
            rd = min(rd, d)
            tucker_bytes = (m * rt * rd + t * rt + d * rd) * factor_bytes
            tau = max(0.0, max(1.0 - rt / max(t, 1), 1.0 - rd / max(d, 1)))
            for b in bits_grid:
                cost = tucker_bytes + (b // 8) * m * t * d
                grid.append((rt, rd, b, cost, eps.get(b, 1.0) * tau))
    return grid


def _argmin(grids, lam):
    """allocator.py:410-434 (first strict minimum of error + lam * cost)."""
    out = []
    for grid in grids:
        best = grid[0]
        best_obj = grid[0][4] + lam * grid[0][3]
        for a in grid[1:]:
            obj = a[4] + lam * a[3]
            if obj < best_obj:
                best, best_obj = a, obj
        out.append(best)
    return out


def allocate(
    shapes,
    target_ratio: float,
    *,
    bits_grid=(0, 2, 4, 8),
    epsilon_squared=None,
    factor_dtype_bytes: int = 2,
    element_size_bytes: int = 2,
    max_token_rank: int = 512,
):
    """``JointAllocator.optimize`` (allocator.py:169-303, make_result 436-466).

    Returns a dict with per-cell ``(r_token, r_feature, bits, cost, error)``
    tuples and the result scalars.
    """
    eps = dict(epsilon_squared or EPSILON_SQUARED)
    if not shapes:
        return dict(allocations=[], total_bytes=0, target_bytes=0, achieved_ratio=1.0,
                    target_ratio=float(target_ratio), lambda_star=0.0)
    original = sum(bytes_original(s, element_size_bytes) for s in shapes)
    target_bytes = max(1, int(round(original / target_ratio)))
    grids = [_cell_grid(s, tuple(bits_grid), eps, factor_dtype_bytes, max_token_rank) for s in shapes]

    cands = []
    for i in range(180):
        lam = 10.0 ** (-12 + 0.1 * i)
        cand = _argmin(grids, lam)
        total = sum(a[3] for a in cand)
        if total <= 0:
            continue
        score = abs(math.log(original / total) - math.log(target_ratio))
        cands.append((score, total, cand, lam))
    cands.sort(key=lambda c: c[0])
    _, _, best_cand, best_lam = cands[0]

    lo = best_lam / 10 if best_lam > 0 else 1e-12
    hi = best_lam * 10 if best_lam > 0 else 1e-6
    cand_lo, cand_hi = _argmin(grids, lo), _argmin(grids, hi)
    cost_lo = sum(a[3] for a in cand_lo)
    cost_hi = sum(a[3] for a in cand_hi)
    if cost_lo > cost_hi:
        lo, hi, cost_lo, cost_hi = hi, lo, cost_hi, cost_lo
    for _ in range(60):
        if cost_lo > target_bytes and cost_hi < target_bytes:
            break
        if cost_lo < target_bytes:
            lo /= 10
            cost_lo = sum(a[3] for a in _argmin(grids, lo))
        elif cost_hi > target_bytes:
            hi *= 10
            cost_hi = sum(a[3] for a in _argmin(grids, hi))
        else:
            break
    for _ in range(40):
        mid = (lo + hi) / 2
        cost_mid = sum(a[3] for a in _argmin(grids, mid))
        if cost_mid > target_bytes:
            lo, cost_lo = mid, cost_mid
        else:
            hi, cost_hi = mid, cost_mid
    cand_mid = _argmin(grids, (lo + hi) / 2)
    cost_mid = sum(a[3] for a in cand_mid)
    if cost_mid > 0:
        score_mid = abs(math.log(original / cost_mid) - math.log(target_ratio))
        if score_mid < cands[0][0]:
            best_cand, best_lam = cand_mid, (lo + hi) / 2
    total = sum(a[3] for a in best_cand)
    per_cell = [bytes_original(s, element_size_bytes) for s in shapes]
    return dict(
        allocations=best_cand,
        total_bytes=total,
        target_bytes=target_bytes,
        achieved_ratio=(sum(per_cell) / total) if total > 0 else 1.0,
        target_ratio=float(target_ratio),
        lambda_star=best_lam,
    )


def flashjolt_cap(context_length: int, target_ratio: float) -> int:
    """flashjolt.py:49-66."""
    q_min = 64 if target_ratio >= 5.0 else 32
    return min(max(q_min, math.ceil(context_length / 32)), 512)


# ---------------------------------------------------------------------------
# SVD -- svd.py
# ---------------------------------------------------------------------------


def sketch_width(rows: int, cols: int, rank: int, oversampling: int = 10, cap=None):
    """Clipped rank and sketch width of ``SVD.randomise`` (svd.py:447-455)."""
    max_rank = min(rows, cols)
    rank = max(1, min(int(rank), max_rank))
    k = rank + oversampling
    if cap is not None:
        k = min(k, int(cap))
    k = max(k, rank + 1)
    k = min(k, max_rank)
    return rank, k


def randomised_svd(a: np.ndarray, rank: int, omega: np.ndarray, n_power: int = 2):
    """``SVD.randomise`` (svd.py:221-316) for a float32 matrix ``a``.

    ``omega`` is the (cols x k) Gaussian sketch.  Returns ``(u_r, s_r, tail)``
    in float32 (the caller casts ``u_r`` to the input dtype, svd.py:507-510).
    """
    a = a.astype(np.float32)
    rows, cols = a.shape
    rank = max(1, min(int(rank), min(rows, cols)))
    y = a @ omega.astype(np.float32)
    for _ in range(n_power):
        y = a @ (a.T @ y)
    q, _ = np.linalg.qr(y, mode="reduced")
    b = q.T @ a
    u_b, s_b, _ = np.linalg.svd(b, full_matrices=False)
    u = q @ u_b
    rank = min(rank, s_b.shape[0])
    u_r = np.ascontiguousarray(u[:, :rank]).astype(np.float32)
    s_r = s_b[:rank].astype(np.float32)
    a_fro_sq = float(np.sum(a.astype(np.float64) ** 2))
    retained = float(np.sum(s_r.astype(np.float64) ** 2))
    tail = max(0.0, 1.0 - retained / a_fro_sq) if a_fro_sq > 0 else 0.0
    return u_r, s_r, tail


def exact_svd(a: np.ndarray, rank: int):
    """``SVD.exact`` (svd.py:181-219) and ``tail_mass`` (svd.py:98-110)."""
    a = a.astype(np.float32)
    max_rank = min(a.shape)
    rank = max(1, min(int(rank), max_rank))
    u, s, _ = np.linalg.svd(a, full_matrices=False)
    if rank >= max_rank:
        tail = 0.0
    else:
        s64 = s.astype(np.float64)
        total = float(np.sum(s64 * s64))
        tail = float(np.sum(s64[rank:] ** 2)) / total if total > 0 else 0.0
    return np.ascontiguousarray(u[:, :rank]).astype(np.float32), s[:rank].astype(np.float32), tail


# ---------------------------------------------------------------------------
# Tucker -- tucker.py
# ---------------------------------------------------------------------------


def partial_tucker(x: np.ndarray, dt: str, r_token: int, r_feature: int, svd_fn):
    """``partial_tucker_st_hosvd`` (tucker.py:192-279).

    ``svd_fn(a, rank, mode)`` returns ``(u_r, s_r, tail)`` for the float32
    unfolding ``a``; ``mode`` is 'feature' or 'token'.  Bases are rounded to
    ``dt`` as the reference's SVD does on its way out (svd.py:417-421,
    507-510); the two einsums round their outputs to ``dt``.
    """
    m, t, d = x.shape
    rt = max(1, min(int(r_token), t))
    rd = max(1, min(int(r_feature), d))
    feat = np.moveaxis(x, 2, 0).reshape(d, m * t)  # tucker.py:244, mode_n_unfold 99-121
    u_d, _, tail_f = svd_fn(feat, rd, "feature")
    u_d = round_to(u_d, dt)
    x_proj = matmul_round(x.reshape(m * t, d), u_d, dt).reshape(m, t, -1)  # tucker.py:251
    tok = np.moveaxis(x_proj, 1, 0).reshape(t, -1)  # tucker.py:254
    u_t, _, tail_t = svd_fn(tok, rt, "token")
    u_t = round_to(u_t, dt)
    # core[m, n, r] = sum_t x_proj[m, t, r] u_t[t, n]  (tucker.py:261)
    core = round_to(np.einsum("mtr,tn->mnr", x_proj, u_t, dtype=np.float32), dt)
    return dict(u_feature=u_d, x_proj=x_proj, u_token=u_t, core=core,
                tail_feature_mass=tail_f, tail_token_mass=tail_t)


def reconstruct_tucker(core, u_token, u_feature, dt: str) -> np.ndarray:
    """``reconstruct_partial_tucker`` (tucker.py:159-189).

    torch.einsum("mar,ta,dr->mtd") contracts left to right (opt_einsum is
    absent): first over the token rank ``a``, rounding the (m, t, r)
    intermediate to ``dt``, then over the feature rank ``r``.
    """
    tmp = round_to(np.einsum("mar,ta->mtr", core, u_token, dtype=np.float32), dt)
    m, t, rd = tmp.shape
    out = matmul_round(tmp.reshape(m * t, rd), u_feature.T, dt)
    return out.reshape(m, t, -1)


# ---------------------------------------------------------------------------
# Quantisation -- quantization.py
# ---------------------------------------------------------------------------


def _qrange(bits: int, symmetric: bool):
    """IntQuantizer.__post_init__ (quantization.py:300-309)."""
    if bits not in (2, 4, 8):
        raise ValueError(bits)
    if symmetric:
        return -(1 << (bits - 1)), (1 << (bits - 1)) - 1
    return 0, (1 << bits) - 1


def quant_params(x: np.ndarray, dt: str, bits: int, symmetric=True, per_channel=True,
                 group_size=None):
    """``IntQuantizer.compute_params`` (quantization.py:410-452).

    ``x`` is (n, d) holding ``dt`` values; statistics are computed in ``dt``
    arithmetic and the scale is returned as float32, zero point as int32.
    """
    qmin, qmax = _qrange(bits, symmetric)
    if per_channel:
        xf = x.reshape(-1, x.shape[-1])
        x_min, x_max = xf.min(axis=0), xf.max(axis=0)
    elif group_size is not None:
        last = x.shape[-1]
        if last % group_size != 0:
            raise ValueError(f"last dim {last} not divisible by group_size {group_size}")
        xg = x.reshape(*x.shape[:-1], last // group_size, group_size)
        x_min, x_max = xg.min(axis=-1), xg.max(axis=-1)
    else:
        x_min, x_max = np.float32(x.min()), np.float32(x.max())
    x_min = np.asarray(x_min, np.float32)
    x_max = np.asarray(x_max, np.float32)
    eps = round_to(np.float32(1e-12), dt)
    if symmetric:
        abs_max = np.maximum(np.abs(x_min), np.abs(x_max))
        abs_max = np.maximum(abs_max, eps)
        scale = dt_op(lambda a: a / np.float32(qmax), dt, abs_max)
        zp = np.zeros(np.shape(scale), dtype=np.int32)
    else:
        rng = np.maximum(dt_op(lambda a, b: a - b, dt, x_max, x_min), eps)
        scale = dt_op(lambda a: a / np.float32(qmax - qmin), dt, rng)
        ratio = dt_op(lambda a, b: a / b, dt, x_min, scale)
        zp_f = dt_op(lambda a: np.float32(qmin) - a, dt, ratio)
        zp = np.rint(zp_f).astype(np.int32)
    return np.asarray(scale, np.float32), np.asarray(zp, np.int32)


def quantize_codes(x: np.ndarray, dt: str, scale, zp, bits: int, symmetric=True,
                   group_size=None) -> np.ndarray:
    """Scale, round-half-even and clamp: ``IntQuantizer.quantize``
    (quantization.py:340-357).  Returns int32 codes in ``[qmin, qmax]``.

    A 0-dim scale does not promote a bf16/fp16 ``x`` (torch's zero-dim type
    promotion), so that branch divides and adds in ``dt`` arithmetic.
    """
    qmin, qmax = _qrange(bits, symmetric)
    scale = np.asarray(scale, np.float32)
    zp = np.asarray(zp, np.int32)
    with np.errstate(all="ignore"):
        if scale.ndim == 0:
            scaled = dt_op(lambda a, s: a / s, dt, x, scale)
            scaled = dt_op(lambda a, z: a + z, dt, scaled, zp.astype(np.float32))
        elif group_size is not None:
            last = x.shape[-1]
            ng = last // group_size
            xg = x.reshape(*x.shape[:-1], ng, group_size)
            scaled = (xg / scale[..., None] + zp[..., None].astype(np.float32)).reshape(x.shape)
        else:
            scaled = x / scale + zp.astype(np.float32)
        q = np.clip(np.rint(scaled), qmin, qmax)
    return q.astype(np.int32)


def pack_codes(q: np.ndarray, bits: int, symmetric=True) -> np.ndarray:
    """``bit_packing_signed`` after the int8 cast (quantization.py:357-361, 181-238).

    8-bit: ``(q + offset) mod 256``; 4-bit: first element in the high
    nibble; 2-bit: first element in bits 7..6.  The last axis is
    zero-padded to a whole byte.
    """
    offset = (1 << (bits - 1)) if symmetric else 0
    u = ((q.astype(np.int64) + offset) & 0xFF).astype(np.uint8)
    if bits == 8:
        return u
    per = 8 // bits
    last = u.shape[-1]
    pad = (-last) % per
    if pad:
        u = np.concatenate([u, np.zeros(u.shape[:-1] + (pad,), np.uint8)], axis=-1)
    u = u.reshape(*u.shape[:-1], -1, per).astype(np.uint16)
    out = np.zeros(u.shape[:-1], np.uint16)
    for j in range(per):
        out |= (u[..., j] & ((1 << bits) - 1)) << (bits * (per - 1 - j))
    return out.astype(np.uint8)


def unpack_codes(packed: np.ndarray, bits: int, original_last: int, symmetric=True) -> np.ndarray:
    """``bit_unpacking_signed`` (quantization.py:241-275) -> int32 codes."""
    offset = (1 << (bits - 1)) if symmetric else 0
    p = packed.astype(np.int32)
    if bits == 8:
        return p - offset
    per = 8 // bits
    parts = [(p >> (bits * (per - 1 - j))) & ((1 << bits) - 1) for j in range(per)]
    flat = np.stack(parts, axis=-1).reshape(*packed.shape[:-1], -1)[..., :original_last]
    return flat - offset


def dequantize(q: np.ndarray, scale, zp, group_size=None) -> np.ndarray:
    """``IntQuantizer.dequantize`` (quantization.py:365-408) in float32."""
    scale = np.asarray(scale, np.float32)
    zp = np.asarray(zp, np.int32)
    if scale.ndim == 0:
        return ((q - zp).astype(np.float32) * scale).astype(np.float32)
    if group_size is not None:
        last = q.shape[-1]
        ng = last // group_size
        qg = q.reshape(*q.shape[:-1], ng, group_size)
        out = (qg - zp[..., None]).astype(np.float32) * scale[..., None]
        return out.reshape(q.shape).astype(np.float32)
    return ((q - zp).astype(np.float32) * scale).astype(np.float32)


def fp8_e4m3fn_round(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn -> float32 as ``Tensor.to(float8_e4m3fn)``.

    Round to nearest even on the 3-bit mantissa (subnormal step 2^-9);
    magnitudes that round above 448 become NaN (the format has no
    infinity and torch's cast does not saturate: identity.py:68-89 with
    dispatch.py:106-110).
    """
    x = np.asarray(x, np.float32).astype(np.float64)
    ax = np.abs(x)
    nan = ~np.isfinite(x)
    ax = np.where(nan, 1.0, ax)
    # exponent of each value, clamped to the subnormal range
    e = np.floor(np.log2(np.where(ax > 0, ax, 1.0)))
    e = np.maximum(e, -6.0)
    step = np.power(2.0, e - 3.0)
    q = np.round(ax / step) * step  # numpy rounds half to even
    q = np.where(q > 448.0, np.nan, q)
    out = np.copysign(q, x)
    out[nan] = np.nan
    return out.astype(np.float32)


# ---------------------------------------------------------------------------
# JoLT cell -- jolt.py / flashjolt.py / residual.py
# ---------------------------------------------------------------------------


def jolt_compress_cell(
    x: np.ndarray,
    dt: str,
    alloc,
    *,
    proj: np.ndarray,
    svd_mode: str,
    cap=None,
    omega_fn: Callable[[int, int], np.ndarray] | None = None,
    oversampling: int = 10,
    n_power: int = 2,
    symmetric: bool = True,
    per_channel: bool = True,
    group_size=None,
):
    """One cell of ``JoLTCompressor.compress_cell`` (jolt.py:273-329) or
    ``FlashJoLTCompressor.compress_cell`` (flashjolt.py:102-169), then the
    payload arrays of ``build_payload`` (jolt.py:331-399).

    ``svd_mode``: 'exact' (JoLT default, jolt.py:134), 'randomised' with
    ``cap`` (FlashJoLT's CapWrapper, flashjolt.py:172-210).
    """
    rt, rd, bits = int(alloc[0]), int(alloc[1]), int(alloc[2])
    m, t, d = x.shape

    def svd_fn(a, rank, mode):
        if svd_mode == "exact":
            return exact_svd(a, rank)
        _, k = sketch_width(a.shape[0], a.shape[1], rank, oversampling, cap)
        om = omega_fn(a.shape[1], k)
        return randomised_svd(a, rank, om, n_power)

    tk = partial_tucker(x, dt, rt, rd, svd_fn)
    recon = reconstruct_tucker(tk["core"], tk["u_token"], tk["u_feature"], dt)
    residual = dt_op(lambda a, b: a - b, dt, x, recon)  # jolt.py:311 / flashjolt.py:150
    out = dict(tk)
    out.update(recon=recon, residual=residual, bits=bits)
    if bits == 0:  # residual.py:183-198
        out.update(rotated=None, scale=np.zeros(0, np.float32), zero_point=np.zeros(0, np.int32),
                   packed=np.zeros(0, np.uint8))
        return out
    flat = residual.reshape(m * t, d).astype(np.float32)  # residual.py:201-204
    rotated = (flat @ proj.T.astype(np.float32)).astype(np.float32)  # residual.py:216
    if per_channel and group_size not in (None, 1):
        # quantization.py:338-346 broadcasts a (d,) scale against a
        # (n, d/g, g) view, which torch rejects.
        raise RuntimeError("per-channel scales cannot be combined with group_size > 1")
    scale, zp = quant_params(rotated, "f32", bits, symmetric, per_channel, group_size)
    q = quantize_codes(rotated, "f32", scale, zp, bits, symmetric,
                       group_size if not per_channel else None)
    out.update(rotated=rotated, scale=scale, zero_point=zp, codes=q,
               packed=pack_codes(q, bits, symmetric))
    return out


def jolt_decompress_cell(core16, u_token16, u_feature16, packed, scale, zp, bits, proj,
                         out_dt: str, shape, *, symmetric=True, group_size=None):
    """``JoLTCompressor.reconstruct_payload`` (jolt.py:401-463) with
    ``decode_residual`` (residual.py:242-288).

    Factors arrive as float16 values; the Tucker product and the residual
    decode run in float32; the sum is rounded to ``out_dt``.
    """
    m, t, d = shape
    x = reconstruct_tucker(core16.astype(np.float32), u_token16.astype(np.float32),
                           u_feature16.astype(np.float32), "f32")
    if bits > 0 and packed.size > 0:
        q = unpack_codes(packed, bits, d, symmetric)
        rot = dequantize(q, scale, zp, group_size)
        flat = (rot @ proj.astype(np.float32)).astype(np.float32)  # residual.py:287
        x = (x + flat.reshape(m, t, d)).astype(np.float32)
    return round_to(x, out_dt)
