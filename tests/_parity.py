"""Helpers shared by the GPU parity tests (the oracle is the checker)."""

from __future__ import annotations

import numpy as np
import torch

import oracle
import oracle.jolt as _oj

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
NP_DT = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def rel(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))


def cuda_omega(n: int, k: int, seed: int = 0) -> np.ndarray:
    """The sketch the reference draws on a CUDA device (svd.py:259-260)."""
    torch.manual_seed(seed)
    return torch.randn(n, k, dtype=torch.float32, device="cuda").cpu().numpy()


def to_cuda(a: np.ndarray, dt: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to("cuda").to(TORCH_DT[dt])


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def oracle_jolt(x: np.ndarray, dt: str, alloc, *, method: str, cap, proj: np.ndarray, **kw):
    """Oracle compress + decompress of one cell with the CUDA sketches."""
    out = oracle.jolt_compress_cell(x, dt, alloc, proj=proj,
                                    svd_mode="randomised" if method == "flashjolt" else "exact",
                                    cap=cap, omega_fn=cuda_omega, **{k: v for k, v in kw.items()})
    m, t, d = x.shape
    gs = kw.get("group_size") if not kw.get("per_channel", True) else None
    dec = oracle.jolt_decompress_cell(
        out["core"].astype(np.float16), out["u_token"].astype(np.float16),
        out["u_feature"].astype(np.float16), out["packed"], out["scale"], out["zero_point"],
        out["bits"], proj, dt, (m, t, d), symmetric=kw.get("symmetric", True), group_size=gs)
    out["decompressed"] = dec
    return out


def projector(u: np.ndarray) -> np.ndarray:
    u = np.asarray(u, np.float64)
    return u @ u.T


def recon_rows(core, u_token, u_feature, dt: str, rows: np.ndarray, t: int) -> np.ndarray:
    """Rows ``rows`` of the (m*T, d) view of ``reconstruct_partial_tucker``
    (tucker.py:159-189), rounded as the reference rounds: the token-rank
    contraction in float32 rounded to ``dt``, then the feature rank."""
    core = np.asarray(core, np.float32)
    u_token = np.asarray(u_token, np.float32)
    u_feature = np.asarray(u_feature, np.float32)
    h, tt = rows // t, rows % t
    tmp = _oj.round_to(np.einsum("nar,na->nr", core[h], u_token[tt], dtype=np.float32), dt)
    return _oj.matmul_round(tmp, u_feature.T, dt)


def near_ties(x_rows, recon, dt: str, proj, scale, margin: float = 1e-3) -> np.ndarray:
    """Codes whose quantiser input lies within ``margin`` quantisation steps of
    a rounding boundary (symmetric scales, zero point 0): the fp32 rotation may
    round either way there.  The rotated residual is evaluated in float64 from
    the residual in the cell dtype (jolt.py:311, residual.py:201-216)."""
    resid = _oj.dt_op(lambda a, b: a - b, dt, np.asarray(x_rows, np.float32), recon)
    rot = np.asarray(resid, np.float64) @ np.asarray(proj, np.float64).T
    v = rot / np.asarray(scale, np.float64)
    return np.abs(v - np.floor(v) - 0.5) < margin


def assert_codes_match(got_packed, ref_packed, bits: int, d: int, ties: np.ndarray) -> float:
    """Every code away from a tie is identical; returns the fraction of the
    near-tie codes that differ (the flip rate)."""
    got = oracle.unpack_codes(np.asarray(got_packed), bits, d)
    ref = oracle.unpack_codes(np.asarray(ref_packed), bits, d)
    diff = got != ref
    bad = diff & ~ties
    assert not bad.any(), f"{int(bad.sum())} codes differ away from ties (first at {np.argwhere(bad)[0]})"
    return float(diff.sum()) / max(1, int(ties.sum()))
