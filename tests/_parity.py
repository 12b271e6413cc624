"""Helpers shared by the GPU parity tests (the oracle is the checker)."""

from __future__ import annotations

import numpy as np
import torch

import oracle

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
