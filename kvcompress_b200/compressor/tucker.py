"""Partial Tucker ST-HOSVD on sm_100a (API of kvcompress/compressor/tucker.py).

``partial_tucker_st_hosvd`` runs the feature mode then the token mode of
one ``(m, T, d)`` tensor through the Gram / sketch-solve / projection
kernels (:func:`kvcompress_b200.compressor.cells.tucker_cells`); bases and
core come back in the input dtype, rounded where the reference rounds.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from kvcompress_b200 import ops
from kvcompress_b200.compressor.cells import tucker_cells
from kvcompress_b200.compressor.svd import SVD

__all__ = ["TuckerFactors", "mode_n_fold", "mode_n_unfold", "partial_tucker_st_hosvd",
           "reconstruct_partial_tucker"]


@dataclass
class TuckerFactors:
    """``X ~ core x_2 U_T x_3 U_d`` (tucker.py:41-96)."""

    core: torch.Tensor
    u_token: torch.Tensor
    u_feature: torch.Tensor
    token_sv: torch.Tensor
    feature_sv: torch.Tensor
    token_tail_mass: float
    feature_tail_mass: float

    @property
    def r_token(self) -> int:
        return int(self.u_token.shape[1])

    @property
    def r_feature(self) -> int:
        return int(self.u_feature.shape[1])

    @property
    def bytes_factors(self) -> int:
        return int(self.core.numel() + self.u_token.numel() + self.u_feature.numel()) * 2


def mode_n_unfold(x: torch.Tensor, mode: int) -> torch.Tensor:
    """Mode-``mode`` unfolding of a 3-D tensor (tucker.py:99-121)."""
    if x.dim() != 3:
        raise ValueError(f"mode_n_unfold expects a 3-D tensor, got {tuple(x.shape)}")
    return torch.moveaxis(x, mode, 0).reshape(x.shape[mode], -1)


def mode_n_fold(mat: torch.Tensor, mode: int, shape: tuple[int, int, int]) -> torch.Tensor:
    """Inverse of :func:`mode_n_unfold` (tucker.py:124-156)."""
    if len(shape) != 3:
        raise ValueError(f"shape must have 3 dims, got {shape}")
    order = [(0, 1, 2), (1, 0, 2), (2, 0, 1)][mode]
    full = mat.reshape(*(shape[i] for i in order))
    return torch.moveaxis(full, 0, mode).contiguous()


def partial_tucker_st_hosvd(x: torch.Tensor, *, r_token: int | None = None, r_feature: int | None = None,
                            svd: SVD | None = None, cap: int | None = None,
                            forced_randomised: bool = False) -> TuckerFactors:
    """ST-HOSVD with the head mode pinned: feature mode first, then token mode."""
    if x.dim() != 3:
        raise ValueError(f"x must be 3-D, got {tuple(x.shape)}")
    m, t, d = x.shape
    rt = t if r_token is None else max(1, min(int(r_token), t))
    rd = d if r_feature is None else max(1, min(int(r_feature), d))
    core, ut, ud, tail_t, tail_f = tucker_cells([x.contiguous()], r_token=rt, r_feature=rd,
                                                svd=svd or SVD(), cap=cap,
                                                forced_randomised=forced_randomised)
    tails = torch.stack([tail_t[0], tail_f[0]]).cpu().tolist()
    return TuckerFactors(core=core[0], u_token=ut[0], u_feature=ud[0], token_sv=torch.empty(0),
                         feature_sv=torch.empty(0), token_tail_mass=float(tails[0]),
                         feature_tail_mass=float(tails[1]))


def reconstruct_partial_tucker(factors: TuckerFactors, target_shape) -> torch.Tensor:
    """``einsum("mar,ta,dr->mtd")`` in float32 (the decompress-side product of
    jolt.py:424-438), cast to the factors' dtype."""
    m, t, d = (int(s) for s in target_shape)
    rt, rd = factors.r_token, factors.r_feature
    if tuple(factors.core.shape) != (m, rt, rd):
        raise ValueError(f"core shape {tuple(factors.core.shape)} != expected {(m, rt, rd)}")
    if tuple(factors.u_token.shape) != (t, rt):
        raise ValueError(f"u_token shape {tuple(factors.u_token.shape)} != expected {(t, rt)}")
    if tuple(factors.u_feature.shape) != (d, rd):
        raise ValueError(f"u_feature shape {tuple(factors.u_feature.shape)} != expected {(d, rd)}")
    f = ([factors.core.contiguous()], [factors.u_token.contiguous()], [factors.u_feature.contiguous()])
    return ops.decompress((m, t, d), factors.core.dtype, factors=f, device=factors.core.device)[0]
