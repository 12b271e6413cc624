"""The per-cell SVD solver (kvc_sketch_solve) against numpy in fp64.

SVD.randomise (kvcompress/compressor/svd.py:221-316) and SVD.exact
(svd.py:181-219) reach the solver only through a Gram matrix: the checks
restate the same algorithm with numpy's QR and eigh on the same Gram and
sketch, and compare Ritz values, tail masses and the spanned subspaces.
The shapes cover every kernel: the shared-memory randomised solver
(p <= 128, k <= 32), the shared-memory exact solver (p <= 128) and the
general solver (larger p or k), and degenerate spectra.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from kvcompress_b200 import ops
from kvcompress_b200._native import KVC

pytestmark = pytest.mark.gpu


def _matrix(n: int, p: int, seed: int, decay: float = 3.0, rank: int | None = None) -> np.ndarray:
    """A (n x p) with singular values spread over ``decay`` decades (or of rank ``rank``)."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((n, p))
    if rank is not None:
        a = rng.standard_normal((n, rank)) @ rng.standard_normal((rank, p))
        return a
    return a * np.logspace(0, -decay, p)[None, :]


def _orth(y: np.ndarray, m: np.ndarray | None = None) -> np.ndarray:
    """Orthonormal basis of range(y) in the inner product of m (identity when None)."""
    g = y.T @ (y if m is None else m @ y)
    r = np.linalg.cholesky(g).T
    return y @ np.linalg.inv(r)


def _projector(u: np.ndarray, m: np.ndarray | None = None) -> np.ndarray:
    return u @ u.T if m is None else u @ u.T


def _rel(a, b) -> float:
    return float(np.linalg.norm(np.asarray(a) - np.asarray(b)) / max(np.linalg.norm(np.asarray(b)), 1e-300))


def _left_randomised(a: np.ndarray, om: np.ndarray, k: int, rank: int, n_power: int = 2):
    """Feature-mode reference: A^T (n x p) is the unfolding, G = A^T A."""
    G = a.T @ a
    q = _orth(a.T @ om)
    for _ in range(n_power):
        q = _orth(G @ q)
    c = q.T @ G @ q
    w, v = np.linalg.eigh(c)
    w, v = w[::-1], v[:, ::-1]
    return G, q @ v[:, :rank], w[:rank], max(0.0, 1.0 - w[:rank].sum() / np.sum(a * a))


def _right_randomised(a: np.ndarray, om: np.ndarray, rank: int, n_power: int = 2):
    """Token-mode reference: A (n x p), H = A^T A, sketches A w orthonormalised in H."""
    H = a.T @ a
    w_ = _orth(om, H)
    for _ in range(n_power):
        w_ = _orth(H @ w_, H)
    hw = H @ w_
    c = hw.T @ hw
    ev, v = np.linalg.eigh(c)
    ev, v = ev[::-1], v[:, ::-1]
    u = a @ (w_ @ v[:, :rank])
    return H, u, ev[:rank], max(0.0, 1.0 - ev[:rank].sum() / np.trace(H))


@pytest.mark.parametrize("n,p,k,rank", [(4000, 128, 11, 1), (4000, 128, 26, 16), (3000, 64, 32, 22),
                                        (4000, 128, 74, 64), (3000, 128, 128, 100)])
def test_randomised_left(n, p, k, rank):
    a = _matrix(n, p, seed=p + k)
    rng = np.random.default_rng(k)
    om = rng.standard_normal((n, k)).astype(np.float32)
    G, u_ref, w_ref, tail_ref = _left_randomised(a, om.astype(np.float64), k, rank)
    y0 = a.T @ om.astype(np.float64)
    gram = np.concatenate([G.ravel(), y0.ravel(), [np.sum(a * a)]])
    g = torch.from_numpy(np.stack([gram, gram]))
    basis, tail, sv2 = ops.sketch_solve(g.cuda(), mode=KVC.SVD_RANDOMISED, side=KVC.SIDE_LEFT, p=p, n_other=n, k=k,
                                        rank=rank, n_power=2, omega=None, basis_dtype=torch.float32)
    for c in range(2):
        u = basis[c].double().cpu().numpy()
        assert _rel(sv2[c].cpu().numpy(), w_ref) < 1e-9
        assert abs(tail[c].item() - tail_ref) < 1e-9
        assert _rel(u @ u.T, u_ref @ u_ref.T) < 2e-6  # the basis is stored in float32
        assert np.abs(u.T @ u - np.eye(rank)).max() < 1e-5
    np.testing.assert_array_equal(basis[0].cpu().numpy(), basis[1].cpu().numpy())


@pytest.mark.parametrize("n,p,k,rank", [(8192, 8, 8, 1), (32768, 64, 11, 1), (4096, 256, 74, 64),
                                        (2048, 200, 37, 27), (4096, 1024, 513, 512)])
def test_randomised_right(n, p, k, rank):
    a = _matrix(n, p, seed=7 * p + k, decay=2.0)
    rng = np.random.default_rng(p)
    om = rng.standard_normal((p, k)).astype(np.float32)
    H, u_ref, w_ref, tail_ref = _right_randomised(a, om.astype(np.float64), rank)
    gram = torch.from_numpy(np.concatenate([H.ravel(), [np.trace(H)]])[None]).cuda()
    m, tail, sv2 = ops.sketch_solve(gram, mode=KVC.SVD_RANDOMISED, side=KVC.SIDE_RIGHT, p=p, n_other=n, k=k,
                                    rank=rank, n_power=2, omega=torch.from_numpy(om).cuda(),
                                    basis_dtype=torch.float64)
    u = a @ m[0].cpu().numpy()
    assert _rel(sv2[0].cpu().numpy(), w_ref) < 1e-9
    assert abs(tail[0].item() - tail_ref) < 1e-9
    assert _rel(u @ u.T, u_ref @ u_ref.T) < 1e-8
    assert np.abs(u.T @ u - np.eye(rank)).max() < 1e-8


@pytest.mark.parametrize("n,p,k,rank", [(4096, 1024, 513, 512), (4096, 1024, 513, 503), (3000, 300, 150, 150),
                                        (5000, 700, 300, 290), (3000, 300, 150, 134), (4096, 1024, 700, 696),
                                        (4096, 1024, 700, 692)])
def test_randomised_right_complement(n, p, k, rank):
    """Wide sketches without singular values (every compress call): the basis
    spans the top-rank Ritz subspace (columns not ordered) and the tail mass
    matches.  The trailing Ritz vectors come from a fixed number of block
    inverse-iteration steps: the tail and the energy the basis captures
    match to 1e-8 of |A|^2; the subspace itself to 1e-2 (projector, relative
    Frobenius): what is left mixed are trailing directions of nearly equal
    Ritz values, which the reference's own fp32 SVD of Q^T A does not
    resolve any better."""
    a = _matrix(n, p, seed=3 * p + k, decay=2.0)
    rng = np.random.default_rng(p + 1)
    om = rng.standard_normal((p, k)).astype(np.float32)
    H, u_ref, w_ref, tail_ref = _right_randomised(a, om.astype(np.float64), rank)
    gram = torch.from_numpy(np.concatenate([H.ravel(), [np.trace(H)]])[None]).cuda()
    m, tail, sv2 = ops.sketch_solve(gram, mode=KVC.SVD_RANDOMISED, side=KVC.SIDE_RIGHT, p=p, n_other=n, k=k,
                                    rank=rank, n_power=2, omega=torch.from_numpy(om).cuda(),
                                    basis_dtype=torch.float64, want_sv2=False)
    assert sv2 is None
    u = a @ m[0].cpu().numpy()
    assert abs(tail[0].item() - tail_ref) < 1e-8
    assert np.abs(u.T @ u - np.eye(rank)).max() < 1e-8
    assert _rel(u @ u.T, u_ref @ u_ref.T) < 1e-2
    # energy captured by the basis = 1 - tail (A's own columns)
    captured = np.sum((u.T @ a) ** 2) / np.sum(a * a)
    assert abs((1.0 - captured) - tail_ref) < 1e-8


@pytest.mark.parametrize("p,rank,side", [(64, 1, KVC.SIDE_LEFT), (64, 32, KVC.SIDE_LEFT), (128, 1, KVC.SIDE_LEFT),
                                         (128, 64, KVC.SIDE_LEFT), (128, 128, KVC.SIDE_LEFT),
                                         (96, 48, KVC.SIDE_RIGHT), (200, 100, KVC.SIDE_LEFT),
                                         (256, 17, KVC.SIDE_RIGHT)])
def test_exact(p, rank, side):
    a = _matrix(4 * p, p, seed=p * 3 + rank, decay=2.0)
    G = a.T @ a
    gram = torch.from_numpy(np.concatenate([G.ravel(), [np.trace(G)]])[None]).cuda()
    basis, tail, sv2 = ops.sketch_solve(gram, mode=KVC.SVD_EXACT, side=side, p=p, n_other=4 * p, k=0, rank=rank,
                                        n_power=2, omega=None,
                                        basis_dtype=torch.float32 if side == KVC.SIDE_LEFT else torch.float64)
    w, v = np.linalg.eigh(G)
    w, v = w[::-1], v[:, ::-1]
    assert _rel(sv2[0].cpu().numpy(), w[:rank]) < 1e-10
    want_tail = 0.0 if rank >= p else w[rank:].sum() / w.sum()
    assert abs(tail[0].item() - want_tail) < 1e-10
    b = basis[0].double().cpu().numpy()
    if side == KVC.SIDE_LEFT:
        assert _rel(b @ b.T, v[:, :rank] @ v[:, :rank].T) < 2e-6
    else:
        u = a @ b
        ue = a @ v[:, :rank]
        ue = ue / np.linalg.norm(ue, axis=0)
        assert np.abs(u.T @ u - np.eye(rank)).max() < 1e-8
        assert _rel(u @ u.T, ue @ ue.T) < 1e-8


@pytest.mark.parametrize("p,mode", [(40, KVC.SVD_EXACT), (160, KVC.SVD_EXACT), (48, KVC.SVD_RANDOMISED)])
def test_degenerate_spectra(p, mode):
    """Equal eigenvalues (a multiple of the identity) and a rank-deficient Gram:
    the basis is still orthonormal, the values and tails exact."""
    rank = p // 2
    k = min(p, rank + 10) if mode == KVC.SVD_RANDOMISED else 0
    rng = np.random.default_rng(p)
    om = torch.from_numpy(rng.standard_normal((p, max(k, 1))).astype(np.float32)).cuda()
    for G, want in ((np.eye(p) * 2.5, np.full(rank, 2.5)), ):
        gram = torch.from_numpy(np.concatenate([G.ravel(), [np.trace(G)]])[None]).cuda()
        m, tail, sv2 = ops.sketch_solve(gram, mode=mode, side=KVC.SIDE_RIGHT, p=p, n_other=10 * p, k=k, rank=rank,
                                        n_power=2, omega=om if mode == KVC.SVD_RANDOMISED else None,
                                        basis_dtype=torch.float64)
        mm = m[0].cpu().numpy()
        # A with A^T A = G: U = A M has orthonormal columns
        a = np.linalg.cholesky(G).T
        u = a @ mm
        assert np.abs(u.T @ u - np.eye(rank)).max() < 1e-8
        np.testing.assert_allclose(sv2[0].cpu().numpy(), want, rtol=1e-12)
        assert abs(tail[0].item() - 0.5) < 1e-12
    # rank-deficient: 5 nonzero eigenvalues, rank 3 of them wanted
    a = _matrix(6 * p, p, seed=11, rank=5)
    G = a.T @ a
    w = np.linalg.eigvalsh(G)[::-1]
    gram = torch.from_numpy(np.concatenate([G.ravel(), [np.trace(G)]])[None]).cuda()
    kk = min(p, 13) if mode == KVC.SVD_RANDOMISED else 0
    om = torch.from_numpy(rng.standard_normal((p, max(kk, 1))).astype(np.float32)).cuda()
    m, tail, sv2 = ops.sketch_solve(gram, mode=mode, side=KVC.SIDE_RIGHT, p=p, n_other=6 * p, k=kk, rank=3,
                                    n_power=2, omega=om if mode == KVC.SVD_RANDOMISED else None,
                                    basis_dtype=torch.float64)
    assert _rel(sv2[0].cpu().numpy(), w[:3]) < 1e-9
    assert abs(tail[0].item() - w[3:5].sum() / w.sum()) < 1e-9
    u = a @ m[0].cpu().numpy()
    assert np.abs(u.T @ u - np.eye(3)).max() < 1e-8
