"""kvc_decompress_noalloc: the workspace-free decode against kvc_decompress.

This file is collected last and builds all of its own state (payloads, kernel
policy), so it passes alone in a fresh process and after every other test.
"""

from __future__ import annotations

import pytest
import torch

from kvcompress_b200 import build_compressor, ops
from kvcompress_b200._native import KVC, lib, ptr_array
from kvcompress_b200.compressor.cells import scale_mode_of
from kvcompress_b200.compressor.jl import cached_projection
from kvcompress_b200.synthetic import WORKLOADS, make_kv_layer


def _decode_args(payloads):
    p0 = payloads[0]
    meta = p0.metadata
    m, t, d = (int(s) for s in p0.shape)
    dev = p0.data["core"].device
    factors = ([p.data["core"] for p in payloads], [p.data["u_token"] for p in payloads],
               [p.data["u_feature"] for p in payloads])
    bits = int(meta["bits"])
    proj = cached_projection(d, d, distribution=meta["residual_distribution"], seed=int(meta["residual_seed"]),
                             device=dev, dtype=torch.float32, sparsity=float(meta["residual_sparsity"])).matrix
    kw = dict(codes=[p.data["residual_packed"] for p in payloads],
              scales=[p.data["residual_scale"] for p in payloads],
              zps=[p.data["residual_zero_point"] for p in payloads], bits=bits,
              symmetric=bool(meta["residual_symmetric"]),
              scale_mode=scale_mode_of(bool(meta["residual_per_channel"]), meta.get("residual_group_size"), d),
              group_size=meta.get("residual_group_size"), proj=proj, factors=factors)
    return (m, t, d), p0.dtype, dev, kw


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [(0, 2, 4, 8), (0, 2, 4)])
def test_noalloc_decompress_matches_workspace_entry_point(bits):
    ops.set_kernel_policy(0)
    w = WORKLOADS["llama3-8b-kv-b1-t8192-bf16"]
    k, v = make_kv_layer(w, 3, tokens=2048)
    comp = build_compressor("flashjolt", compression_ratio=4.0, bits=bits)
    kp, vp = comp.compress(k.reshape(8, 2048, 128).cuda(), v.reshape(8, 2048, 128).cuda())
    shape, dt, dev, kw = _decode_args([kp, vp])
    ref = ops.decompress(shape, dt, device=dev, n_cells=2, **kw)
    for t0, t1 in ((0, None), (100, 612)):
        ref_r = ops.decompress(shape, dt, device=dev, t0=t0, t1=t1, n_cells=2, **kw)
        out = [torch.empty_like(r) for r in ref_r]
        for _ in range(2):  # two calls in a row reuse the same scratch
            out = [o.fill_(float("nan")) for o in out]
            ops.decompress_noalloc(shape, dt, t0=t0, t1=t1, out=out, **kw)
            torch.cuda.synchronize()
            for a, b in zip(out, ref_r):
                assert torch.isfinite(a.float()).all()
                assert (a.float() - b.float()).norm() <= 1e-3 * b.float().norm()
    assert ops.device_error() == 0
    # the full-range noalloc decode equals the public API's decode
    full = [torch.empty_like(r) for r in ref]
    ops.decompress_noalloc(shape, dt, out=full, **kw)
    kd, vd = comp.decompress(kp, vp)
    assert (full[0].float() - kd.float()).norm() <= 1e-3 * kd.float().norm()
    assert (full[1].float() - vd.float()).norm() <= 1e-3 * vd.float().norm()


def test_noalloc_rejects_decodes_above_the_fixed_scratch():
    """Host-side size check: returns KVC_ERR_WORKSPACE before touching the GPU."""
    L = lib()
    m, t, d, rd = 64, 32768, 128, 16  # 2M rows x 16 x 4 B of Tucker rows alone: far above 8 MiB
    assert L.kvc_decompress_workspace_bytes(2, m * t, d, rd) > KVC.NOALLOC_SCRATCH_BYTES
    z = ptr_array([0, 0])
    rc = L.kvc_decompress_noalloc(2, z, z, z, 8, 1, KVC.SCALE_CHANNEL, 0, z, z, z, KVC.F16, m, t, d, 1, rd,
                                  None, 0, t, KVC.BF16, z, None)
    assert rc == KVC.ERR_WORKSPACE
    assert b"above the fixed" in L.kvc_last_error()
