"""kvc_decompress_noalloc: the workspace-free decode against kvc_decompress.

Some callers cannot allocate device memory: a host runtime that binds the C
ABI directly (ctypes, cgo, JNI) without a device allocator of its own, or a
serving engine that reserves all device memory at start-up and allows no
allocation on its decode path.  kvc_decompress_noalloc decodes in a fixed
array inside the library instead of a caller workspace.

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


def _allocations() -> int:
    return int(torch.cuda.memory_stats().get("allocation.all.allocated", 0))


@pytest.mark.gpu
def test_noalloc_decompress_matches_workspace_entry_point():
    ops.set_kernel_policy(0)
    w = WORKLOADS["llama3-8b-kv-b1-t8192-bf16"]
    # two different payload sets: the second decode between two decodes of the
    # first overwrites the shared scratch, so a stale scratch would show
    sets = []
    for layer, bits in ((3, (0, 2, 4, 8)), (5, (0, 2, 4))):
        k, v = make_kv_layer(w, layer, tokens=2048)
        comp = build_compressor("flashjolt", compression_ratio=4.0, bits=bits)
        kp, vp = comp.compress(k.reshape(8, 2048, 128).cuda(), v.reshape(8, 2048, 128).cuda())
        sets.append((comp, kp, vp, _decode_args([kp, vp])))
    assert sets[0][1].metadata["bits"] != sets[1][1].metadata["bits"]
    for t0, t1 in ((0, None), (100, 612)):
        refs, outs = [], []
        for _, _, _, (shape, dt, dev, kw) in sets:
            refs.append(ops.decompress(shape, dt, device=dev, t0=t0, t1=t1, n_cells=2, **kw))
            outs.append([torch.empty_like(r) for r in refs[-1]])
        torch.cuda.synchronize()
        for which in (0, 1, 0, 1):  # two calls in a row on each set, interleaved
            shape, dt, dev, kw = sets[which][3]
            out = outs[which]
            for o in out:
                o.fill_(float("nan"))
            torch.cuda.synchronize()
            n_alloc = _allocations()
            ops.decompress_noalloc(shape, dt, t0=t0, t1=t1, out=out, **kw)
            torch.cuda.synchronize()
            assert _allocations() == n_alloc, "decompress_noalloc allocated device memory"
            for a, b in zip(out, refs[which]):
                assert torch.equal(a, b)
    assert ops.device_error() == 0
    # the full-range noalloc decode equals the public API's decode
    comp, kp, vp, (shape, dt, dev, kw) = sets[0]
    full = [torch.empty(shape, dtype=dt, device=dev) for _ in range(2)]
    ops.decompress_noalloc(shape, dt, out=full, **kw)
    kd, vd = comp.decompress(kp, vp)
    assert torch.equal(full[0], kd) and torch.equal(full[1], vd)


def test_noalloc_rejects_decodes_above_the_fixed_scratch():
    """Host-side size check: returns KVC_ERR_WORKSPACE before touching the GPU."""
    L = lib()
    m, t, d, rd = 64, 32768, 128, 16  # 2M rows x 16 x 4 B of Tucker rows alone: far above 8 MiB
    assert L.kvc_decompress_workspace_bytes(2, m * t, d, rd) > KVC.NOALLOC_SCRATCH_BYTES
    z = ptr_array([0, 0])
    # a tensor-core layout (bf16 out, d = 128, 8-bit symmetric per-channel, a
    # rotation): the pointer stands for a JL matrix and is never dereferenced
    fake_proj = 256
    rc = L.kvc_decompress_noalloc(2, z, z, z, 8, 1, KVC.SCALE_CHANNEL, 0, z, z, z, KVC.F16, m, t, d, 1, rd,
                                  fake_proj, 0, t, KVC.BF16, z, None)
    assert rc == KVC.ERR_WORKSPACE
    assert b"above the fixed" in L.kvc_last_error()


def test_noalloc_size_limit_only_for_the_tensor_core_layouts():
    """A layout the SIMT decoder handles (float32 output) needs no scratch, so
    its size is not checked: the call gets past the gate and fails only on its
    NULL pointers (kvc_decompress's argument check, before any launch; without
    a GPU, at the device query)."""
    L = lib()
    m, t, d, rd = 64, 32768, 128, 16
    z = ptr_array([0, 0])
    rc = L.kvc_decompress_noalloc(2, z, z, z, 8, 1, KVC.SCALE_CHANNEL, 0, z, z, z, KVC.F16, m, t, d, 1, rd,
                                  256, 0, t, KVC.F32, z, None)
    assert rc != KVC.ERR_WORKSPACE
    assert rc in (KVC.ERR_ARG, -6)
