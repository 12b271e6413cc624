"""Stage-level parity of the sm_100a kernels against the oracle / golden vectors.

Integer outputs (scales from the same values, codes, packed bytes, fp8
bytes) are compared bit for bit; floating-point stages with tolerances
written next to each assert.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from kvcompress_b200 import ops
from kvcompress_b200._native import KVC
from kvcompress_b200.compressor.quantization import dequantize_tensor, quantize_tensor

from _parity import assert_codes_match, f32, near_ties, recon_rows, rel, to_cuda

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case,bits", [("f32_flash_r1_b8", 8), ("bf16_flash_r1_b8", 8),
                                       ("f32_flash_r4_b4", 4), ("f16_flash_r2_b2", 2)])
def test_codes_bit_exact_given_reference_rotated(golden, case, bits):
    """Same fp32 rotated residual -> same scales and same packed codes, bit for bit."""
    rot = golden[case + "/rotated"]
    cell = torch.from_numpy(rot).cuda().view(1, *rot.shape)
    scales, zps = ops.residual_stats([cell], None, None, bits=bits, symmetric=True,
                                     scale_mode=KVC.SCALE_CHANNEL, stat_dtype=torch.float32)
    np.testing.assert_array_equal(scales[0].cpu().numpy(), golden[case + "/payload_residual_scale"])
    np.testing.assert_array_equal(zps[0].cpu().numpy(), golden[case + "/payload_residual_zero_point"])
    codes, _, _ = ops.residual_quant([cell], None, None, scales, zps, bits=bits, symmetric=True,
                                     scale_mode=KVC.SCALE_CHANNEL, group_size=None,
                                     stat_dtype=torch.float32, arith_dtype=torch.float32)
    np.testing.assert_array_equal(codes[0].cpu().numpy(), golden.raw(case + "/payload_residual_packed"))


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("symmetric", [True, False])
@pytest.mark.parametrize("mode", ["channel", "group", "tensor"])
def test_quantize_tensor_bit_exact(golden, bits, symmetric, mode):
    x = torch.from_numpy(golden["quant/x"]).cuda()
    tag = f"quant/b{bits}_{'sym' if symmetric else 'asym'}_{mode}/"
    kw = dict(symmetric=symmetric, per_channel=(mode == "channel"), group_size=(32 if mode == "group" else None))
    pay = quantize_tensor(x, dtype=f"int{bits}", **kw)
    np.testing.assert_array_equal(pay["q"].cpu().numpy(), golden[tag + "q"])
    np.testing.assert_array_equal(pay["scale"].cpu().numpy(), golden[tag + "scale"])
    np.testing.assert_array_equal(pay["zero_point"].cpu().numpy(), golden[tag + "zero_point"])
    deq = dequantize_tensor(pay, dtype=f"int{bits}", **kw)
    np.testing.assert_array_equal(deq.cpu().numpy(), golden[tag + "deq"])


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_quant_only_compressor_bit_exact(golden, bits):
    from kvcompress_b200 import build_compressor

    x = to_cuda(golden["intonly/x"], "bf16")
    comp = build_compressor(f"int{bits}")
    kp, vp = comp.compress(x, x)
    p = f"intonly{bits}/"
    np.testing.assert_array_equal(kp.data["q"].cpu().numpy(), golden[p + "q"])
    np.testing.assert_array_equal(kp.data["scale"].cpu().numpy(), golden[p + "scale"])
    np.testing.assert_array_equal(vp.data["q"].cpu().numpy(), golden[p + "q"])
    kd, _ = comp.decompress(kp, vp)
    assert kd.dtype == torch.bfloat16 and kd.shape == x.shape
    np.testing.assert_array_equal(f32(kd), golden[p + "decompressed"])
    assert kp.bytes_compressed == golden.meta[f"intonly{bits}"]["bytes"]


def test_fp8_cast_all_bf16_patterns(golden):
    allv = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).cuda()
    got = ops.cast(allv, torch.float8_e4m3fn).view(torch.uint8).cpu().numpy()
    np.testing.assert_array_equal(got, golden["fp8/all_bf16_bytes"])
    # every fp8 byte back to bf16 / fp32 as torch decodes it
    b = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn)
    for dt in (torch.bfloat16, torch.float32, torch.float16):
        ours = ops.cast(b.cuda(), dt).cpu()
        ref = b.to(dt)
        assert torch.equal(ours.isnan(), ref.isnan())
        ok = ~ref.isnan()
        assert torch.equal(ours[ok], ref[ok])


def test_fp8_compressor(golden):
    from kvcompress_b200 import build_compressor

    y = to_cuda(golden["fp8/x"], "bf16")
    comp = build_compressor("fp8")
    kp, vp = comp.compress(y, y)
    np.testing.assert_array_equal(kp.data["value"].view(torch.uint8).cpu().numpy(), golden["fp8/bytes"])
    kd, _ = comp.decompress(kp, vp)
    np.testing.assert_array_equal(np.isnan(f32(kd)), np.isnan(golden["fp8/decompressed"]))
    ok = ~np.isnan(golden["fp8/decompressed"])
    np.testing.assert_array_equal(f32(kd)[ok], golden["fp8/decompressed"][ok])


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_gram_matches_fp64(dt):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(3, 1000, 64, generator=g)
    om = torch.randn(3000, 7, generator=g)
    cells = [to_cuda(x.numpy(), dt).view(3000, 64), to_cuda((x * 2).numpy(), dt).view(3000, 64)]
    out = ops.gram(cells, om.cuda()).cpu().numpy()
    for i, c in enumerate(cells):
        a = c.float().cpu().numpy().astype(np.float64)
        G = a.T @ a
        Y = a.T @ om.numpy().astype(np.float64)
        o = out[i]
        # fp32 accumulation over 2048-row chunks, fp64 across chunks
        assert rel(o[:64 * 64].reshape(64, 64), G) < 2e-5
        assert rel(o[64 * 64:64 * 64 + 64 * 7].reshape(64, 7), Y) < 2e-5
        assert abs(o[-1] / np.sum(a * a) - 1) < 2e-5
    # bit-reproducible
    out2 = ops.gram(cells, om.cuda()).cpu().numpy()
    np.testing.assert_array_equal(out, out2)


@pytest.mark.parametrize("p,side", [(64, KVC.SIDE_LEFT), (128, KVC.SIDE_LEFT), (40, KVC.SIDE_RIGHT)])
def test_exact_solver_matches_numpy(p, side):
    g = torch.Generator().manual_seed(p)
    a = torch.randn(3 * p, p, generator=g, dtype=torch.float64) @ torch.diag(
        torch.linspace(3, 0.1, p, dtype=torch.float64))
    G = (a.T @ a).numpy()
    gram = torch.from_numpy(np.concatenate([G.ravel(), [np.trace(G)]])[None]).cuda()
    rank = 5
    basis, tail, sv2 = ops.sketch_solve(gram, mode=KVC.SVD_EXACT, side=side, p=p, n_other=3 * p, k=0,
                                        rank=rank, n_power=2, omega=None,
                                        basis_dtype=torch.float32 if side == KVC.SIDE_LEFT else torch.float64)
    w, v = np.linalg.eigh(G)
    w, v = w[::-1], v[:, ::-1]
    assert rel(sv2[0].cpu().numpy(), w[:rank]) < 1e-10
    assert abs(tail[0].item() - w[rank:].sum() / w.sum()) < 1e-10
    b = basis[0].double().cpu().numpy()
    if side == KVC.SIDE_LEFT:
        assert rel(b @ b.T, v[:, :rank] @ v[:, :rank].T) < 1e-5
    else:
        u = a.numpy() @ b  # U = A M has orthonormal columns
        assert rel(u.T @ u, np.eye(rank)) < 1e-8


def test_randomised_solver_full_sketch_is_exact():
    """With k = p the sketch spans everything: randomised == exact."""
    p = 24
    g = torch.Generator().manual_seed(1)
    a = torch.randn(200, p, generator=g, dtype=torch.float64)
    G = (a.T @ a).numpy()
    om = torch.randn(p, p, generator=g, dtype=torch.float32)
    gram = torch.from_numpy(np.concatenate([G.ravel(), [np.trace(G)]])[None]).cuda()
    m_r, t_r, s_r = ops.sketch_solve(gram, mode=KVC.SVD_RANDOMISED, side=KVC.SIDE_RIGHT, p=p, n_other=200,
                                     k=p, rank=3, n_power=2, omega=om.cuda(), basis_dtype=torch.float64)
    m_e, t_e, s_e = ops.sketch_solve(gram, mode=KVC.SVD_EXACT, side=KVC.SIDE_RIGHT, p=p, n_other=200,
                                     k=0, rank=3, n_power=2, omega=None, basis_dtype=torch.float64)
    assert rel(s_r.cpu().numpy(), s_e.cpu().numpy()) < 1e-10
    ur = a.numpy() @ m_r[0].cpu().numpy()
    ue = a.numpy() @ m_e[0].cpu().numpy()
    assert rel(ur @ ur.T, ue @ ue.T) < 1e-8


def test_decompress_reference_payloads(golden):
    """Fused decode of the reference's own payloads vs the oracle decode."""
    for case in ["f32_flash_r1_b8", "f32_flash_r4_b4", "bf16_flash_r1_b8", "bf16_flash_r128_b4",
                 "bf16_jolt_r8_b2", "f16_flash_r2_b2", "bf16_flash_r3_b0"]:
        meta = golden.meta[case]
        m, t, d = meta["shape"]
        bits = meta["alloc"][2]
        p = case + "/"
        proj = golden[f"jl/pi_d{d}_seed0"]
        ref = oracle.jolt_decompress_cell(
            golden.raw(p + "payload_core"), golden.raw(p + "payload_u_token"),
            golden.raw(p + "payload_u_feature"), golden.raw(p + "payload_residual_packed"),
            golden[p + "payload_residual_scale"], golden[p + "payload_residual_zero_point"], bits,
            proj, meta["dtype"], (m, t, d))
        dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[meta["dtype"]]
        fac = ([torch.from_numpy(golden.raw(p + "payload_core")).cuda()],
               [torch.from_numpy(golden.raw(p + "payload_u_token")).cuda()],
               [torch.from_numpy(golden.raw(p + "payload_u_feature")).cuda()])
        kw = {}
        if bits:
            kw = dict(codes=[torch.from_numpy(golden.raw(p + "payload_residual_packed")).cuda()],
                      scales=[torch.from_numpy(golden[p + "payload_residual_scale"]).cuda()],
                      zps=[torch.from_numpy(golden[p + "payload_residual_zero_point"]).cuda()],
                      bits=bits, proj=torch.from_numpy(proj).cuda())
        out = ops.decompress((m, t, d), dt, factors=fac, device="cuda", **kw)[0]
        got = f32(out)
        # fp32: summation order only; 16-bit: a few last-bit flips of the final cast
        assert rel(got, ref) < (1e-6 if dt == torch.float32 else 2e-3), case
        assert rel(got, golden[p + "decompressed"]) < (1e-5 if dt == torch.float32 else 4e-3), case


def test_residual_kernel_on_reference_factors(golden):
    """Scales and codes from the reference's own factors agree up to ties."""
    for case in ["bf16_flash_r1_b8", "f32_flash_r4_b4", "bf16_flash_r128_b4"]:
        meta = golden.meta[case]
        m, t, d = meta["shape"]
        bits = meta["alloc"][2]
        p = case + "/"
        dt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[meta["dtype"]]
        x = to_cuda(golden.case_input(case), meta["dtype"])
        fac = ([to_cuda(golden[p + "core"], meta["dtype"])], [to_cuda(golden[p + "u_token"], meta["dtype"])],
               [to_cuda(golden[p + "u_feature"], meta["dtype"])])
        proj = torch.from_numpy(golden[f"jl/pi_d{d}_seed0"]).cuda()
        scales, zps = ops.residual_stats([x], fac, proj, bits=bits, symmetric=True,
                                         scale_mode=KVC.SCALE_CHANNEL, stat_dtype=torch.float32)
        assert rel(scales[0].cpu().numpy(), golden[p + "payload_residual_scale"]) < 1e-5
        codes, _, _ = ops.residual_quant([x], fac, proj, scales, zps, bits=bits, symmetric=True,
                                         scale_mode=KVC.SCALE_CHANNEL, group_size=None,
                                         stat_dtype=torch.float32, arith_dtype=torch.float32)
        # every code more than 1e-3 quantisation steps from a rounding boundary
        # of the exact rotated residual equals the reference's
        rows = np.arange(m * t)
        recon = recon_rows(golden[p + "core"], golden[p + "u_token"], golden[p + "u_feature"], meta["dtype"], rows, t)
        ties = near_ties(golden.case_input(case).reshape(m * t, d), recon, meta["dtype"], golden[f"jl/pi_d{d}_seed0"],
                         golden[p + "payload_residual_scale"])
        flip = assert_codes_match(codes[0].cpu().numpy(), golden.raw(p + "payload_residual_packed"), bits, d, ties)
        print(f"{case}: {int(ties.sum())} near-tie codes, {flip:.3f} of them flipped")
        del dt


def _policy(p):
    ops.set_kernel_policy(p)


def _exact_codes(x, recon, proj, scale, bits, d):
    """Packed codes of the float64 rotated residual (the rounding away from ties)."""
    import oracle
    import oracle.jolt

    m, t, _ = x.shape
    resid = oracle.jolt.dt_op(lambda a, b: a - b, "bf16", f32(x).reshape(m * t, d), recon)
    rot = (np.asarray(resid, np.float64) @ proj.cpu().numpy().astype(np.float64).T)
    qmax = (1 << (bits - 1)) - 1
    q = np.clip(np.rint(rot / np.asarray(scale, np.float64)), -qmax - 1, qmax).astype(np.int32)
    return oracle.pack_codes(q, bits)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("bits", [8, 4, 2])
@pytest.mark.parametrize("rank", [(1, 1), (5, 3), (12, 6), (20, 16)])
def test_tensor_core_residual_matches_simt(d, bits, rank):
    """tcgen05 encode vs the SIMT encode of the same bf16 cells (two cells, ragged rows)."""
    from kvcompress_b200.compressor.jl import cached_projection

    g = torch.Generator(device="cuda").manual_seed(d + bits)
    m, t = 3, 333
    xs = [torch.randn(m, t, d, generator=g, device="cuda").bfloat16() for _ in range(2)]
    rt, rd = rank
    fac = ([torch.randn(m, rt, rd, generator=g, device="cuda").bfloat16() for _ in xs],
           [(torch.randn(t, rt, generator=g, device="cuda") / 10).bfloat16() for _ in xs],
           [(torch.randn(d, rd, generator=g, device="cuda") / 5).bfloat16() for _ in xs])
    proj = cached_projection(d, d, seed=0, device="cuda").matrix
    out = {}
    try:
        for pol in (0, 1):
            _policy(pol)
            sc, zp = ops.residual_stats(xs, fac, proj, bits=bits, symmetric=True, scale_mode=KVC.SCALE_CHANNEL,
                                        stat_dtype=torch.float32)
            codes, _, _ = ops.residual_quant(xs, fac, proj, sc, zp, bits=bits, symmetric=True,
                                             scale_mode=KVC.SCALE_CHANNEL, group_size=None,
                                             stat_dtype=torch.float32, arith_dtype=torch.float32)
            out[pol] = ([s.cpu().numpy() for s in sc], [c.cpu().numpy() for c in codes])
    finally:
        _policy(0)
    assert ops.device_error() == 0
    for a, b in zip(out[0][0], out[1][0]):
        assert rel(a, b) < 1e-6
    # every code more than 1e-3 quantisation steps from a rounding boundary of
    # the exact rotated residual is identical on both paths
    rows = np.arange(m * t)
    flips = []
    for i, x in enumerate(xs):
        cf = [f32(f[i]) for f in fac]
        recon = recon_rows(cf[0], cf[1], cf[2], "bf16", rows, t)
        ties = near_ties(f32(x).reshape(m * t, d), recon, "bf16", proj.cpu().numpy(), out[1][0][i], margin=1e-3)
        for pol in (0, 1):
            flips.append(assert_codes_match(out[pol][1][i], _exact_codes(x, recon, proj, out[1][0][i], bits, d),
                                            bits, d, ties))
    print(f"near-tie flip rate d={d} bits={bits} rank={rank}: {max(flips):.3f}")


@pytest.mark.parametrize("bits", [8, 4, 2])
@pytest.mark.parametrize("rank", [(1, 1), (5, 3), (7, 4)])
@pytest.mark.parametrize("symmetric", [True, False])
def test_tensor_core_residual_f32_matches_simt(bits, rank, symmetric):
    """tcgen05 encode of fp32 cells with head_dim 64 (R and Pi each in three
    bf16 terms) vs the SIMT fp32 encode of the same cells (two cells, ragged
    rows): scales to 2e-6, zero points within one step, and on each path
    every code more than 1e-3 quantisation steps from a rounding boundary of
    the float64 rotated residual (with that path's scale and zero point)
    equal to the exact code."""
    import oracle.jolt
    from kvcompress_b200.compressor.jl import cached_projection

    g = torch.Generator(device="cuda").manual_seed(100 + bits + 10 * rank[1] + int(symmetric))
    m, t, d = 3, 333, 64
    xs = [torch.randn(m, t, d, generator=g, device="cuda") * 3 + 0.5 for _ in range(2)]
    rt, rd = rank
    fac = ([torch.randn(m, rt, rd, generator=g, device="cuda") for _ in xs],
           [torch.randn(t, rt, generator=g, device="cuda") / 10 for _ in xs],
           [torch.randn(d, rd, generator=g, device="cuda") / 5 for _ in xs])
    proj = cached_projection(d, d, seed=0, device="cuda").matrix
    out = {}
    try:
        for pol in (0, 1):
            _policy(pol)
            sc, zp = ops.residual_stats(xs, fac, proj, bits=bits, symmetric=symmetric, scale_mode=KVC.SCALE_CHANNEL,
                                        stat_dtype=torch.float32)
            codes, _, _ = ops.residual_quant(xs, fac, proj, sc, zp, bits=bits, symmetric=symmetric,
                                             scale_mode=KVC.SCALE_CHANNEL, group_size=None,
                                             stat_dtype=torch.float32, arith_dtype=torch.float32)
            out[pol] = ([s_.cpu().numpy() for s_ in sc], [z.cpu().numpy() for z in zp],
                        [c.cpu().numpy() for c in codes])
    finally:
        _policy(0)
    assert ops.device_error() == 0
    for a, b in zip(out[0][0], out[1][0]):
        assert rel(a, b) < 2e-6
    for a, b in zip(out[0][1], out[1][1]):
        assert np.abs(a.astype(np.int64) - b.astype(np.int64)).max() <= 1
    qmin, qmax = (-(1 << (bits - 1)), (1 << (bits - 1)) - 1) if symmetric else (0, (1 << bits) - 1)
    rows = np.arange(m * t)
    flips = []
    for i, x in enumerate(xs):
        cf = [f32(f[i]) for f in fac]
        recon = recon_rows(cf[0], cf[1], cf[2], "f32", rows, t)
        resid = oracle.jolt.dt_op(lambda a, b: a - b, "f32", f32(x).reshape(m * t, d), recon)
        rot = np.asarray(resid, np.float64) @ proj.cpu().numpy().astype(np.float64).T
        for pol in (0, 1):
            v = rot / out[pol][0][i].astype(np.float64) + out[pol][1][i].astype(np.float64)
            ties = np.abs(v - np.floor(v) - 0.5) < 1e-3
            exact = oracle.pack_codes(np.clip(np.rint(v), qmin, qmax).astype(np.int32), bits, symmetric)
            flips.append(assert_codes_match(out[pol][2][i], exact, bits, d, ties))
    print(f"fp32 near-tie flip rate bits={bits} rank={rank} symmetric={symmetric}: {max(flips):.3f}")


@pytest.mark.parametrize("symmetric", [True, False])
@pytest.mark.parametrize("mode", [KVC.SCALE_CHANNEL, KVC.SCALE_TENSOR])
def test_tensor_core_stats_wide_range(symmetric, mode):
    """Encode stats of rank-1 d = 128 cells on the tensor cores (policy 0:
    three bf16 terms of Pi; policy 2: two fp16 terms, one power-of-two scale
    of R per 128-row tile) against the SIMT pass, on cells of magnitude
    2^-100, 1 and 2^60, the last with tiles stepping through 2^-20, 1, 2^20."""
    from kvcompress_b200.compressor.jl import cached_projection

    g = torch.Generator(device="cuda").manual_seed(7)
    m, t, d = 2, 1024, 128
    proj = cached_projection(d, d, seed=0, device="cuda").matrix
    tile_step = 2.0 ** (20 * (torch.arange(t, device="cuda") // 128 % 3 - 1).float())
    xs, cores, uts, uds = [], [], [], []
    for e, stepped in ((-100, False), (0, False), (60, True)):
        x = torch.randn(m, t, d, generator=g, device="cuda") * 2.0 ** e
        if stepped:
            x = x * tile_step[None, :, None]
        xs.append(x.bfloat16())
        cores.append((torch.randn(m, 1, 1, generator=g, device="cuda") * 2.0 ** e).bfloat16())
        uts.append((torch.randn(t, 1, generator=g, device="cuda") / 30).bfloat16())
        uds.append((torch.randn(d, 1, generator=g, device="cuda") / 11).bfloat16())
    out = {}
    try:
        for pol in (0, 1, 2):
            _policy(pol)
            sc, zp = ops.residual_stats(xs, (cores, uts, uds), proj, bits=8, symmetric=symmetric, scale_mode=mode,
                                        stat_dtype=torch.float32)
            out[pol] = ([s.cpu().numpy() for s in sc], [z.cpu().numpy() for z in zp])
    finally:
        _policy(0)
    assert ops.device_error() == 0
    # 2e-6 (about 16 fp32 ulps): the two passes accumulate the 128 (x 3 terms)
    # products of a rotated value in different orders
    for pol in (0, 2):
        for a, b in zip(out[pol][0], out[1][0]):
            assert np.all(np.isfinite(a)) and np.all(a > 0) and rel(a, b) < 2e-6, pol
        for a, b in zip(out[pol][1], out[1][1]):
            assert np.abs(a.astype(np.int64) - b.astype(np.int64)).max() <= 1, pol


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("bits", [8, 4, 2])
@pytest.mark.parametrize("rank", [(1, 1), (7, 4), (6, 12), (16, 12)])
def test_tensor_core_decompress_matches_simt(d, bits, rank):
    from kvcompress_b200.compressor.jl import cached_projection

    g = torch.Generator(device="cuda").manual_seed(7 * d + bits)
    m, t = 2, 300
    rt, rd = rank
    cb = d * bits // 8
    codes = [torch.randint(0, 256, (m * t, cb), generator=g, device="cuda", dtype=torch.int32).to(torch.uint8)
             for _ in range(3)]
    scales = [torch.rand(d, generator=g, device="cuda") * 0.1 + 0.01 for _ in range(3)]
    zps = [torch.zeros(d, dtype=torch.int32, device="cuda") for _ in range(3)]
    fac = ([torch.randn(m, rt, rd, generator=g, device="cuda").half() for _ in range(3)],
           [(torch.randn(t, rt, generator=g, device="cuda") / 10).half() for _ in range(3)],
           [(torch.randn(d, rd, generator=g, device="cuda") / 5).half() for _ in range(3)])
    proj = cached_projection(d, d, seed=0, device="cuda").matrix
    res = {}
    try:
        for pol in (0, 1):
            _policy(pol)
            outs = ops.decompress((m, t, d), torch.bfloat16, codes=codes, scales=scales, zps=zps, bits=bits,
                                  factors=fac, proj=proj, n_cells=3, device="cuda")
            part = ops.decompress((m, t, d), torch.bfloat16, codes=codes, scales=scales, zps=zps, bits=bits,
                                  factors=fac, proj=proj, n_cells=3, device="cuda", t0=37, t1=299)
            res[pol] = ([f32(o) for o in outs], [f32(o) for o in part])
    finally:
        _policy(0)
    assert ops.device_error() == 0
    for a, b in zip(res[0][0], res[1][0]):
        assert rel(a, b) < 2e-3
    for full, part in zip(res[0][0], res[0][1]):
        np.testing.assert_array_equal(full[:, 37:299], part)


@pytest.mark.parametrize("bits", [8, 4, 2])
@pytest.mark.parametrize("rank", [(1, 1), (7, 4), (6, 12)])
def test_tensor_core_decompress_f32_matches_simt(bits, rank):
    """fp32 output at head_dim 64 (diag(scale) Pi in three bf16 terms, the
    fp32 Tucker term added by the epilogue) vs the SIMT fp32 decode: 1e-6
    relative, and a token range equal to the same rows of the whole decode."""
    from kvcompress_b200.compressor.jl import cached_projection

    d = 64
    g = torch.Generator(device="cuda").manual_seed(11 * bits + rank[1])
    m, t = 2, 300
    rt, rd = rank
    cb = d * bits // 8
    codes = [torch.randint(0, 256, (m * t, cb), generator=g, device="cuda", dtype=torch.int32).to(torch.uint8)
             for _ in range(3)]
    scales = [torch.rand(d, generator=g, device="cuda") * 0.1 + 0.01 for _ in range(3)]
    zps = [torch.zeros(d, dtype=torch.int32, device="cuda") for _ in range(3)]
    fac = ([torch.randn(m, rt, rd, generator=g, device="cuda") for _ in range(3)],
           [torch.randn(t, rt, generator=g, device="cuda") / 10 for _ in range(3)],
           [torch.randn(d, rd, generator=g, device="cuda") / 5 for _ in range(3)])
    proj = cached_projection(d, d, seed=0, device="cuda").matrix
    res = {}
    try:
        for pol in (0, 1):
            _policy(pol)
            outs = ops.decompress((m, t, d), torch.float32, codes=codes, scales=scales, zps=zps, bits=bits,
                                  factors=fac, proj=proj, n_cells=3, device="cuda")
            part = ops.decompress((m, t, d), torch.float32, codes=codes, scales=scales, zps=zps, bits=bits,
                                  factors=fac, proj=proj, n_cells=3, device="cuda", t0=37, t1=299)
            res[pol] = ([f32(o) for o in outs], [f32(o) for o in part])
    finally:
        _policy(0)
    assert ops.device_error() == 0
    for a, b in zip(res[0][0], res[1][0]):
        assert rel(a, b) < 1e-6
        assert np.abs(a - b).max() <= 1e-6 * np.abs(b).max()
    for full, part in zip(res[0][0], res[0][1]):
        np.testing.assert_array_equal(full[:, 37:299], part)


@pytest.mark.parametrize("n_cells,rows,k", [(3, 1332, 11), (64, 300, 14), (2, 65536, 11), (1, 129, 32)])
def test_tensor_core_gram_matches_simt(n_cells, rows, k):
    g = torch.Generator(device="cuda").manual_seed(rows + k)
    cells = [torch.randn(rows, 128, generator=g, device="cuda").bfloat16() * (1 + i) for i in range(n_cells)]
    om = torch.randn(rows, k, generator=g, device="cuda")
    try:
        _policy(0)
        a = ops.gram(cells, om)
        _policy(1)
        b = ops.gram(cells, om)
    finally:
        _policy(0)
    assert ops.device_error() == 0
    a, b = a.cpu().numpy(), b.cpu().numpy()
    G = slice(0, 128 * 128)
    Y = slice(128 * 128, 128 * 128 + 128 * k)
    for i in range(n_cells):
        assert rel(a[i, G], b[i, G]) < 1e-5  # fp32 accumulation order (segment vs 2048-row chunk)
        assert rel(a[i, Y], b[i, Y]) < 5e-5  # Omega carried as bf16 hi + lo
        # the trace sums the fp32 diagonal; the tensor core accumulates a
        # segment of up to 4096 rows in fp32 before the fp64 reduction
        assert abs(a[i, -1] / b[i, -1] - 1) < 2e-5
    # deterministic for a given batch
    np.testing.assert_array_equal(a, ops.gram(cells, om).cpu().numpy())


@pytest.mark.parametrize("dt,d,rd", [("bf16", 128, 1), ("bf16", 64, 3), ("f32", 64, 4), ("f16", 128, 2)])
def test_projection_kernel_matches_oracle(dt, d, rd):
    g = torch.Generator().manual_seed(d + rd)
    m, t = 3, 257
    x_np = oracle.round_to(torch.randn(m, t, d, generator=g).numpy(), dt)
    u_np = oracle.round_to((torch.randn(d, rd, generator=g) / 8).numpy(), dt)
    xp = ops.project_feature([to_cuda(x_np, dt)], [to_cuda(u_np, dt)])[0]
    ref = oracle.jolt.matmul_round(x_np.reshape(-1, d), u_np, dt).reshape(m, t, rd)
    ref_t = np.moveaxis(ref, 1, 0).reshape(t, m * rd)
    got = f32(xp)
    if dt != "f32":
        # 16-bit outputs: equal except 1-ulp flips where the fp32 summation
        # order meets a rounding tie
        mism = np.mean(got != ref_t)
        assert mism < 5e-3, mism
    assert rel(got, ref_t) < (1e-6 if dt == "f32" else 1e-2)
