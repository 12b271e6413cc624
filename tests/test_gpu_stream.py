"""Token-range decode streams (DecodeStream / kvc_decode_plan_*).

Every block of a stream must equal, bit for bit, the same token range decoded
by ``decompress_tokens``, and the full-range decode of a stream must equal
``decompress``; layouts without a tensor-core plan take the regular path.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from kvcompress_b200 import DecodeStream, build_compressor, ops
from kvcompress_b200._native import KVC, lib
from kvcompress_b200.synthetic import WORKLOADS, make_kv_layer


def _pairs(layers, tokens, dtype=torch.bfloat16):
    w = WORKLOADS["llama3-8b-kv-b1-t8192-bf16"]
    out = []
    for li in range(layers):
        k, v = make_kv_layer(w, li, tokens=tokens)
        out.append((k.reshape(8, tokens, 128).to(dtype).cuda(), v.reshape(8, tokens, 128).to(dtype).cuda()))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [(0, 2, 4, 8), (0, 2, 4)])
def test_stream_blocks_equal_token_range_decodes(bits):
    comp = build_compressor("flashjolt", compression_ratio=4.0, bits=bits)
    pays = comp.compress_many(_pairs(3, 1024))
    stream = DecodeStream(pays)
    if bits == (0, 2, 4, 8):
        assert stream.planned  # (1, 1, 8) for K and V: tensor-core plans
    ranges = [(t0, min(t0 + 256, 1024)) for t0 in range(0, 1024, 256)] + [(100, 612), (1000, 1024), (0, 1)]
    for t0, t1 in ranges:
        got = stream.decode(t0, t1)
        for (kp, vp), (kd, vd) in zip(pays, got):
            assert kd.shape == (8, t1 - t0, 128) and kd.dtype == torch.bfloat16
            assert torch.equal(kd, comp.decompress_tokens(kp, t0, t1))
            assert torch.equal(vd, comp.decompress_tokens(vp, t0, t1))
    full = stream.decode(0, 1024)
    for (kp, vp), (kd, vd) in zip(pays, full):
        k_ref, v_ref = comp.decompress(kp, vp)
        assert torch.equal(kd, k_ref) and torch.equal(vd, v_ref)
    blocks = list(stream.blocks(300))
    assert [(a, b) for a, b, _ in blocks] == [(0, 300), (300, 600), (600, 900), (900, 1024)]
    assert ops.device_error() == 0


@pytest.mark.gpu
def test_captured_stream_replays_every_block():
    comp = build_compressor("flashjolt", compression_ratio=4.0)
    pays = comp.compress_many(_pairs(2, 1024))
    stream = DecodeStream(pays)
    cap = stream.capture(256)
    assert cap.spans == [(0, 256), (256, 512), (512, 768), (768, 1024)]
    for _ in range(2):
        for o in cap.outputs:  # poison, then replay must rewrite every block
            for pair in o:
                for x in pair:
                    x.fill_(float("nan"))
        outs = cap.replay()
        torch.cuda.synchronize()
        for (t0, t1), blk in zip(cap.spans, outs):
            for (kp, vp), (kd, vd) in zip(pays, blk):
                assert torch.equal(kd, comp.decompress_tokens(kp, t0, t1))
                assert torch.equal(vd, comp.decompress_tokens(vp, t0, t1))
    assert ops.device_error() == 0


@pytest.mark.gpu
def test_stream_without_a_plan_uses_the_regular_decode():
    comp = build_compressor("flashjolt", compression_ratio=4.0)
    pays = comp.compress_many(_pairs(2, 512, torch.float32))  # fp32 cells: no tensor-core plan
    stream = DecodeStream([p for pair in pays for p in pair])
    assert not stream.planned
    got = stream.decode(64, 320)
    flat = [p for pair in pays for p in pair]
    for p, d in zip(flat, got):
        assert torch.equal(d, comp.decompress_tokens(p, 64, 320))


def test_plan_run_rejects_an_uninitialised_plan():
    """Host-side check: nothing reaches the GPU."""
    L = lib()
    nb = L.kvc_decode_plan_bytes()
    assert nb > 8192  # the codes tensor maps of 64 cells live in the plan
    buf = ctypes.create_string_buffer(nb)
    z = (ctypes.c_void_p * 1)(0)
    assert L.kvc_decode_plan_run(buf, nb, 0, 1, z, None) == KVC.ERR_ARG
    assert b"not an initialised plan" in L.kvc_last_error()
    assert L.kvc_decode_plan_run(buf, 16, 0, 1, z, None) == KVC.ERR_ARG
