"""Host-side logic on CPU: JL matrices, sketch sizes, dispatch, loud failures."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from kvcompress_b200 import build_compressor, flashjolt_cap
from kvcompress_b200.compressor.jl import cached_projection, clear_projection_cache
from kvcompress_b200.compressor.svd import SVD, sketch_width
from kvcompress_b200._native import KVC


def test_jl_matrix_bit_identical(golden):
    clear_projection_cache()
    for d in (64, 128):
        got = cached_projection(d, d, seed=0).matrix.numpy()
        np.testing.assert_array_equal(got, golden[f"jl/pi_d{d}_seed0"])
    np.testing.assert_array_equal(cached_projection(128, 128, seed=7).matrix.numpy(),
                                  golden["jl/pi_d128_seed7"])


def test_cap_and_sketch_width_match_oracle(golden):
    for t, r, cap in golden.meta["flashjolt_cap"]:
        assert flashjolt_cap(t, r) == cap
    for rows, cols, rank, cap in [(128, 65536, 1, 256), (4096, 1024, 512, 128), (8192, 8, 1, 256),
                                  (64, 8192, 4, 64), (128, 2097152, 16, 512), (10, 10, 10, None)]:
        assert sketch_width(rows, cols, rank, 10, cap) == oracle.sketch_width(rows, cols, rank, 10, cap)
    # q = 513 when the 512 cap meets rank 512 (svd.py:244)
    assert sketch_width(4096, 1024, 512, 10, 512) == (512, 513)


def test_svd_dispatch_rules():
    s = SVD(method="auto")
    assert s.resolve(128, 65536, 1, None)[0] == KVC.SVD_RANDOMISED
    assert s.resolve(128, 65536, 100, None)[0] == KVC.SVD_EXACT
    assert SVD(method="exact").resolve(128, 65536, 1, None, forced_randomised=True)[0] == KVC.SVD_RANDOMISED
    assert SVD(method="exact").resolve(128, 65536, 1, None)[0] == KVC.SVD_EXACT


def test_dispatch_allow_lists():
    with pytest.raises(NotImplementedError):
        build_compressor("nope")
    with pytest.raises(ValueError):
        build_compressor("flashjolt", per_chanel=True)
    with pytest.raises(ValueError):
        build_compressor("jolt", compression_ratio=1.0)
    c = build_compressor("flashjolt", compression_ratio=4.0, seed=3)
    assert c.name == "flashjolt" and c.seed == 3 and c.svd.method == "randomised"
    assert build_compressor("int4").bits == 4
    assert build_compressor("fp8").factor_dtype == torch.float8_e4m3fn


def test_cpu_tensors_fail_loudly():
    """There is no CPU fallback: CPU inputs raise instead of silently running elsewhere."""
    k = torch.randn(2, 16, 64)
    for method in ("flashjolt", "jolt"):
        with pytest.raises(RuntimeError, match="CUDA"):
            build_compressor(method, compression_ratio=4.0).compress(k, k)
    with pytest.raises(ValueError):
        build_compressor("flashjolt", compression_ratio=4.0).compress(k, k[:1])
    with pytest.raises(ValueError):
        build_compressor("flashjolt", compression_ratio=4.0).compress(k[0], k[0])


def test_library_calls_run_on_the_tensors_device(monkeypatch):
    """``ops._on``: the library launches on the calling thread's current
    device, so every wrapper makes the tensors' device current first; no
    switch (no driver call) when it already is."""
    from kvcompress_b200 import ops

    switched = []

    class FakeDevice:
        def __init__(self, idx):
            switched.append(idx)

    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(torch.cuda, "device", FakeDevice)
    assert ops._on(torch.device("cuda", 0)) is ops._NO_GUARD
    assert ops._on(torch.device("cuda")) is ops._NO_GUARD
    assert isinstance(ops._on(torch.device("cuda", 1)), FakeDevice)
    assert switched == [1]
