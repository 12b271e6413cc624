"""ctypes binding of the C ABI in ``include/kvc_b200.h``.

The library is built in-tree (``kvcompress_b200/_lib/libkvc_b200.so``) by
``kvcompress_b200._build``.  There is no fallback: if the library is
missing, every GPU entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

from kvcompress_b200 import _build

__all__ = ["lib", "check", "KVC", "ptr_array"]

_LOCK = threading.Lock()
_LIB = None

P = ctypes.c_void_p
PP = ctypes.POINTER(ctypes.c_void_p)
I = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t
DP = ctypes.c_void_p  # double* / float* / int32* passed as raw addresses


class KVC:
    """Constants mirrored from ``kvc_b200.h``."""

    OK = 0
    F32, F16, BF16, F64, FP8E4M3 = 0, 1, 2, 3, 4
    SVD_EXACT, SVD_RANDOMISED = 0, 1
    SIDE_LEFT, SIDE_RIGHT = 0, 1
    SCALE_CHANNEL, SCALE_GROUP, SCALE_TENSOR = 0, 1, 2
    MAX_CELLS = 64
    NOALLOC_SCRATCH_BYTES = 8 << 20
    ERR_ARG = -1
    ERR_WORKSPACE = -5
    ERR_UNSUPPORTED = -8


_SIGNATURES = {
    "kvc_last_error": (ctypes.c_char_p, []),
    "kvc_launch_count": (ctypes.c_ulonglong, []),
    "kvc_abi_version": (I, []),
    "kvc_gram_workspace_bytes": (SZ, [I, I64, I, I]),
    "kvc_gram": (I, [I, PP, I64, I, I, P, I, P, P, SZ, P]),
    "kvc_sketch_solve_workspace_bytes": (SZ, [I, I, I, I]),
    "kvc_sketch_solve": (I, [I, I, I, I, I64, I, I, I, P, I64, P, P, I, P, P, P, SZ, P]),
    "kvc_project_feature": (I, [I, PP, I64, I64, I, I, PP, I, PP, P]),
    "kvc_apply_basis": (I, [I, PP, I64, I, I, P, I, PP, P]),
    "kvc_core_workspace_bytes": (SZ, [I, I64, I, I, I]),
    "kvc_core": (I, [I, PP, PP, I64, I, I, I, I, PP, P, SZ, P]),
    "kvc_residual_stats_workspace_bytes": (SZ, [I, I64, I, I]),
    "kvc_residual_stats": (I, [I, PP, I64, I64, I, I, PP, PP, PP, I, I, P, I, I, I, I, PP, PP, P,
                               SZ, P]),
    "kvc_residual_quant_workspace_bytes": (SZ, [I, I64, I, I]),
    "kvc_residual_quant": (I, [I, PP, I64, I64, I, I, PP, PP, PP, I, I, P, I, I, I, I, I, I, PP, PP,
                               PP, P, SZ, P]),
    "kvc_decompress_workspace_bytes": (SZ, [I, I64, I, I]),
    "kvc_decompress": (I, [I, PP, PP, PP, I, I, I, I, PP, PP, PP, I, I64, I64, I, I, I, P, I64, I64, I,
                           PP, P, SZ, P]),
    "kvc_decompress_noalloc": (I, [I, PP, PP, PP, I, I, I, I, PP, PP, PP, I, I64, I64, I, I, I, P, I64,
                                   I64, I, PP, P]),
    "kvc_decode_plan_bytes": (SZ, []),
    "kvc_decode_plan_init": (I, [P, SZ, I, PP, PP, PP, I, I, I, I, PP, PP, PP, I, I64, I64, I, I, I, P, I,
                                 P, SZ, P]),
    "kvc_decode_plan_run": (I, [P, SZ, I64, I64, PP, P]),
    "kvc_compress_workspace_bytes": (SZ, [I, I64, I64, I, I, I, I, I, I, I, I, I, I]),
    "kvc_compress": (I, [I, PP, I64, I64, I, I, I, I, I, I, P, I, I, P, I, P, I, I, I, I, I, I, I, P, P, P, P, P,
                         P, P, P, P, P, P, P, P, P, SZ, P]),
    "kvc_trace_stages": (I, [PP, I]),
    "kvc_set_kernel_policy": (I, [I]),
    "kvc_device_error": (I, [ctypes.POINTER(I)]),
    "kvc_cast": (I, [I64, P, I, P, I, P]),
}


def lib():
    """Load the extension (once).  Raises if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            path = _build.LIB_PATH
            if not os.path.exists(path):
                raise RuntimeError(
                    f"kvcompress_b200: native library {path} is missing; build it with "
                    "`python -m kvcompress_b200._build` (there is no CPU fallback)")
            L = ctypes.CDLL(path)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = L
    return _LIB


def exported_symbols() -> list[str]:
    """Names of the C ABI entry points this binding declares."""
    return list(_SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc != KVC.OK:
        msg = lib().kvc_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (code {rc}): {msg}")


def ptr_array(ptrs) -> ctypes.Array:
    """Host array of device pointers for the batched entry points."""
    ptrs = list(ptrs)
    return (ctypes.c_void_p * max(1, len(ptrs)))(*[p or 0 for p in ptrs])
