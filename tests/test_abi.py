"""The C-ABI library loads and exports every entry point include/kvc_b200.h declares (CPU)."""

from __future__ import annotations

import ctypes
import os
import re

from kvcompress_b200 import _build
from kvcompress_b200._native import exported_symbols, lib

HEADER = os.path.join(os.path.dirname(__file__), "..", "include", "kvc_b200.h")


def declared_functions() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(kvc_\w+)\s*\(", src)))


def test_library_built_in_tree():
    assert os.path.exists(_build.LIB_PATH)
    assert os.path.dirname(_build.LIB_PATH).startswith(os.path.dirname(os.path.dirname(_build.__file__)))


def test_every_declared_symbol_is_exported():
    L = ctypes.CDLL(_build.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(L, name), f"{name} declared in kvc_b200.h but not exported"


def test_binding_covers_header():
    assert sorted(exported_symbols()) == declared_functions()


def test_host_only_entry_points():
    L = lib()
    assert L.kvc_abi_version() == 1
    assert isinstance(L.kvc_launch_count(), int) and L.kvc_launch_count() >= 0
    # workspace queries are pure host arithmetic
    assert L.kvc_sketch_solve_workspace_bytes(2, 1, 128, 11) > 0
    assert L.kvc_sketch_solve_workspace_bytes(0, 1, 128, 11) == 0
