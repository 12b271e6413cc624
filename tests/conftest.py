"""Shared fixtures: the golden vectors and the ``gpu`` marker."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")
    config.addinivalue_line("markers", "slow: long-running")


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    """bf16 raw bits (uint16) -> float32 values."""
    return (a.astype(np.uint32) << np.uint32(16)).view(np.float32)


class Golden:
    """Lazy view of ``tests/golden/golden.npz`` + ``golden.json``.

    uint16 arrays hold bfloat16 bit patterns and are widened to float32.
    """

    def __init__(self) -> None:
        self.npz = np.load(os.path.join(GOLDEN_DIR, "golden.npz"))
        with open(os.path.join(GOLDEN_DIR, "golden.json")) as f:
            self.meta = json.load(f)

    def __getitem__(self, key: str) -> np.ndarray:
        a = self.npz[key]
        if a.dtype == np.uint16:
            return bf16_bits_to_f32(a)
        return a

    def raw(self, key: str) -> np.ndarray:
        return self.npz[key]

    def __contains__(self, key: str) -> bool:
        return key in self.npz.files

    def case_input(self, case: str) -> np.ndarray:
        return self["inputs/" + self.meta[case]["input"]]


@pytest.fixture(scope="session")
def golden() -> Golden:
    return Golden()
