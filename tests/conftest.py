"""Shared pytest setup: the `gpu` marker, import paths and golden-fixture loading."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "softhier-mlir_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def golden(name: str):
    return np.load(GOLDEN / name)


@pytest.fixture(scope="session")
def gpu_lib():
    """The loaded CUDA library on cuda:0 with a device arena bound (GPU tests only)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from softhier_cuda import runtime
    rt = runtime.Runtime.open(arena_bytes=2 << 30)
    return rt
