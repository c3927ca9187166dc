"""HBM preload images (softhier_mlir/sim/preload.py ELF32): the library's parser on the CPU against the segments the
reference's own reader returns (tests/golden/preload_small.npz)."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from conftest import golden
from softhier_cuda import lib as L

GOLDEN = Path(__file__).resolve().parent / "golden"
HBM_BASE = 0xC0000000


def test_preload_segments_match_reference_reader():
    lib = L.load()
    g = golden("preload_small.npz")
    n = len(g["offsets"])
    offs, sizes = (ctypes.c_uint64 * 8)(), (ctypes.c_uint64 * 8)()
    assert lib.sh_preload_elf_segments(str(GOLDEN / "preload_small.elf").encode(), HBM_BASE, offs, sizes, 8) == n
    assert list(offs[:n]) == [int(o) for o in g["offsets"]]
    assert list(sizes[:n]) == [len(g[f"seg_{int(o):x}"]) for o in g["offsets"]]
    # the last segment is the 64-byte sentinel (16 x 0x5EEDC0DE) the program waits for
    last = g[f"seg_{int(g['offsets'][-1]):x}"]
    assert last.view(np.uint32).tolist() == [0x5EEDC0DE] * 16


def test_preload_rejects_other_files(tmp_path):
    lib = L.load()
    bad = tmp_path / "bad.elf"
    bad.write_bytes(b"not an elf" * 10)
    assert lib.sh_preload_elf_segments(str(bad).encode(), HBM_BASE, None, None, 0) == -1
    assert lib.sh_preload_elf_segments(str(tmp_path / "missing.elf").encode(), HBM_BASE, None, None, 0) == -1
    # a wrong HBM base puts every segment below it
    assert lib.sh_preload_elf_segments(str(GOLDEN / "preload_small.elf").encode(), 0xD0000000, None, None, 0) == -1
    assert lib.sh_cuda_last_error() == -1
