"""The GEMM planner through sh_cuda_gemm_plan, on the CPU (the query makes no CUDA call when given the SM count):
which kernel and tiling sh_cuda_gemm uses for the shapes the bench and SUMMA run, on 148 SMs (74 SM pairs)."""
from __future__ import annotations

import ctypes as C

import pytest

from softhier_cuda import lib as L

SMS = 148


@pytest.fixture(scope="module")
def plan():
    lib = L.load()

    def run(M, N, K, splits=0, sms=SMS):
        p = L.GemmPlan()
        assert lib.sh_cuda_gemm_plan(M, N, K, splits, sms, C.byref(p)) == 0
        return {f: getattr(p, f) for f, _ in L.GemmPlan._fields_}
    return run


def test_encoder_shapes_use_256x256_pair_tiles(plan):
    # K = 768: 12 k-blocks, too short for 256 x 512 tiles (their epilogue would not overlap the next tile)
    for N in (2304, 768, 3072):
        p = plan(131072, N, 768)
        assert (p["kernel"], p["bn"], p["tiles_m"], p["splits"]) == (2, 256, 512, 1)
        assert p["units"] == p["full_units"] == 512 * (N // 256) and p["grid"] == SMS
    p = plan(131072, 768, 3072)                 # FC2: N % 512 != 0
    assert (p["kernel"], p["bn"], p["k_blocks"]) == (2, 256, 48)


def test_long_k_shapes_use_256x512_pair_tiles(plan):
    p = plan(16384, 16384, 16384)               # 2048 wide tiles: 27 full waves + 50 (too many to slice)
    assert (p["kernel"], p["bn"], p["tiles_m"], p["tiles_n"]) == (2, 512, 64, 32)
    assert p["full_units"] == p["units"] == 2048 and p["grid"] == SMS
    p = plan(8192, 4096, 16384)                 # the 2x4 SUMMA rank: 3 full waves + 34 tiles as 68 slices
    assert (p["kernel"], p["bn"], p["full_units"], p["units"], p["grid"]) == (2, 512, 222, 290, SMS)
    p = plan(4096, 4096, 2048)                  # 128 wide tiles (6 half-tile-times) vs 256 narrow (8)
    assert (p["kernel"], p["bn"], p["units"]) == (2, 512, 128)
    p = plan(4096, 4096, 1984)                  # 31 k-blocks: below the 32 that wide tiles need
    assert (p["kernel"], p["bn"]) == (2, 256)


def test_small_shapes_single_cta_and_split_k(plan):
    p = plan(512, 512, 512)                     # 8 k-blocks: no split; 64-column tiles to occupy more SMs
    assert (p["kernel"], p["bn"], p["tiles_m"], p["tiles_n"], p["splits"], p["grid"]) == (1, 64, 4, 8, 1, 32)
    p = plan(256, 768, 3072)                    # 24 tiles, 48 k-blocks: 6 splits of 8 blocks
    assert (p["kernel"], p["bn"], p["splits"], p["units"], p["grid"]) == (1, 64, 6, 144, 144)
    p = plan(256, 768, 3072, splits=1)
    assert (p["splits"], p["units"]) == (1, 24)
    p = plan(256, 768, 3072, splits=3)
    assert (p["splits"], p["units"]) == (3, 72)


def test_degenerate_shapes_and_arguments(plan):
    assert plan(0, 64, 64)["kernel"] == 0
    assert plan(64, 64, 0)["kernel"] == 0
    assert L.load().sh_cuda_gemm_plan(64, 64, 64, 0, SMS, None) == -1
    # fewer SMs: the same tile rules against the smaller machine
    p = plan(131072, 3072, 768, sms=16)
    assert (p["kernel"], p["bn"], p["grid"]) == (2, 256, 16)
