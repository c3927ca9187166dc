"""sh_cuda_gemm_splitk_noalloc: the split-K GEMM for callers that cannot let the library allocate device memory
(hosts whose own pool owns all device memory, loops that cannot take cudaMalloc's implicit synchronisation).

It must give the same numbers as the allocating entry point sh_cuda_gemm, call after call, while its split-K
scratch comes from a fixed array compiled into the library. This file is collected last so that a run stopping
at the first failure has already run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import lcg, ops
from softhier_cuda import lib as L

pytestmark = pytest.mark.gpu


def _tol(got, want):
    got = np.asarray(got, np.float32)
    err = np.abs(got - np.asarray(want, np.float32))
    return bool(np.all(err <= 2e-2 + 2.0 ** -10 * np.abs(want))), float(err.max())


def test_noalloc_matches_allocating_gemm_on_consecutive_calls(gpu_lib):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    cases = [(256, 768, 3072, L.EPI_BIAS | L.EPI_GELU, 4), (384, 512, 2048, L.EPI_BIAS | L.EPI_RESIDUAL, 0)]
    for i, (M, N, K, flags, splits) in enumerate(cases):
        x = lcg.uniform_fp16(M, K, 10 + i)
        w = lcg.uniform_fp16(K, N, 20 + i)
        bias = lcg.normal_fp16(1, N, 30 + i, 0.0, 0.5)
        res = lcg.normal_fp16(M, N, 40 + i)
        dx, dw, db, dr = rt.upload(x), rt.upload(w), rt.upload(bias), rt.upload(res)
        z_alloc, z_fixed = rt.alloc(M, N), rt.alloc(M, N)
        assert lib.sh_cuda_gemm(dx, dw, z_alloc, M, N, K, K, N, N, db, dr, N, flags, splits) == 0
        assert lib.sh_cuda_gemm_splitk_noalloc(dx, dw, z_fixed, M, N, K, K, N, N, db, dr, N, flags, splits) == 0
        rt.check()
        a, b = rt.get(z_alloc, M, N), rt.get(z_fixed, M, N)
        ok, err = _tol(b, a.astype(np.float32))
        assert ok, (i, err)
        want = ops.gemm(x, w) + bias.astype(np.float32)
        want = ops.gelu(want) if flags & L.EPI_GELU else want + res.astype(np.float32)
        ok, err = _tol(b, want)
        assert ok, (i, err)


def test_noalloc_allocates_nothing_and_rejects_oversize(gpu_lib, capfd):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    M, N, K = 512, 768, 4096
    x, w = rt.upload(lcg.uniform_fp16(M, K, 1)), rt.upload(lcg.uniform_fp16(K, N, 2))
    z = rt.alloc(M, N)
    assert lib.sh_cuda_gemm_splitk_noalloc(x, w, z, M, N, K, K, N, N, 0, 0, 0, 0, 2) == 0   # warm (module load)
    rt.check()
    free0, _ = torch.cuda.mem_get_info()
    for splits in (3, 4):      # 48 tiles of 128 x 64: up to 6.3 MB of partials
        assert lib.sh_cuda_gemm_splitk_noalloc(x, w, z, M, N, K, K, N, N, 0, 0, 0, 0, splits) == 0
    rt.check()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    ok, err = _tol(rt.get(z, M, N), ops.gemm(rt.get(x, M, K), rt.get(w, K, N)))
    assert ok, err
    capfd.readouterr()
    bx, bw, bz = rt.alloc(1024, 3072), rt.alloc(3072, 3072), rt.alloc(1024, 3072)
    assert lib.sh_cuda_gemm_splitk_noalloc(bx, bw, bz, 1024, 3072, 3072, 3072, 3072, 3072, 0, 0, 0, 0, 16) == -2
    assert "[sh_cuda_gemm_splitk_noalloc]" in capfd.readouterr().out
    assert lib.sh_cuda_last_error() == -2


def _get_f32(rt, addr, rows, cols):
    rt.lib.sh_cuda_synchronize()
    off = addr - rt.base
    return rt.arena[off:off + 4 * rows * cols].view(torch.float32).reshape(rows, cols).cpu().numpy()


@pytest.mark.parametrize("splits", [0, 1])
def test_noalloc_on_pair_plan_shapes(gpu_lib, splits):
    """4096 x 4096 x 2048: sh_cuda_gemm runs 256 x 512 two-CTA tiles here; every output column must be written."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    M, N, K = 4096, 4096, 2048
    plan = L.GemmPlan()
    assert lib.sh_cuda_gemm_plan(M, N, K, splits, 0, C.byref(plan)) == 0
    assert (plan.kernel, plan.bn) == (2, 512)   # the plan whose tile count the no-alloc path must not reuse
    x, w = lcg.uniform_fp16(M, K, 61), lcg.uniform_fp16(K, N, 62)
    dx, dw = rt.upload(x), rt.upload(w)
    za, zb = rt.alloc(M, N), rt.alloc(M, N)
    rt.view(zb, M, N).fill_(float("nan"))
    assert lib.sh_cuda_gemm(dx, dw, za, M, N, K, K, N, N, 0, 0, 0, 0, splits) == 0
    assert lib.sh_cuda_gemm_splitk_noalloc(dx, dw, zb, M, N, K, K, N, N, 0, 0, 0, 0, splits) == 0
    rt.check()
    a, b = rt.get(za, M, N).astype(np.float32), rt.get(zb, M, N).astype(np.float32)
    assert np.isfinite(b).all()
    ok, err = _tol(b, a)
    assert ok, err
    ok, err = _tol(b, ops.gemm(x, w))
    assert ok, err


def test_noalloc_accumulate_and_fp32_modes(gpu_lib):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    M, N, K = 256, 768, 3072
    x, w = lcg.uniform_fp16(M, K, 71), lcg.uniform_fp16(K, N, 72)
    z0 = lcg.normal_fp16(M, N, 73)
    dx, dw = rt.upload(x), rt.upload(w)
    prod = ops.gemm(x, w)
    # Z (+)= X W in fp16, split 4 ways, twice in a row against the allocating entry point
    za, zb = rt.upload(z0), rt.upload(z0)
    for _ in range(2):
        assert lib.sh_cuda_gemm(dx, dw, za, M, N, K, K, N, N, 0, 0, 0, L.EPI_ACCUMULATE, 4) == 0
        assert lib.sh_cuda_gemm_splitk_noalloc(dx, dw, zb, M, N, K, K, N, N, 0, 0, 0, L.EPI_ACCUMULATE, 4) == 0
    rt.check()
    a, b = rt.get(za, M, N).astype(np.float32), rt.get(zb, M, N).astype(np.float32)
    ok, err = _tol(b, a)
    assert ok, err
    want = (z0.astype(np.float32) + prod).astype(np.float16).astype(np.float32) + prod
    ok, err = _tol(b, want)
    assert ok, err
    # fp32 out, then an fp32 carry-in of that result: Z32 = X W + X W
    z32 = rt.alloc_bytes(4 * M * N, 256)
    z32b = rt.alloc_bytes(4 * M * N, 256)
    f32 = L.EPI_F32_OUT
    assert lib.sh_cuda_gemm_splitk_noalloc(dx, dw, z32, M, N, K, K, N, N, 0, 0, 0, f32, 3) == 0
    assert lib.sh_cuda_gemm_splitk_noalloc(dx, dw, z32b, M, N, K, K, N, N, 0, z32, N, f32 | L.EPI_ACC_F32_IN, 3) == 0
    rt.check()
    got1, got2 = _get_f32(rt, z32, M, N), _get_f32(rt, z32b, M, N)
    assert np.abs(got1 - prod).max() <= 1e-2, np.abs(got1 - prod).max()
    assert np.abs(got2 - 2 * prod).max() <= 2e-2, np.abs(got2 - 2 * prod).max()


def test_noalloc_rejects_unsupported_flags(gpu_lib, capfd):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    M, N, K = 256, 256, 1024
    dx, dw, z = rt.alloc(M, K), rt.alloc(K, N), rt.alloc(M, N)
    capfd.readouterr()
    for bad in (L.EPI_LN_IN, L.EPI_STATS_OUT, 0x200, L.EPI_RESIDUAL | L.EPI_ACC_F32_IN):
        assert lib.sh_cuda_gemm_splitk_noalloc(dx, dw, z, M, N, K, K, N, N, 0, dx, N, bad, 2) == -1
        assert "[sh_cuda_gemm_splitk_noalloc]" in capfd.readouterr().out
        assert lib.sh_cuda_last_error() == -1


def test_noalloc_under_forced_wide_pair_tiles():
    """SH_GEMM_PAIR_BN=512 makes sh_cuda_gemm pick 256 x 512 tiles at 4096 x 2048 x 768 (a fresh process)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    worker = Path(__file__).resolve().parent / "noalloc_worker.py"
    env = dict(os.environ, SH_GEMM_PAIR_BN="512")
    r = subprocess.run([sys.executable, str(worker), "4096", "2048", "768", "0", str(L.EPI_BIAS | L.EPI_GELU)],
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("OK ")][-1].split()
    vs_alloc, vs_oracle, kernel, bn = float(line[1]), float(line[2]), int(line[3]), int(line[4])
    assert (kernel, bn) == (2, 512)
    assert vs_alloc <= 2e-2 and vs_oracle <= 2e-2 + 2.0 ** -10 * 32, (vs_alloc, vs_oracle)
