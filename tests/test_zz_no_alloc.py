"""sh_cuda_gemm_splitk_noalloc: the split-K GEMM for callers that cannot let the library allocate device memory
(hosts whose own pool owns all device memory, loops that cannot take cudaMalloc's implicit synchronisation).

It must give the same numbers as the allocating entry point sh_cuda_gemm, call after call, while its split-K
scratch comes from a fixed array compiled into the library. This file is collected last so that a run stopping
at the first failure has already run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

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
