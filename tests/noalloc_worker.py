"""Child process for tests/test_zz_no_alloc.py: one sh_cuda_gemm_splitk_noalloc call under planner overrides.

The planner reads its environment overrides (SH_GEMM_PAIR_BN, ...) once per process, so a case that needs one runs
here, in a fresh process started with that environment. Usage: python noalloc_worker.py M N K splits flags.
Prints "OK <max-abs vs sh_cuda_gemm> <max-abs vs the oracle> <planner kernel> <planner bn>" and exits 0, or
raises.
"""
from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "softhier-mlir_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import ctypes as C  # noqa: E402

import numpy as np  # noqa: E402

from oracle import lcg, ops  # noqa: E402
from softhier_cuda import lib as L  # noqa: E402
from softhier_cuda.runtime import Runtime  # noqa: E402


def main(M: int, N: int, K: int, splits: int, flags: int) -> None:
    rt = Runtime.open(0, arena_bytes=1 << 30)
    lib = rt.lib
    plan = L.GemmPlan()
    assert lib.sh_cuda_gemm_plan(M, N, K, splits, 0, C.byref(plan)) == 0
    x, w = lcg.uniform_fp16(M, K, 51), lcg.uniform_fp16(K, N, 52)
    bias = lcg.normal_fp16(1, N, 53, 0.0, 0.5)
    dx, dw, db = rt.upload(x), rt.upload(w), rt.upload(bias)
    za, zb = rt.alloc(M, N), rt.alloc(M, N)
    assert lib.sh_cuda_gemm(dx, dw, za, M, N, K, K, N, N, db, 0, 0, flags, splits) == 0
    assert lib.sh_cuda_gemm_splitk_noalloc(dx, dw, zb, M, N, K, K, N, N, db, 0, 0, flags, splits) == 0
    rt.check()
    a, b = rt.get(za, M, N).astype(np.float32), rt.get(zb, M, N).astype(np.float32)
    want = ops.gemm(x, w) + bias.astype(np.float32)
    if flags & L.EPI_GELU:
        want = ops.gelu(want)
    print("OK", float(np.abs(b - a).max()), float(np.abs(b - want).max()), plan.kernel, plan.bn)


if __name__ == "__main__":
    main(*(int(v, 0) for v in sys.argv[1:6]))
