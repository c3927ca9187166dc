"""Runs a small encoder forward (2 SigLIP-base layers, B = 12: 2-CTA and 1-CTA GEMMs, tcgen05 attention, LayerNorm),
one wide GEMM (2816 x 4096 x 256: 11 x 16 pair tiles, a partial tile group) and two long-K GEMMs (4096 x 4096 x
2048: 256 x 512 pair tiles; 8192 x 4096 x 2048: the same with a tail wave of column slices) on GPU 0 and prints the SHA-1 of their output bytes. tests/test_launch_modes_gpu.py runs it
under different launch settings (SH_PDL, SH_GEMM_GROUP_M, SH_GEMM_PAIR_BN, SH_GEMM_KS), which are read once per
process, and requires identical bytes: the launch mode, the tile order, the tile width and the barrier grouping must
not change any result."""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "softhier-mlir_b200")]

import numpy as np  # noqa: E402

from oracle import lcg, siglip  # noqa: E402
from softhier_cuda import encoder  # noqa: E402
from softhier_cuda.runtime import Runtime  # noqa: E402


def main():
    rt = Runtime.open(0, arena_bytes=1 << 30)
    lib = rt.lib
    B, S, D, F, H = 12, 256, 768, 3072, 12
    layers = [siglip.baseline_layer_params(D, F, 40 + i) for i in range(2)]
    x = lcg.normal_fp16(B * S, D, 9)
    ws = [encoder.upload_layer(rt, p) for p in layers]
    act = encoder.alloc_activations(rt, B, S, D, F)
    rt.put(act.x, x)
    res = encoder.encoder_forward(lib, act, ws, H, 1e-6, 0.125)
    rt.check()
    enc = rt.get(res, B * S, D)

    M, N, K = 2816, 4096, 256
    a, w, z = rt.alloc(M, K), rt.alloc(K, N), rt.alloc(M, N)
    lib.sh_test_fill_fp16(a, M, K, K, 3, -1024, 1023, 1.0 / 1024)
    lib.sh_test_fill_fp16(w, K, N, N, 4, -1024, 1023, 1.0 / 1024)
    if lib.sh_cuda_gemm(a, w, z, M, N, K, K, N, N, 0, 0, N, 0, 0):
        raise RuntimeError(lib.sh_cuda_last_error_string().decode())
    rt.check()
    gem = rt.get(z, M, N)
    want = lcg.fill_fp16(M, K, 3, -1024, 1023, 1 / 1024).astype(np.float32) @ \
        lcg.fill_fp16(K, N, 4, -1024, 1023, 1 / 1024).astype(np.float32)
    err = float(np.abs(gem.astype(np.float32) - want).max())
    if err > 2e-2 + 2.0 ** -10 * float(np.abs(want).max()):
        raise AssertionError(f"wide GEMM max err {err}")
    # 4096 x 4096 x 2048: the planner's 256 x 512 pair tiles (SH_GEMM_PAIR_BN=256 forces 256 x 256)
    M2, N2, K2 = 4096, 4096, 2048
    a2, w2, z2 = rt.alloc(M2, K2), rt.alloc(K2, N2), rt.alloc(M2, N2)
    lib.sh_test_fill_fp16(a2, M2, K2, K2, 5, -1024, 1023, 1.0 / 1024)
    lib.sh_test_fill_fp16(w2, K2, N2, N2, 6, -1024, 1023, 1.0 / 1024)
    if lib.sh_cuda_gemm(a2, w2, z2, M2, N2, K2, K2, N2, N2, 0, 0, N2, 0, 0):
        raise RuntimeError(lib.sh_cuda_last_error_string().decode())
    rt.check()
    wide = rt.get(z2, M2, N2)
    # 8192 x 4096 x 2048: 256 wide tiles, the last 34 as 68 column slices (SH_GEMM_PAIR_BN=256: 512 narrow tiles)
    M3, N3, K3 = 8192, 4096, 2048
    a3, w3, z3 = rt.alloc(M3, K3), rt.alloc(K3, N3), rt.alloc(M3, N3)
    lib.sh_test_fill_fp16(a3, M3, K3, K3, 7, -1024, 1023, 1.0 / 1024)
    lib.sh_test_fill_fp16(w3, K3, N3, N3, 8, -1024, 1023, 1.0 / 1024)
    if lib.sh_cuda_gemm(a3, w3, z3, M3, N3, K3, K3, N3, N3, 0, 0, N3, 0, 0):
        raise RuntimeError(lib.sh_cuda_last_error_string().decode())
    rt.check()
    tail = rt.get(z3, M3, N3)
    h = lambda t: hashlib.sha1(np.ascontiguousarray(t).view(np.uint8).tobytes()).hexdigest()  # noqa: E731
    print(f"HASH {h(enc)} {h(gem)} {h(wide)} {h(tail)}", flush=True)


if __name__ == "__main__":
    main()
