"""tcgen05 GEMM through the C ABI against the fp32 oracle, the reference's KATs and its error conventions."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import lcg, ops
from softhier_cuda import lib as L

pytestmark = pytest.mark.gpu


def _close(got, want, K):
    """fp16 output of an fp32-accumulated dot product: within 2e-2 + one fp16 ulp of the magnitude."""
    got = np.asarray(got, np.float32)
    err = np.abs(got - want)
    lim = 2e-2 + 2.0 ** -10 * np.abs(want)
    assert np.all(err <= lim), (float(err.max()), K)


def _run(rt, M, N, K, flags=0, splits=0, ldx=None, ldw=None, ldz=None, seed=1, off=(0, 0, 0)):
    lib = rt.lib
    rt.reset()
    ldx, ldw, ldz = ldx or K, ldw or N, ldz or N
    x = lcg.uniform_fp16(M, ldx, seed)
    w = lcg.uniform_fp16(K, ldw, seed + 1)
    z0 = lcg.uniform_fp16(M, ldz, seed + 2)
    bias = lcg.normal_fp16(1, N, seed + 3, 0.0, 0.5)
    res = lcg.normal_fp16(M, N, seed + 4)
    dx = rt.upload(x) + 2 * off[0]
    dw = rt.upload(w) + 2 * off[1]
    dz = rt.upload(z0) + 2 * off[2]
    db, dr = rt.upload(bias), rt.upload(res)
    rc = lib.sh_cuda_gemm(dx, dw, dz, M, N, K, ldx, ldw, ldz, db, dr, N, flags, splits)
    assert rc == 0
    rt.check()
    got = rt.get(dz, M, N, ldz)
    xs = x[:, off[0]:off[0] + K]
    ws = w[:K, off[1]:off[1] + N] if off[1] else w[:, :N]
    acc = ops.gemm(xs, ws)
    if flags & L.EPI_ACCUMULATE:
        acc = acc + z0[:, off[2]:off[2] + N].astype(np.float32)
    if flags & L.EPI_BIAS:
        acc = acc + bias.astype(np.float32)
    if flags & L.EPI_GELU:
        acc = ops.gelu(acc)
    if flags & L.EPI_RESIDUAL:
        acc = acc + res.astype(np.float32)
    return got, acc


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (256, 768, 768), (256, 3072, 768), (256, 768, 3072),
                                   (1024, 2304, 768), (128, 64, 64), (256, 256, 64), (256, 64, 256)])
def test_gemm_matches_fp32(gpu_lib, M, N, K):
    got, want = _run(gpu_lib, M, N, K)
    _close(got, want, K)
    if (M, N, K) == (512, 512, 512):
        err, rel = ops.max_abs_and_rel_l2(got, want)
        assert err <= 2e-2 and rel <= 5e-3, (err, rel)


@pytest.mark.parametrize("splits", [1, 2, 3, 8])
def test_split_k_equals_unsplit(gpu_lib, splits):
    got, want = _run(gpu_lib, 256, 512, 2048, splits=splits)
    _close(got, want, 2048)


@pytest.mark.parametrize("flags", [L.EPI_ACCUMULATE, L.EPI_BIAS, L.EPI_BIAS | L.EPI_GELU,
                                   L.EPI_BIAS | L.EPI_RESIDUAL, L.EPI_ACCUMULATE | L.EPI_BIAS | L.EPI_RESIDUAL])
@pytest.mark.parametrize("splits", [1, 4])
def test_fused_epilogues(gpu_lib, flags, splits):
    got, want = _run(gpu_lib, 384, 768, 1024, flags=flags, splits=splits)
    _close(got, want, 1024)


@pytest.mark.parametrize("M,N,K", [(50, 1600, 720), (200, 720, 2048), (130, 100, 70), (1, 8, 8), (300, 40, 1000)])
def test_ragged_shapes(gpu_lib, M, N, K):
    got, want = _run(gpu_lib, M, N, K)
    _close(got, want, K)


def test_strided_views(gpu_lib):
    # X a column slice of a wider buffer (ld 4096, the xmcast test's view), W and Z with padded leading dims
    got, want = _run(gpu_lib, 200, 720, 2048, ldx=4096, ldw=728, ldz=736, off=(8, 0, 8))
    _close(got, want, 2048)


def test_unaligned_views_use_fallback(gpu_lib):
    # element offsets that break 16-byte alignment: the CUDA-core path must give the same numbers
    got, want = _run(gpu_lib, 96, 72, 136, ldx=141, ldw=77, ldz=75, off=(3, 1, 2))
    _close(got, want, 136)


def test_simt_flag_matches_tensor_cores(gpu_lib):
    a, want = _run(gpu_lib, 256, 512, 512, flags=L.GEMM_SIMT)
    b, _ = _run(gpu_lib, 256, 512, 512)
    _close(a, want, 512)
    _close(b, want, 512)


def test_kat_gemm512_constant(gpu_lib, capfd):
    """examples/gemm512.mlir: X = 1.0, W = 1/512 -> Z == 1.0 within 16 ulp."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    x, w, z = rt.alloc(512, 512), rt.alloc(512, 512), rt.alloc(512, 512)
    lib.sh_test_fill_const_fp16(x, 512, 512, 512, 15360)
    lib.sh_test_fill_const_fp16(w, 512, 512, 512, 6144)
    cfg = L.cfg(0, 0, 0, 0, 0, L.SH_FP16, 0)
    assert lib.sh_gemm(x, w, z, 512, 512, 512, 512, 512, 512, cfg, 0) == 0
    assert lib.sh_test_check_const_fp16(z, 512, 512, 512, 15360, 16, b"GEMM512") == 512 * 512
    assert "GEMM512_CHECK ok=262144/262144 GEMM512_PASS" in capfd.readouterr().out


def test_kat_gemm_nonconst_colparity(gpu_lib):
    """examples/gemm_nonconst.mlir: X even cols 1.0 / odd cols 0.5, W = 1/512 -> Z == 0.75 (0x3A00)."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    x, w, z = rt.alloc(512, 512), rt.alloc(512, 512), rt.alloc(512, 512)
    lib.sh_test_fill_colparity_fp16(x, 512, 512, 512, 15360, 14336)
    lib.sh_test_fill_const_fp16(w, 512, 512, 512, 6144)
    assert lib.sh_gemm(x, w, z, 512, 512, 512, 512, 512, 512, None, 0) == 0
    assert lib.sh_test_check_const_fp16(z, 512, 512, 512, 14848, 16, b"NC") == 512 * 512


def test_kat_summa1024_single_process(gpu_lib):
    """examples/gemm1024_summa.mlir through sh_gemm_mesh: X = 1.0, W = 1/1024 -> Z == 1.0."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    x, w, z = rt.alloc(1024, 1024), rt.alloc(1024, 1024), rt.alloc(1024, 1024)
    lib.sh_test_fill_const_fp16(x, 1024, 1024, 1024, 15360)
    lib.sh_test_fill_const_fp16(w, 1024, 1024, 1024, 5120)
    assert lib.sh_gemm_mesh(x, w, z, 1024, 1024, 1024, 1024, 1024, 1024, None) == 0
    assert lib.sh_test_check_const_fp16(z, 1024, 1024, 1024, 15360, 16, b"S") == 1024 * 1024


def test_reference_accumulate_cfg(gpu_lib):
    """sh_gemm with cfg.accumulate = 1 (gemm/main.c: Z0 = 3.0, int data -1..1 / -2..2, tol 0.5)."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    M, N, K = 256, 256, 512
    x, w, z = rt.alloc(M, K), rt.alloc(K, N), rt.alloc(M, N)
    lib.sh_test_fill_int_fp16(x, M, K, K, 1, -1, 1)
    lib.sh_test_fill_int_fp16(w, K, N, N, 2, -2, 2)
    lib.sh_test_fill_int_fp16(z, M, N, N, 3, 3, 3)
    cfg = L.cfg(256, 256, 256, 1, 1, L.SH_FP16, 0)
    assert lib.sh_gemm(x, w, z, M, N, K, K, N, N, cfg, L.SH_ALL) == 0
    assert lib.sh_test_check_gemm(x, w, z, M, N, K, K, N, N, 256, 0.5, 3.0, b"[gemm]") == 0


def test_error_codes_match_reference(gpu_lib, capfd):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    x, w, z = rt.alloc(300, 256), rt.alloc(256, 256), rt.alloc(300, 256)
    capfd.readouterr()
    assert lib.sh_gemm(x, w, z, 300, 256, 256, 256, 256, 256, None, 0) == -1        # 300 % 256
    assert "[sh_gemm] shape 300x256x256 not divisible by tile 256x256x256" in capfd.readouterr().out
    cfg = L.cfg(0, 0, 0, 1, 0, L.SH_FP8, 0)
    assert lib.sh_gemm(x, w, z, 256, 256, 256, 256, 256, 256, cfg, 0) == -3
    cfg = L.cfg(128, 0, 0, 1, 0, 0, 0)                                                 # 300 % 128 rows per block
    assert lib.sh_gemm_xmcast_ex(x, w, z, 300, 256, 256, 256, 256, 256, cfg, L.SH_XM_AUTO) == -1
    cfg = L.cfg(64, 128, 0, 1, 0, 0, 0)
    assert lib.sh_gemm_mesh(x, w, z, 256, 256, 256, 256, 256, 256, cfg) == -1        # tm != tn
    assert lib.sh_cuda_last_error() != 0
    assert lib.sh_cuda_last_error() == 0                                             # cleared after reading
    assert lib.sh_gemm_l1_bytes(131072, 768, 768, None) <= lib.sh_l1_size()


def test_xmcast_small_m(gpu_lib):
    """sh_gemm_xmcast_ex on the gemm_xmcast_translate.mlir shapes: 50 x 1600 x 720 and a strided 200 x 720 x 2048."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    for M, N, K, ldx, mode in [(50, 1600, 720, 720, L.SH_XM_AUTO), (200, 720, 2048, 4096, L.SH_XM_PANEL)]:
        x = lcg.uniform_fp16(M, ldx, 3)
        w = lcg.uniform_fp16(K, N, 4)
        dx, dw, dz = rt.upload(x), rt.upload(w), rt.alloc(M, N)
        cfg = L.cfg(M, 0, 0, 1, 0, 0, 0)
        assert lib.sh_gemm_xmcast_ex(dx, dw, dz, M, N, K, ldx, N, N, cfg, mode) == 0
        rt.check()
        _close(rt.get(dz, M, N), ops.gemm(x[:, :K], w), K)


def test_fp32_carried_k_split(gpu_lib):
    """SH_EPI_F32_OUT / SH_EPI_ACC_F32_IN: a K = 3 x 1024 product done as three calls with the running sum kept in
    fp32 equals the one-call product to within one final fp16 rounding."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    M, N, Kp = 256, 384, 1024
    xs = [lcg.uniform_fp16(M, Kp, 50 + i) for i in range(3)]
    ws = [lcg.uniform_fp16(Kp, N, 60 + i) for i in range(3)]
    dx = [rt.upload(x) for x in xs]
    dw = [rt.upload(w) for w in ws]
    acc = rt.alloc_bytes(M * N * 4)
    z = rt.alloc(M, N)
    assert lib.sh_cuda_gemm(dx[0], dw[0], acc, M, N, Kp, Kp, N, N, 0, 0, 0, L.EPI_F32_OUT, 0) == 0
    assert lib.sh_cuda_gemm(dx[1], dw[1], acc, M, N, Kp, Kp, N, N, 0, 0, 0, L.EPI_F32_OUT | L.EPI_ACCUMULATE, 2) == 0
    assert lib.sh_cuda_gemm(dx[2], dw[2], z, M, N, Kp, Kp, N, N, 0, acc, N, L.EPI_ACC_F32_IN, 0) == 0
    rt.check()
    want = sum(ops.gemm(x, w) for x, w in zip(xs, ws))
    _close(rt.get(z, M, N), want, 3 * Kp)
    err = np.abs(rt.get(z, M, N).astype(np.float32) - want)
    assert float(err.max()) <= 2.0 ** -10 * float(np.abs(want).max()) + 1e-3


@pytest.mark.parametrize("M,N,K,flags", [(8192, 768, 768, 0), (8192, 2304, 768, L.EPI_BIAS),
                                         (8000, 768, 3072, L.EPI_BIAS | L.EPI_RESIDUAL),
                                         (8192, 3072, 768, L.EPI_BIAS | L.EPI_GELU), (9984, 1024, 640, 0),
                                         (2816, 4096, 256, L.EPI_BIAS),
                                         (6400, 768, 768, L.EPI_BIAS | L.EPI_RESIDUAL),
                                         (8192, 768, 768, L.EPI_ACCUMULATE | L.EPI_BIAS | L.EPI_RESIDUAL),
                                         (7936, 1536, 512, L.EPI_RESIDUAL), (8192, 768, 832, L.EPI_BIAS),
                                         (8192, 1536, 1024, L.EPI_ACCUMULATE | L.EPI_BIAS),
                                         (8192, 904, 768, L.EPI_BIAS | L.EPI_RESIDUAL)])
def test_pair_tiles(gpu_lib, M, N, K, flags):
    """Shapes with enough 256 x 256 tiles run on the 2-CTA (cta_group::2) kernel. 9984 and 2816 rows (39 and 11
    row-tiles) end with a partial group of the grouped tile order, 2816 x 4096 with 16 column-tiles per row. Without a
    residual an even k-block count runs with one barrier per two stages (K = 256, 640, 768, 1024), an odd one (K = 832:
    13 k-blocks) with one per stage. With a residual the residual tiles come in by TMA beside the epilogue's store
    slots: 8000 rows end in a partial row-tile, 6400 x 768 (75 tiles on 74 SM pairs) leaves most pairs a single tile,
    accumulate adds Z on top, and at N = 904 the last column tile's second half has one 32-column chunk inside N and
    three past it (no stores for those)."""
    got, want = _run(gpu_lib, M, N, K, flags=flags)
    _close(got, want, K)


# Shapes the planner gives 256 x 512 pair tiles (N % 512 == 0, K >= 2048, and cheaper waves on 74 SM pairs):
# 4096 x 4096, 2816 x 2048 (11 row-tiles, ragged), 4096 x 2048; 8192 / 8000 x 4096 have 256 wide tiles, 3 full waves
# and a tail of 34 that runs as 68 256-column slices.
@pytest.mark.parametrize("M,N,K,flags", [(4096, 4096, 2048, 0), (2816, 2048, 4096, L.EPI_BIAS | L.EPI_RESIDUAL),
                                         (4096, 2048, 2048, L.EPI_ACCUMULATE | L.EPI_BIAS),
                                         (8192, 4096, 2048, L.EPI_BIAS | L.EPI_RESIDUAL), (8000, 4096, 2048, 0)])
def test_wide_pair_tiles(gpu_lib, M, N, K, flags):
    got, want = _run(gpu_lib, M, N, K, flags=flags)
    _close(got, want, K)


def test_wide_pair_tiles_fp32_carry(gpu_lib):
    """The SUMMA panel pattern on 256 x 512 tiles: fp32 out, then fp32 carry-in rounded to fp16 once."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    M, N, Kp = 4096, 2048, 2048
    xs = [lcg.uniform_fp16(M, Kp, 70 + i) for i in range(2)]
    ws = [lcg.uniform_fp16(Kp, N, 80 + i) for i in range(2)]
    dx = [rt.upload(x) for x in xs]
    dw = [rt.upload(w) for w in ws]
    acc = rt.alloc_bytes(M * N * 4)
    z = rt.alloc(M, N)
    assert lib.sh_cuda_gemm(dx[0], dw[0], acc, M, N, Kp, Kp, N, N, 0, 0, 0, L.EPI_F32_OUT, 1) == 0
    assert lib.sh_cuda_gemm(dx[1], dw[1], z, M, N, Kp, Kp, N, N, 0, acc, N, L.EPI_ACC_F32_IN, 1) == 0
    rt.check()
    want = sum(ops.gemm(x, w) for x, w in zip(xs, ws))
    _close(rt.get(z, M, N), want, 2 * Kp)
