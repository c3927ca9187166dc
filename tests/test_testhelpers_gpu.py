"""On-device test helpers (sh_test.inc.c) against the oracle: LCG fills are bit-exact, dumps use the reference's
line format and positions."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import lcg

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("args", [(64, 96, 7, -16, 16, 0.125), (256, 768, 1, -16, 16, 0.125),
                                  (33, 17, 5, -1024, 1023, 1 / 1024), (1000, 1000, 99, -8, 8, 1 / 128)])
def test_device_fill_is_bit_exact(gpu_lib, args):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    r, c, seed, lo, hi, sc = args
    ld = c + 5
    a = rt.alloc(r, c, ld)
    lib.sh_test_fill_fp16(a, r, c, ld, seed, lo, hi, sc)
    rt.check()
    got = rt.get(a, r, c, ld)
    assert (got.view(np.uint16) == lcg.fill_fp16(r, c, seed, lo, hi, sc).view(np.uint16)).all()


def test_const_and_colparity_fills_and_check(gpu_lib, capfd):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    a = rt.alloc(16, 40)
    lib.sh_test_fill_colparity_fp16(a, 16, 40, 40, 15360, 14336)
    rt.check()
    assert (rt.get(a, 16, 40).view(np.uint16) == lcg.colparity_fp16(16, 40, 15360, 14336).view(np.uint16)).all()
    lib.sh_test_fill_const_fp16(a, 16, 40, 40, 0x3C00)
    ok = lib.sh_test_check_const_fp16(a, 16, 40, 40, 0x3C00, 0, b"K")
    assert ok == 640
    assert "K_CHECK ok=640/640 K_PASS" in capfd.readouterr().out


def test_dump_samples_format(gpu_lib, capfd):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    x = lcg.fill_fp16(50, 70, 3, -16, 16, 0.125)
    a = rt.upload(x)
    capfd.readouterr()
    lib.sh_test_dump_samples(a, 50, 70, 70, 42, 16, b"T")
    lib.sh_test_dump_samples_idx(a, 50, 70, 70, 42, 4, b"L", 3)
    out = capfd.readouterr().out
    got = lcg.parse_samples(out)
    assert [(r, c) for r, c, _ in got["T"]] == lcg.sample_positions(50, 70, 42, 16)
    assert len(got["L3"]) == 4
    bad, err = lcg.compare_samples(got["T"], x.astype(np.float32), 0.0, 0.0)
    assert bad == 0


def test_check_gemm_helper(gpu_lib, capfd):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    M, N, K = 256, 256, 512
    x, w = rt.alloc(M, K), rt.alloc(K, N)
    z = rt.alloc(M, N)
    lib.sh_test_fill_int_fp16(x, M, K, K, 1, -1, 1)
    lib.sh_test_fill_int_fp16(w, K, N, N, 2, -2, 2)
    assert lib.sh_gemm(x, w, z, M, N, K, K, N, N, None, 0) == 0
    bad = lib.sh_test_check_gemm(x, w, z, M, N, K, K, N, N, 128, 0.5, 0.0, b"[gemm]")
    assert bad == 0
    assert "[gemm] samples=128 bad=0" in capfd.readouterr().out


def test_preload_elf_into_arena(gpu_lib):
    """An image written by the reference's sim/preload.make_preload_elf lands at sh_hbm_addr(offset)."""
    from pathlib import Path
    import numpy as np
    from conftest import golden
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    rt.arena.zero_()
    g = golden("preload_small.npz")
    path = Path(__file__).resolve().parent / "golden" / "preload_small.elf"
    assert lib.sh_cuda_preload_elf(str(path).encode(), 0xC0000000) == len(g["offsets"])
    for off in g["offsets"]:
        seg = g[f"seg_{int(off):x}"]
        got = rt.arena[int(off):int(off) + len(seg)].cpu().numpy()
        np.testing.assert_array_equal(got, seg)
    lib.sh_preload_wait(lib.sh_hbm_addr(int(g["offsets"][-1])))
    rt.check()


def test_normal_fill_is_bit_exact_with_the_oracle(gpu_lib):
    """sh_cuda_fill_normal_fp16 on the device == oracle.lcg.normal_fp16 for every element (strided destination,
    a chunk boundary inside a row, a non-default mean / std), and leaves the padding columns alone."""
    import numpy as np

    from oracle import lcg
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    for rows, cols, seed, mean, std in ((300, 77, 5, 0.0, 1.0), (768, 2304, 7000, 0.0, 0.02), (5, 4099, 3, 1.0, 0.5)):
        ld = cols + 13
        a = rt.alloc(rows, ld)
        rt.view(a, rows, ld).fill_(7.0)
        lib.sh_cuda_fill_normal_fp16(a, rows, cols, ld, seed, mean, std)
        got = rt.get(a, rows, ld, ld)
        want = lcg.normal_fp16(rows, cols, seed, mean, std)
        assert np.array_equal(got[:, :cols].view(np.uint16), want.view(np.uint16)), (rows, cols, seed)
        assert (got[:, cols:] == 7.0).all()
    rt.check()
