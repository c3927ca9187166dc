"""SUMMA on the GPU: bit-exact block generation, the panel pipeline on one GPU, and the multi-GPU run (2+ GPUs,
as torch.distributed ranks over NCCL with IPC panel pulls)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import lcg
from softhier_cuda import summa as SU

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_lcg_block_fill_is_a_slice_of_the_global_fill(gpu_lib):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    R, C = 300, 500
    full = lcg.fill_fp16(R, C, 77, -1024, 1023, 1 / 1024)
    for r0, c0, rows, cols in [(0, 0, 300, 500), (17, 33, 100, 200), (299, 499, 1, 1), (64, 256, 128, 244)]:
        a = rt.alloc(rows, cols + 3)
        lib.sh_cuda_fill_lcg_block(a, rows, cols, cols + 3, 77, -1024, 1023, 1 / 1024, r0, c0, C)
        rt.check()
        got = rt.get(a, rows, cols, cols + 3)
        assert (got.view(np.uint16) == full[r0:r0 + rows, c0:c0 + cols].view(np.uint16)).all()


@pytest.mark.parametrize("kb", [2048, 512])
def test_summa_single_gpu_panels(gpu_lib, kb):
    rt, lib = gpu_lib, gpu_lib.lib
    n = 2048
    lay = SU.Layout(n, n, n, 1, 1, kb)
    su = SU.SummaGPU(lib, lay, 0, lambda x: [x], lambda: None, (torch.cuda.Stream(), torch.cuda.Stream()))
    try:
        su.fill_inputs(5, 6)
        for _ in range(2):
            assert su.step(torch) == 0
        torch.cuda.synchronize()
        rt.check()
        c = torch.empty((n, n), dtype=torch.float16, device="cuda")
        lib.sh_cuda_copy2d(c.data_ptr(), n * 2, su.c, n * 2, n * 2, n, None)
        torch.cuda.synchronize()
        want = lcg.uniform_fp16(n, n, 5).astype(np.float32) @ lcg.uniform_fp16(n, n, 6).astype(np.float32)
        err = np.abs(c.cpu().numpy().astype(np.float32) - want)
        assert np.all(err <= 2e-2 + 2.0 ** -10 * np.abs(want)), float(err.max())
    finally:
        su.close()


@pytest.mark.parametrize("kb", [16384, 4096])
def test_summa_config4_size_sampled(gpu_lib, capfd, kb):
    """BASELINE config 4 at full size on one GPU (16384^3, uniform [-1, 1) from the LCG): the block fill is
    bit-exact on sampled rows of A, and 64 sampled outputs match float64 dot products of the stored operands within
    half an fp16 ulp of the result plus 2e-3; the reference's own sampled check (sh_test_check_gemm,
    runtime/sh_test.inc.c:32-51) passes on 256 more positions. kb = 4096 carries the sum over four panels in fp32."""
    lib = gpu_lib.lib
    n = 16384
    lay = SU.Layout(n, n, n, 1, 1, kb)
    su = SU.SummaGPU(lib, lay, 0, lambda x: [x], lambda: None, (torch.cuda.Stream(), torch.cuda.Stream()))
    try:
        su.fill_inputs(5, 6)
        assert su.step(torch) == 0
        torch.cuda.synchronize()
        gpu_lib.check()

        def dev(addr, rows, cols, ld):
            t = torch.empty((rows, cols), dtype=torch.float16, device="cuda")
            lib.sh_cuda_copy2d(t.data_ptr(), cols * 2, addr, ld * 2, cols * 2, rows, None)
            torch.cuda.synchronize()
            return t.cpu().numpy()

        rng = np.random.default_rng(4)
        rows = rng.integers(0, n, 8)
        cols = rng.integers(0, n, 8)
        for r in rows[:3]:
            want = lcg.uniform_fp16(1, n, 5, row0=int(r))
            assert np.array_equal(dev(su.a_loc + 2 * int(r) * n, 1, n, n).view(np.uint16), want.view(np.uint16))
        a_rows = {int(r): dev(su.a_loc + 2 * int(r) * n, 1, n, n)[0].astype(np.float64) for r in rows}
        b_cols = {int(c): dev(su.b_loc + 2 * int(c), n, 1, n)[:, 0].astype(np.float64) for c in cols}
        worst = 0.0
        for r in a_rows:
            zrow = dev(su.c + 2 * r * n, 1, n, n)[0].astype(np.float64)
            for c in b_cols:
                want = float(a_rows[r] @ b_cols[c])
                ulp = 2.0 ** (np.floor(np.log2(max(abs(want), 2.0 ** -14))) - 10)
                err = abs(zrow[c] - want)
                worst = max(worst, err / (0.5 * ulp + 2e-3))
                assert err <= 0.5 * ulp + 2e-3, (r, c, zrow[c], want)
        capfd.readouterr()
        lib.sh_cuda_set_stream(None)
        bad = lib.sh_test_check_gemm(su.a_loc, su.b_loc, su.c, n, n, n, n, n, n, 256, 0.25, 0.0, b"[summa16384]")
        gpu_lib.activate()
        out = capfd.readouterr().out
        assert bad == 0 and "[summa16384] samples=256 bad=0" in out, out
        print(f"config 4 sampled: worst error / bound {worst:.3f}")
    finally:
        torch.cuda.synchronize()
        su.close()
        gpu_lib.activate()


# panel width 128: every panel one piece per operand; 512 = n / 2: on 2x4 each A panel spans two owners' blocks;
# 1024 = n (the default): one panel per step, pulled during the previous step's GEMM
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("kb", [128, 512, 1024])
def test_summa_multi_gpu(kb):
    world = 8 if torch.cuda.device_count() >= 8 else (4 if torch.cuda.device_count() >= 4 else 2)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SUMMA_KB=str(kb))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={29533 + kb % 7}",
           str(ROOT / "tests" / "summa_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=360)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("SUMMA_OK") == world, r.stdout
