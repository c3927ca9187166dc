"""One rank of the multi-GPU SUMMA check, launched by tests/test_summa_gpu.py under torch.distributed.run:
every rank generates its own LCG blocks on its GPU, runs the SUMMA steps, and compares its C block with the
numpy product of the same slices of the global matrices. Prints `SUMMA_OK rank max_err` or raises."""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "softhier-mlir_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import lcg  # noqa: E402
from softhier_cuda import summa as SU  # noqa: E402
from softhier_cuda.runtime import Runtime  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        pr, pc = SU.default_grid(world)
        n = int(os.environ.get("SUMMA_N", "1024"))
        lay = SU.Layout(n, n, n, pr, pc, int(os.environ.get("SUMMA_KB", "128")))
        rt = Runtime.open(local, arena_bytes=64 << 20)

        def exchange(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        su = SU.SummaGPU(rt.lib, lay, rank, exchange, dist.barrier, (torch.cuda.Stream(), torch.cuda.Stream()))
        su.fill_inputs(31, 32)
        # three steps: the second reuses the panel slots, and the first two pull the next step's first panel
        # early (prefetch_next), so the last one runs on a prefetched panel 0
        for k in range(3):
            assert su.step(torch, prefetch_next=k < 2) == 0
        su.finish(torch)
        torch.cuda.synchronize()
        rt.check()
        i, j = lay.coords(rank)
        c = torch.empty((lay.Mb, lay.Nb), dtype=torch.float16, device="cuda")
        rt.lib.sh_cuda_copy2d(c.data_ptr(), lay.Nb * 2, su.c, lay.Nb * 2, lay.Nb * 2, lay.Mb, None)
        torch.cuda.synchronize()
        A = lcg.uniform_fp16(n, n, 31).astype(np.float32)
        B = lcg.uniform_fp16(n, n, 32).astype(np.float32)
        want = A[i * lay.Mb:(i + 1) * lay.Mb] @ B[:, j * lay.Nb:(j + 1) * lay.Nb]
        err = float(np.abs(c.cpu().numpy().astype(np.float32) - want).max())
        lim = 2e-2 + 2.0 ** -10 * float(np.abs(want).max())
        if err > lim:
            raise AssertionError(f"rank {rank}: max err {err} > {lim}")
        dist.barrier()
        su.close()
        print(f"SUMMA_OK {rank} {err:.4g}", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
