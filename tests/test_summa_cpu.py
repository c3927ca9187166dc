"""SUMMA host logic: the panel schedule reproduces A B on every grid, and runs on real gloo ranks (world size 2 / 4)
with blocks exchanged between processes."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from softhier_cuda import summa as SU


def _blocks(lay, A, B):
    a, b = {}, {}
    for r in range(lay.pr * lay.pc):
        i, j = lay.coords(r)
        a[r] = A[i * lay.Mb:(i + 1) * lay.Mb, j * lay.Kc:(j + 1) * lay.Kc]
        b[r] = B[i * lay.Kr:(i + 1) * lay.Kr, j * lay.Nb:(j + 1) * lay.Nb]
    return a, b


# panel widths below, equal to and above the owners' block widths (K / pc, K / pr): panels of several pieces too
@pytest.mark.parametrize("grid,kb", [((1, 1), 32), ((1, 2), 16), ((2, 2), 16), ((2, 4), 8), ((4, 2), 8),
                                     ((2, 3), 8), ((2, 4), 48), ((2, 4), 24), ((1, 2), 96), ((4, 2), 32),
                                     ((2, 3), 32)])
def test_schedule_reproduces_matmul(grid, kb):
    pr, pc = grid
    M, N, K = 48 * pr, 40 * pc, 96
    lay = SU.Layout(M, N, K, pr, pc, kb)
    rng = np.random.default_rng(1)
    A, B = rng.standard_normal((M, K)).astype(np.float32), rng.standard_normal((K, N)).astype(np.float32)
    a, b = _blocks(lay, A, B)
    C = np.zeros((M, N), np.float32)
    for r in range(pr * pc):
        i, j = lay.coords(r)
        sched = SU.panel_schedule(lay, r)
        assert sorted(p.k0 for p in sched) == list(range(0, K, kb))          # every panel exactly once
        assert any(q.rank == r for q in sched[0].a)                          # starts with its own A block
        for p in sched:
            for pieces, block, axis in ((p.a, lay.Kc, 0), (p.b, lay.Kr, 1)):
                # pieces tile the panel in K order, each inside its owner's block, owners in this grid row / column
                assert [q.dst for q in pieces] == list(np.cumsum([0] + [q.width for q in pieces[:-1]]))
                assert sum(q.width for q in pieces) == kb
                assert all(0 <= q.src and q.src + q.width <= block for q in pieces)
                assert all(lay.coords(q.rank)[axis] == (i if axis == 0 else j) for q in pieces)
        C[i * lay.Mb:(i + 1) * lay.Mb, j * lay.Nb:(j + 1) * lay.Nb] = SU.summa_numpy(lay, r, a, b)
    np.testing.assert_allclose(C, A @ B, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("kb", [16384, 8192, 4096])
def test_panel_peer_bytes_match_the_survey_figure(kb):
    # config 4 on 2x4, any panel width: (M/pr) K 2 (pc-1)/pc + K (N/pc) 2 (pr-1)/pr = 201 + 67 MB per GPU
    n = 16384
    lay = SU.Layout(n, n, n, 2, 4, kb)
    want = (n // 2) * n * 2 * 3 // 4 + n * (n // 4) * 2 // 2
    assert all(SU.panel_peer_bytes(lay, r) == want for r in range(8))
    assert SU.panel_peer_bytes(SU.Layout(n, n, n, 1, 1, n), 0) == 0


def test_layout_rejects_bad_splits():
    with pytest.raises(ValueError):
        SU.Layout(100, 64, 64, 3, 1, 16).check()
    with pytest.raises(ValueError):
        SU.Layout(64, 64, 96, 1, 2, 36).check()      # 36 does not divide K = 96
    assert SU.default_grid(8) == (2, 4) and SU.default_grid(2) == (1, 2)
    assert SU.default_panel(16384, 1) == 16384 and SU.default_panel(16384, 8) == 16384


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, grid, out_q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import lcg
        pr, pc = grid
        lay = SU.Layout(64 * pr, 32 * pc, 128, pr, pc, 32)
        A = lcg.uniform_fp16(lay.M, lay.K, 7).astype(np.float32)        # every rank sees only its own block
        B = lcg.uniform_fp16(lay.K, lay.N, 8).astype(np.float32)
        i, j = lay.coords(rank)
        mine = (rank, A[i * lay.Mb:(i + 1) * lay.Mb, j * lay.Kc:(j + 1) * lay.Kc],
                B[i * lay.Kr:(i + 1) * lay.Kr, j * lay.Nb:(j + 1) * lay.Nb])
        got = [None] * world
        dist.all_gather_object(got, mine)
        a = {r: blk_a for r, blk_a, _ in got}
        b = {r: blk_b for r, _, blk_b in got}
        c = SU.summa_numpy(lay, rank, a, b)
        cs = [None] * world
        dist.all_gather_object(cs, (rank, c))
        if rank == 0:
            C = np.zeros((lay.M, lay.N), np.float32)
            for r, blk in cs:
                ii, jj = lay.coords(r)
                C[ii * lay.Mb:(ii + 1) * lay.Mb, jj * lay.Nb:(jj + 1) * lay.Nb] = blk
            out_q.put(float(np.abs(C - A @ B).max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,grid", [(2, (1, 2)), (4, (2, 2))])
def test_gloo_ranks_run_the_schedule(world, grid):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, grid, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=10) < 1e-3
