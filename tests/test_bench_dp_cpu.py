"""The data-parallel encoder's host-side plumbing on gloo ranks (CPU): the batch split and per-rank input seeds,
and the rank-max timing that bench.py's whole-job images/s is computed from. The GPU step itself is covered by the
-m gpu tests; here two and four ranks check that every rank agrees on the slowest rank's time and the job rate."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    for p in (str(ROOT), str(ROOT / "softhier-mlir_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        assert bench.dist_env() == (rank, world, 0)
        B, seed = bench.encoder_shard(world, rank)
        local_ms = 100.0 + 7.0 * rank                 # rank r's timed region took 100 + 7 r ms
        bench.barrier(world)
        ms, value = bench.job_rate(local_ms, 40, world)
        got = [None] * world
        dist.all_gather_object(got, (rank, B, seed, ms, value))
        if rank == 0:
            q.put(got)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_dp_shard_and_rank_max_timing(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(q.get(timeout=10))
    sys.path.insert(0, str(ROOT))
    import bench
    assert sum(B for _, B, _, _, _ in got) == bench.GLOBAL_BATCH            # the shards cover the batch
    assert len({seed for _, _, seed, _, _ in got}) == world                 # each rank its own input shard
    slowest = 100.0 + 7.0 * (world - 1)
    for _, B, _, ms, value in got:
        assert B == bench.GLOBAL_BATCH // world
        assert ms == slowest                                                # every rank sees the slowest rank
        assert value == pytest.approx(bench.GLOBAL_BATCH * 40 / (slowest / 1e3))


def test_batch_must_split_evenly():
    sys.path.insert(0, str(ROOT))
    import bench
    with pytest.raises(SystemExit):
        bench.encoder_shard(3, 0)
