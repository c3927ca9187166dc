"""2-D block-distributed SUMMA GEMM across the GPUs of one node: the multi-GPU form of sh_gemm_mesh
(runtime/sh_gemm.inc.c:120-189, mesh-wide output-stationary SUMMA with diagonal-owner panel broadcasts).

Rank (i, j) of a pr x pc grid (rank = i * pc + j) owns, of C = A B with A [M, K], B [K, N]:
    A_ij = A[i Mb:(i+1) Mb, j Kc:(j+1) Kc]     Mb = M / pr, Kc = K / pc
    B_ij = B[i Kr:(i+1) Kr, j Nb:(j+1) Nb]     Kr = K / pr, Nb = N / pc
    C_ij = C[i Mb:(i+1) Mb, j Nb:(j+1) Nb]  =  sum over K-panels k of  A[i-rows, k] B[k, j-cols]
The A panel of K-panel k lives on rank (i, k // Kc) (this rank's grid row), the B panel on rank (k // Kr, j) (its
grid column). Instead of the reference's row / column multicasts, every rank PULLS the two panels it needs with the
copy engines (CUDA IPC mappings of the owners' blocks + cudaMemcpy2DAsync on a copy stream: no SM is spent on the
transfer), into double-buffered local panels, while the tcgen05 GEMM of the previous panel runs on the compute stream
(C_ij += A_panel B_panel through the accumulate epilogue, carried in fp32 between panels and rounded to fp16 by the
last one). Inputs are read-only during a step, so the step needs no
cross-GPU synchronisation; ranks start at different panels (their own A panel first) to spread the pulls over the
owners.

`panel_schedule` is the host-side logic shared by the GPU driver (`SummaGPU`) and the numpy reference driver used by
the multi-process CPU tests (`summa_numpy`).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import lib as L


@dataclass(frozen=True)
class Layout:
    M: int
    N: int
    K: int
    pr: int
    pc: int
    kb: int

    @property
    def Mb(self) -> int:
        return self.M // self.pr

    @property
    def Nb(self) -> int:
        return self.N // self.pc

    @property
    def Kc(self) -> int:
        return self.K // self.pc

    @property
    def Kr(self) -> int:
        return self.K // self.pr

    def check(self) -> None:
        if self.M % self.pr or self.N % self.pc or self.K % self.pc or self.K % self.pr:
            raise ValueError(f"{self.M}x{self.N}x{self.K} does not split over a {self.pr}x{self.pc} grid")
        if self.Kc % self.kb or self.Kr % self.kb:
            raise ValueError(f"panel width {self.kb} must divide K/pc = {self.Kc} and K/pr = {self.Kr}")

    def coords(self, rank: int) -> tuple[int, int]:
        return divmod(rank, self.pc)

    def rank_of(self, i: int, j: int) -> int:
        return i * self.pc + j


@dataclass(frozen=True)
class Panel:
    k0: int            # first K index of the panel
    a_rank: int        # owner of A[i-rows, k0:k0+kb]
    a_col: int         # its column offset inside the owner's A block
    b_rank: int        # owner of B[k0:k0+kb, j-cols]
    b_row: int         # its row offset inside the owner's B block


def default_grid(world: int) -> tuple[int, int]:
    """1 -> 1x1, 2 -> 1x2, 4 -> 2x2, 8 -> 2x4; otherwise 1 x world."""
    return {1: (1, 1), 2: (1, 2), 4: (2, 2), 8: (2, 4)}.get(world, (1, world))


def panel_schedule(lay: Layout, rank: int) -> list[Panel]:
    """The K-panels rank (i, j) accumulates, in its order: starting with the first panel whose A block it owns."""
    lay.check()
    i, j = lay.coords(rank)
    n = lay.K // lay.kb
    start = (j * lay.Kc) // lay.kb
    out = []
    for t in range(n):
        k0 = ((start + t) % n) * lay.kb
        ja, ib = k0 // lay.Kc, k0 // lay.Kr
        out.append(Panel(k0, lay.rank_of(i, ja), k0 - ja * lay.Kc, lay.rank_of(ib, j), k0 - ib * lay.Kr))
    return out


def summa_numpy(lay: Layout, rank: int, a_blocks: dict, b_blocks: dict):
    """C_ij from the blocks of all ranks (numpy, float32 accumulate): the reference driver the CPU tests run on
    gloo ranks with exactly the panel schedule of the GPU driver."""
    import numpy as np
    c = np.zeros((lay.Mb, lay.Nb), np.float32)
    for p in panel_schedule(lay, rank):
        a = a_blocks[p.a_rank][:, p.a_col:p.a_col + lay.kb].astype(np.float32)
        b = b_blocks[p.b_rank][p.b_row:p.b_row + lay.kb, :].astype(np.float32)
        c += a @ b
    return c


class SummaGPU:
    """One rank of the GPU SUMMA. `exchange(obj) -> list` gathers a picklable object from every rank (e.g.
    torch.distributed.all_gather_object); `barrier()` synchronises the ranks."""

    def __init__(self, lib, lay: Layout, rank: int, exchange, barrier, streams):
        lay.check()
        self.lib, self.lay, self.rank = lib, lay, rank
        self.i, self.j = lay.coords(rank)
        self.barrier = barrier
        self.compute, self.copy = streams        # torch.cuda.Stream pair
        self.sched = panel_schedule(lay, rank)
        al = lib.sh_cuda_ipc_alloc
        self.a_loc = al(lay.Mb * lay.Kc * 2)
        self.b_loc = al(lay.Kr * lay.Nb * 2)
        self.c = al(lay.Mb * lay.Nb * 2)
        # fp32 running sum of the panels (fp32 accumulation); C is rounded to fp16 once
        self.acc = al(lay.Mb * lay.Nb * 4) if lay.K // lay.kb > 1 else None
        remote = any(p.a_rank != rank or p.b_rank != rank for p in self.sched)
        self.a_pan = [al(lay.Mb * lay.kb * 2) for _ in range(2)] if remote else []
        self.b_pan = [al(lay.kb * lay.Nb * 2) for _ in range(2)] if remote else []
        if not (self.a_loc and self.b_loc and self.c) or (remote and not all(self.a_pan + self.b_pan)):
            raise RuntimeError("sh_cuda_ipc_alloc failed")
        ha, hb = ctypes.create_string_buffer(64), ctypes.create_string_buffer(64)
        if lib.sh_cuda_ipc_handle(self.a_loc, ha) or lib.sh_cuda_ipc_handle(self.b_loc, hb):
            raise RuntimeError("sh_cuda_ipc_handle failed")
        handles = exchange((rank, ha.raw, hb.raw))
        self.peer_a: dict[int, int] = {rank: self.a_loc}
        self.peer_b: dict[int, int] = {rank: self.b_loc}
        self.opened: list[int] = []
        need_a = {p.a_rank for p in self.sched} - {rank}
        need_b = {p.b_rank for p in self.sched} - {rank}
        for r, hA, hB in handles:
            for need, table, h in ((need_a, self.peer_a, hA), (need_b, self.peer_b, hB)):
                if r in need:
                    ptr = lib.sh_cuda_ipc_open(ctypes.create_string_buffer(h, 64))
                    if not ptr:
                        raise RuntimeError(f"sh_cuda_ipc_open of rank {r} failed")
                    table[r] = ptr
                    self.opened.append(ptr)

    def fill_inputs(self, seed_a: int, seed_b: int, lo: int = -1024, hi: int = 1023, scale: float = 1.0 / 1024):
        """Each rank generates its own blocks of the global LCG matrices (uniform [-1, 1) by default)."""
        lay, lib = self.lay, self.lib
        lib.sh_cuda_fill_lcg_block(self.a_loc, lay.Mb, lay.Kc, lay.Kc, seed_a, lo, hi, scale, self.i * lay.Mb,
                                   self.j * lay.Kc, lay.K)
        lib.sh_cuda_fill_lcg_block(self.b_loc, lay.Kr, lay.Nb, lay.Nb, seed_b, lo, hi, scale, self.i * lay.Kr,
                                   self.j * lay.Nb, lay.N)
        lib.sh_cuda_synchronize()
        self.barrier()        # every block exists before any rank pulls from it

    def step(self, torch, prefetch_next: bool = False) -> int:
        """C_ij = sum over panels (enqueued; returns 0 or the first failing return code). With prefetch_next the
        first panel of the next step (the same panels: inputs are read-only) is pulled while this step's last GEMM
        runs, so that a run of steps keeps the copy engines busy across step boundaries."""
        lay, lib = self.lay, self.lib
        lib.sh_cuda_set_stream(self.compute.cuda_stream)
        if not hasattr(self, "_ev"):
            self._ev = {"copy": [torch.cuda.Event(), torch.cuda.Event()],
                        "gemm": [torch.cuda.Event(), torch.cuda.Event()]}
            self._gemm_recorded = [False, False]
            self._prefetched = False
        copy_done, gemm_done = self._ev["copy"], self._ev["gemm"]
        pulled = [False, False]
        n = len(self.sched)

        def pull(idx: int):
            p, s = self.sched[idx], idx % 2
            pulled[s] = False
            if p.a_rank == self.rank and p.b_rank == self.rank:
                return
            with torch.cuda.stream(self.copy):
                if self._gemm_recorded[s]:
                    self.copy.wait_event(gemm_done[s])       # the last GEMM that read this slot is done
                if p.a_rank != self.rank:
                    lib.sh_cuda_copy2d(self.a_pan[s], lay.kb * 2, self.peer_a[p.a_rank] + 2 * p.a_col, lay.Kc * 2,
                                       lay.kb * 2, lay.Mb, self.copy.cuda_stream)
                if p.b_rank != self.rank:
                    lib.sh_cuda_copy2d(self.b_pan[s], lay.Nb * 2, self.peer_b[p.b_rank] + 2 * p.b_row * lay.Nb,
                                       lay.Nb * 2, lay.Nb * 2, lay.kb, self.copy.cuda_stream)
                copy_done[s].record(self.copy)
            pulled[s] = True

        if self._prefetched:                      # panel 0 is already on its way (previous step's prefetch)
            p0 = self.sched[0]
            pulled[0] = not (p0.a_rank == self.rank and p0.b_rank == self.rank)
            self._prefetched = False
        else:
            pull(0)
        rc = 0
        for idx, p in enumerate(self.sched):
            s = idx % 2
            if idx + 1 < n:
                pull(idx + 1)
            elif prefetch_next and n % 2 == 0 and n > 1:
                # the next step's panel 0 goes to slot 0, last read by this step's panel n - 2
                pull(0)
                self._prefetched = True
            with torch.cuda.stream(self.compute):
                if pulled[s]:
                    self.compute.wait_event(copy_done[s])
                if p.a_rank == self.rank:
                    a, lda = self.a_loc + 2 * p.a_col, lay.Kc
                else:
                    a, lda = self.a_pan[s], lay.kb
                if p.b_rank == self.rank:
                    b, ldb = self.b_loc + 2 * p.b_row * lay.Nb, lay.Nb
                else:
                    b, ldb = self.b_pan[s], lay.Nb
                last = idx == n - 1
                if self.acc is None:            # one panel: straight to fp16
                    z, flags, res = self.c, 0, 0
                elif idx == 0:
                    z, flags, res = self.acc, L.EPI_F32_OUT, 0
                elif not last:
                    z, flags, res = self.acc, L.EPI_F32_OUT | L.EPI_ACCUMULATE, 0
                else:
                    z, flags, res = self.c, L.EPI_ACC_F32_IN, self.acc
                rc = rc or lib.sh_cuda_gemm(a, b, z, lay.Mb, lay.Nb, lay.kb, lda, ldb, lay.Nb, 0, res, lay.Nb, flags, 1)
                gemm_done[s].record(self.compute)
                self._gemm_recorded[s] = True
        return rc

    def finish(self, torch) -> None:
        """Make the compute stream wait for an outstanding prefetch (so a timed region ends after it)."""
        if getattr(self, "_prefetched", False):
            self.compute.wait_stream(self.copy)

    def close(self):
        for p in self.opened:
            self.lib.sh_cuda_ipc_close(p)
        self.opened = []
        for p in [self.a_loc, self.b_loc, self.c, self.acc, *self.a_pan, *self.b_pan]:
            if p:
                self.lib.sh_cuda_ipc_free(p)
        self.a_loc = self.b_loc = self.c = self.acc = None
        self.a_pan, self.b_pan = [], []
