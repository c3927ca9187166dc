"""2-D block-distributed SUMMA GEMM across the GPUs of one node: the multi-GPU form of sh_gemm_mesh
(runtime/sh_gemm.inc.c:120-189, mesh-wide output-stationary SUMMA with diagonal-owner panel broadcasts).

Rank (i, j) of a pr x pc grid (rank = i * pc + j) owns, of C = A B with A [M, K], B [K, N]:
    A_ij = A[i Mb:(i+1) Mb, j Kc:(j+1) Kc]     Mb = M / pr, Kc = K / pc
    B_ij = B[i Kr:(i+1) Kr, j Nb:(j+1) Nb]     Kr = K / pr, Nb = N / pc
    C_ij = C[i Mb:(i+1) Mb, j Nb:(j+1) Nb]  =  sum over K-panels k of  A[i-rows, k] B[k, j-cols]
The A columns of a K-panel [k0, k0 + kb) live on the ranks (i, *) of this rank's grid row (owner of column k:
k // Kc), its B rows on the ranks (*, j) of its grid column (owner of row k: k // Kr); a panel may span several
owners and is then made of pieces. Instead of the reference's row / column multicasts, every rank PULLS the pieces
it needs with the copy engines (CUDA IPC mappings of the owners' blocks + cudaMemcpy2DAsync on a copy stream: no SM
is spent on the transfer), into double-buffered local panels, while the tcgen05 GEMM of the previous panel runs on
the compute stream (C_ij += A_panel B_panel through the accumulate epilogue, carried in fp32 between panels and
rounded to fp16 by the last one). A panel that is one piece of this rank's own block is read in place. Inputs are
read-only during a step, so the step needs no cross-GPU synchronisation; ranks start at the panel holding their own
A block, to spread the pulls over the owners.

Panel width: every extra panel costs an fp32 read + write of C_ij (the carry), so the default is one panel per step
(`default_panel`). Panel slots alternate by a running count across steps, so the next step's panel is pulled while
this step's GEMM runs. Every step still does one full set of pulls and one GEMM.

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
        if self.kb <= 0 or self.K % self.kb:
            raise ValueError(f"panel width {self.kb} must divide K = {self.K}")

    def coords(self, rank: int) -> tuple[int, int]:
        return divmod(rank, self.pc)

    def rank_of(self, i: int, j: int) -> int:
        return i * self.pc + j


@dataclass(frozen=True)
class Piece:
    rank: int          # owner
    src: int           # first column (A) / row (B) inside the owner's block
    dst: int           # first column (A) / row (B) inside the panel
    width: int         # columns (A) / rows (B)


@dataclass(frozen=True)
class Panel:
    k0: int                    # first K index of the panel
    a: tuple[Piece, ...]       # A[i-rows, k0:k0+kb] by owner, in K order
    b: tuple[Piece, ...]       # B[k0:k0+kb, j-cols] by owner, in K order

    def a_direct(self, rank: int) -> bool:
        """The A panel is one piece of `rank`'s own block (read in place)."""
        return len(self.a) == 1 and self.a[0].rank == rank

    def b_direct(self, rank: int) -> bool:
        return len(self.b) == 1 and self.b[0].rank == rank


def default_grid(world: int) -> tuple[int, int]:
    """1 -> 1x1, 2 -> 1x2, 4 -> 2x2, 8 -> 2x4; otherwise 1 x world."""
    return {1: (1, 1), 2: (1, 2), 4: (2, 2), 8: (2, 4)}.get(world, (1, world))


def default_panel(K: int, world: int) -> int:
    """One panel per step on any grid: no fp32 carry pass, and the pull of a step's whole panel overlaps the previous
    step's GEMM (SummaGPU.step with prefetch_next). Two or more panels also overlap pulls inside a step, at the
    cost of an fp32 read + write of C_ij per extra panel."""
    return K


def _pieces(k0: int, kb: int, block: int, owners: list[int]) -> tuple[Piece, ...]:
    out = []
    for idx, r in enumerate(owners):
        lo, hi = max(k0, idx * block), min(k0 + kb, (idx + 1) * block)
        if lo < hi:
            out.append(Piece(r, lo - idx * block, lo - k0, hi - lo))
    return tuple(out)


def panel_schedule(lay: Layout, rank: int) -> list[Panel]:
    """The K-panels rank (i, j) accumulates, in its order: starting with the panel that holds its own A block."""
    lay.check()
    i, j = lay.coords(rank)
    n = lay.K // lay.kb
    start = (j * lay.Kc) // lay.kb
    row_owners = [lay.rank_of(i, jj) for jj in range(lay.pc)]
    col_owners = [lay.rank_of(ii, j) for ii in range(lay.pr)]
    out = []
    for t in range(n):
        k0 = ((start + t) % n) * lay.kb
        out.append(Panel(k0, _pieces(k0, lay.kb, lay.Kc, row_owners), _pieces(k0, lay.kb, lay.Kr, col_owners)))
    return out


def panel_peer_bytes(lay: Layout, rank: int) -> int:
    """Bytes this rank pulls from other GPUs per step."""
    return sum(sum(lay.Mb * q.width * 2 for q in p.a if q.rank != rank) +
               sum(q.width * lay.Nb * 2 for q in p.b if q.rank != rank) for p in panel_schedule(lay, rank))


def summa_numpy(lay: Layout, rank: int, a_blocks: dict, b_blocks: dict):
    """C_ij from the blocks of all ranks (numpy, float32 accumulate): the reference driver the CPU tests run on
    gloo ranks with exactly the panel schedule of the GPU driver."""
    import numpy as np
    c = np.zeros((lay.Mb, lay.Nb), np.float32)
    for p in panel_schedule(lay, rank):
        a = np.zeros((lay.Mb, lay.kb), np.float32)
        b = np.zeros((lay.kb, lay.Nb), np.float32)
        for q in p.a:
            a[:, q.dst:q.dst + q.width] = a_blocks[q.rank][:, q.src:q.src + q.width]
        for q in p.b:
            b[q.dst:q.dst + q.width, :] = b_blocks[q.rank][q.src:q.src + q.width, :]
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
        need_a_pan = any(not p.a_direct(rank) for p in self.sched)
        need_b_pan = any(not p.b_direct(rank) for p in self.sched)
        self.a_pan = [al(lay.Mb * lay.kb * 2) for _ in range(2)] if need_a_pan else []
        self.b_pan = [al(lay.kb * lay.Nb * 2) for _ in range(2)] if need_b_pan else []
        if not (self.a_loc and self.b_loc and self.c) or not all(self.a_pan + self.b_pan):
            raise RuntimeError("sh_cuda_ipc_alloc failed")
        ha, hb = ctypes.create_string_buffer(64), ctypes.create_string_buffer(64)
        if lib.sh_cuda_ipc_handle(self.a_loc, ha) or lib.sh_cuda_ipc_handle(self.b_loc, hb):
            raise RuntimeError("sh_cuda_ipc_handle failed")
        handles = exchange((rank, ha.raw, hb.raw))
        self.peer_a: dict[int, int] = {rank: self.a_loc}
        self.peer_b: dict[int, int] = {rank: self.b_loc}
        self.opened: list[int] = []
        need_a = {q.rank for p in self.sched for q in p.a} - {rank}
        need_b = {q.rank for p in self.sched for q in p.b} - {rank}
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
        """C_ij = sum over panels (enqueued; returns 0 or the first failing return code). Panels alternate between
        two buffer slots by a running count, across steps too. With prefetch_next the first panel of the next step
        (the same panels: inputs are read-only) is pulled while this step's last GEMM runs, so that a run of steps
        keeps the copy engines busy across step boundaries; with one panel per step that is the whole next pull."""
        lay, lib = self.lay, self.lib
        lib.sh_cuda_set_stream(self.compute.cuda_stream)
        if not hasattr(self, "_ev"):
            self._ev = {"copy": [torch.cuda.Event(), torch.cuda.Event()],
                        "gemm": [torch.cuda.Event(), torch.cuda.Event()]}
            self._gemm_recorded = [False, False]
            self._prefetched = False
            self._count = 0          # panels enqueued so far: panel t of the run uses slot t % 2
        copy_done, gemm_done = self._ev["copy"], self._ev["gemm"]
        pulled = [False, False]
        n, base = len(self.sched), self._count

        def pull(idx: int, s: int):
            p = self.sched[idx]
            pulled[s] = False
            if p.a_direct(self.rank) and p.b_direct(self.rank):
                return
            with torch.cuda.stream(self.copy):
                if self._gemm_recorded[s]:
                    self.copy.wait_event(gemm_done[s])       # the last GEMM that read this slot is done
                if not p.a_direct(self.rank):
                    for q in p.a:                            # column pieces of the A panel (a local one too)
                        lib.sh_cuda_copy2d(self.a_pan[s] + 2 * q.dst, lay.kb * 2, self.peer_a[q.rank] + 2 * q.src,
                                           lay.Kc * 2, q.width * 2, lay.Mb, self.copy.cuda_stream)
                if not p.b_direct(self.rank):
                    for q in p.b:                            # row pieces of the B panel
                        lib.sh_cuda_copy2d(self.b_pan[s] + 2 * q.dst * lay.Nb, lay.Nb * 2,
                                           self.peer_b[q.rank] + 2 * q.src * lay.Nb, lay.Nb * 2, lay.Nb * 2,
                                           q.width, self.copy.cuda_stream)
                copy_done[s].record(self.copy)
            pulled[s] = True

        if self._prefetched:                      # panel 0 is already on its way (previous step's prefetch)
            p0 = self.sched[0]
            pulled[base % 2] = not (p0.a_direct(self.rank) and p0.b_direct(self.rank))
            self._prefetched = False
        else:
            pull(0, base % 2)
        rc = 0
        for idx, p in enumerate(self.sched):
            s = (base + idx) % 2
            if idx + 1 < n:
                pull(idx + 1, (base + idx + 1) % 2)
            elif prefetch_next:
                # the next step's panel 0 goes to the other slot, last read by this step's panel n - 2 (or by the
                # previous step's last panel when n == 1)
                pull(0, (base + n) % 2)
                self._prefetched = True
            with torch.cuda.stream(self.compute):
                if pulled[s]:
                    self.compute.wait_event(copy_done[s])
                if p.a_direct(self.rank):
                    a, lda = self.a_loc + 2 * p.a[0].src, lay.Kc
                else:
                    a, lda = self.a_pan[s], lay.kb
                if p.b_direct(self.rank):
                    b, ldb = self.b_loc + 2 * p.b[0].src * lay.Nb, lay.Nb
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
        self._count += n
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
