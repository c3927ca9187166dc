"""Device arena + stream plumbing around libsh_ops_cuda.so.

torch provides the device memory (one uint8 tensor per device, bound with sh_cuda_set_arena so that
sh_hbm_addr(off) == arena base + off) and the stream the library enqueues on. Everything computed goes through
the library's C ABI.
"""
from __future__ import annotations

import numpy as np
import torch

from . import lib as _lib


class ShCudaError(RuntimeError):
    pass


class Runtime:
    """One per device: the arena, the bound stream and a bump allocator over arena offsets."""

    _instances: dict[int, "Runtime"] = {}

    @classmethod
    def open(cls, device: int = 0, arena_bytes: int = 1 << 30) -> "Runtime":
        rt = cls._instances.get(device)
        if rt is None or rt.arena_bytes < arena_bytes:
            rt = cls(device, arena_bytes)
            cls._instances[device] = rt
        else:
            rt.activate()
        return rt

    def __init__(self, device: int, arena_bytes: int):
        if not torch.cuda.is_available():
            raise ShCudaError("no CUDA device: libsh_ops_cuda.so needs a B200")
        self.device = device
        torch.cuda.set_device(device)
        self.lib = _lib.load()
        self.arena_bytes = int(arena_bytes)
        self.arena = torch.zeros(self.arena_bytes, dtype=torch.uint8, device=f"cuda:{device}")
        self.base = self.arena.data_ptr()
        self.stream = torch.cuda.current_stream(device)
        self.activate()
        self.lib.sh_init()
        self.next_off = 0x1000
        self.check()

    def activate(self, stream: torch.cuda.Stream | None = None) -> None:
        torch.cuda.set_device(self.device)
        if stream is not None:
            self.stream = stream
        if self.lib.sh_cuda_set_arena(self.base, self.arena_bytes) != 0:
            raise ShCudaError("sh_cuda_set_arena failed")
        self.lib.sh_cuda_set_stream(self.stream.cuda_stream)

    # ---- allocation over arena offsets -------------------------------------------------------------------
    def reset(self, off: int = 0x1000) -> None:
        self.next_off = off

    def alloc_bytes(self, nbytes: int, align: int = 4096) -> int:
        off = (self.next_off + align - 1) // align * align
        if off + nbytes > self.arena_bytes:
            raise ShCudaError(f"arena of {self.arena_bytes} B exhausted ({off + nbytes} B needed)")
        self.next_off = off + nbytes
        return self.base + off

    def alloc(self, rows: int, cols: int, ld: int | None = None, align: int = 4096) -> int:
        ld = cols if ld is None else ld
        return self.alloc_bytes(((rows - 1) * ld + cols) * 2 if rows else 0, align)

    # ---- host <-> device -----------------------------------------------------------------------------------
    def view(self, addr: int, rows: int, cols: int, ld: int | None = None) -> torch.Tensor:
        """fp16 [rows, cols] torch view of arena memory at device address `addr` (leading dim ld)."""
        ld = cols if ld is None else ld
        off = addr - self.base
        if off < 0 or off % 2 or off + ((rows - 1) * ld + cols) * 2 > self.arena_bytes:
            raise ShCudaError(f"address {addr:#x} [{rows}x{cols} ld {ld}] outside the arena")
        n = (rows - 1) * ld + cols if rows else 0
        flat = self.arena[off:off + 2 * n].view(torch.float16)
        return flat.as_strided((rows, cols), (ld, 1))

    def put(self, addr: int, a: np.ndarray, ld: int | None = None) -> None:
        a = np.ascontiguousarray(np.asarray(a, dtype=np.float16))
        rows, cols = a.shape
        self.view(addr, rows, cols, ld).copy_(torch.from_numpy(a).to(self.arena.device))

    def get(self, addr: int, rows: int, cols: int, ld: int | None = None) -> np.ndarray:
        self.lib.sh_cuda_synchronize()
        return self.view(addr, rows, cols, ld).cpu().numpy()

    def put_bytes(self, addr: int, data: bytes) -> None:
        """Raw bytes (e.g. a uint16 token array) to an arena address."""
        off = addr - self.base
        if off < 0 or off + len(data) > self.arena_bytes:
            raise ShCudaError(f"address {addr:#x} [{len(data)} B] outside the arena")
        src = torch.frombuffer(bytearray(data), dtype=torch.uint8)
        self.arena[off:off + len(data)].copy_(src.to(self.arena.device))

    def upload(self, a: np.ndarray, align: int = 4096) -> int:
        a = np.asarray(a, dtype=np.float16)
        addr = self.alloc(*a.shape, align=align)
        self.put(addr, a)
        return addr

    # ---- errors -----------------------------------------------------------------------------------------------
    def check(self) -> None:
        """Synchronise; raise on a recorded library error, a CUDA error or a kernel's error word."""
        self.lib.sh_cuda_synchronize()
        code = self.lib.sh_cuda_last_error()
        if code:
            raise ShCudaError(f"libsh_ops_cuda error {code}: {self.lib.sh_cuda_last_error_string().decode()}")
        dev = self.lib.sh_cuda_device_error()
        if dev:
            raise ShCudaError(f"kernel error word {dev} (a bounded wait gave up)")
