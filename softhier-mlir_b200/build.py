"""Build libsh_ops_cuda.so in-tree for sm_100a.

    python softhier-mlir_b200/build.py [--force] [-v]

Each csrc/*.cu is compiled by nvcc (-gencode arch=compute_100a,code=sm_100a, static CUDA runtime, no link-time
dependency on libcuda) into _build/, then linked into softhier-mlir_b200/lib/libsh_ops_cuda.so. A source is
rebuilt when it or any header is newer than its object.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libsh_ops_cuda.so"
INCLUDE = ROOT / "include"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2,-ffp-contract=off", "-I", str(INCLUDE), "-I", str(CSRC),
         "--expt-relaxed-constexpr"]


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(src: Path, obj: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers()])


def _compile(src: Path, verbose: bool, extra: list[str]) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    todo = [s for s in srcs if force or ptxas_info or _stale(s, BUILD / (s.stem + ".o"))]
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for obj, err in ex.map(lambda s: _compile(s, verbose, extra), todo):
            if ptxas_info and err:
                print(f"== {obj.stem}\n{err}")
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / shared memory per kernel")
    a = ap.parse_args()
    try:
        print(build(a.force, a.verbose, a.ptxas_info))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
