"""The C-ABI library loads without a GPU and exports every entry point include/*.h declares (no compute calls)."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "softhier-mlir_b200" / "lib" / "libsh_ops_cuda.so"
DECL = re.compile(r"^\s*(?:[A-Za-z_][\w \*]*?[\s\*])(sh_\w+)\s*\(", re.M)


def declared() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for line in text.splitlines():
            if line.strip().startswith("#"):
                continue
            m = DECL.match(line)
            if m:
                names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def lib_path():
    if not LIB.exists():
        import __graft_entry__  # noqa: F401  (build() compiles it)
        __graft_entry__.build()
    return LIB


def test_headers_declare_the_hot_path():
    names = declared()
    for must in ("sh_gemm", "sh_gemm_mesh", "sh_gemm_xmcast_ex", "sh_gemm_l1_bytes", "sh_layernorm", "sh_softmax_rows",
                 "sh_gelu", "sh_add", "sh_add_bias", "sh_scale", "sh_transpose", "sh_attention", "sh_attention_q",
                 "sh_attention_head", "sh_attention_q_block", "sh_test_fill_fp16", "sh_test_dump_samples",
                 "sh_init", "sh_hbm_addr", "sh_cuda_set_arena", "sh_cuda_gemm", "sh_cuda_attention_batched"):
        assert must in names, must
    assert len(names) >= 60


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = sorted(declared() - exported)
    assert not missing, missing


def test_ctypes_binding_covers_every_declaration(lib_path):
    from softhier_cuda import lib as L
    assert set(L.SIGNATURES) == declared()
    lib = L.load(lib_path)
    assert lib.sh_cuda_abi_version() == 1          # pure host function, no device needed
    assert lib.sh_attention_q_block(256, 64, 12, 16) == 64      # the reference's rule (docs/DSE.md:279)
    assert lib.sh_attention_q_block(1024, 64, 12, 16) == 256
    assert lib.sh_cluster_id() == 0 and lib.sh_num_clusters() == 1 and lib.sh_is_first_core() == 1


def test_host_fp16_conversions(lib_path):
    import numpy as np
    from softhier_cuda import lib as L
    lib = L.load(lib_path)
    vals = np.array([0.0, -0.0, 1.0, 65504.0, 65520.0, 1e-8, 2 ** -24, 3 * 2 ** -26, 0.1, -123.456, 1 / 3], np.float32)
    with np.errstate(over="ignore"):   # 65520 rounds to +inf on purpose
        for v in vals:
            assert lib.sh_f32_to_fp16(float(v)) == int(np.float16(v).view(np.uint16)), v
    for code in (0x0000, 0x0001, 0x03ff, 0x0400, 0x3c00, 0x7bff, 0xfbff, 0x8001):
        assert lib.sh_fp16_to_f32(code) == float(np.uint16(code).view(np.float16)), hex(code)


def test_build_uses_sm100a_and_no_forbidden_forms():
    src = "\n".join(p.read_text() for p in (ROOT / "softhier-mlir_b200" / "csrc").glob("*.cu*"))
    assert "tcgen05.mma" in src and "cp.async.bulk.tensor" in src
    # No load of any kind uses the cluster-broadcast form; the one use of the qualifier is tcgen05.commit's own arrive
    # signal to both CTAs of a pair (a completion signal, not a memory load).
    mc = "." + "multi" + "cast" + "::" + "cluster"
    for line in src.splitlines():
        if mc in line:
            assert "tcgen05.commit" in line and "cp.async" not in line and "ld." not in line, line
    assert not any("cp.async.bulk" in ln and "multi" + "cast" in ln for ln in src.splitlines())
    assert "__trap" not in src and "asm(\"trap" not in src
    build = (ROOT / "softhier-mlir_b200" / "build.py").read_text()
    assert "arch=compute_100a,code=sm_100a" in build


def test_host_normal_generator_matches_the_oracle_bit_for_bit(lib_path):
    """sh_cuda_host_fill_normal_fp16 (the library's N(mean, std) definition, run on the CPU) == oracle.lcg.normal_fp16
    for every element, including a strided destination; the device kernel evaluates the same host/device function."""
    import numpy as np

    from oracle import lcg
    from softhier_cuda import lib as L
    lib = L.load(lib_path)
    for rows, cols, seed, mean, std in ((64, 96, 7, 0.0, 1.0), (3, 1000, 11, 1.0, 0.02), (257, 33, 0, -0.5, 3.0)):
        ld = cols + 5
        buf = np.full((rows, ld), 0x7E00, np.uint16)
        lib.sh_cuda_host_fill_normal_fp16(buf.ctypes.data, rows, cols, ld, seed, mean, std)
        want = lcg.normal_fp16(rows, cols, seed, mean, std).view(np.uint16)
        assert np.array_equal(buf[:, :cols], want), (rows, cols, seed)
        assert (buf[:, cols:] == 0x7E00).all()
