"""The dialect parser and emit_cuda lowering, checked against the reference's FileCheck expectations (read from the
reference checkout when it is present) and against the frontend modules in tests/golden/mlir."""
from __future__ import annotations

import os
import re
import shutil
import subprocess
from pathlib import Path

import pytest

import filecheck_lite
from softhier_cuda import dialect as D
from softhier_cuda import emit_cuda as E

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("SOFTHIER_REF", "/root/reference"))
FC = REF / "tests" / "filecheck"
MLIR = Path(__file__).resolve().parent / "golden" / "mlir"
# translate tests on the operator-library path (the others exercise TCDM / LLM / training ops outside it)
HOT_TRANSLATE = ["gemm512_translate.mlir", "gemm_nonconst_translate.mlir", "hbm_ops_translate.mlir",
                 "attention_translate.mlir", "loop_translate.mlir", "mark_translate.mlir", "gemm_xmcast_translate.mlir"]
OPT = ["distribute_summa.mlir", "pipeline_gemm.mlir", "linalg_gemm512.mlir"]
needs_ref = pytest.mark.skipif(not FC.exists(), reason="reference checkout not present")


@needs_ref
@pytest.mark.parametrize("name", HOT_TRANSLATE)
def test_reference_filecheck_translate(name):
    text = (FC / name).read_text()
    assert "softhier-translate %s | filecheck %s" in text
    filecheck_lite.check(E.emit_c(text), text)


@needs_ref
@pytest.mark.parametrize("name", OPT)
def test_reference_filecheck_passes(name):
    text = (FC / name).read_text()
    run = re.search(r"RUN:.*-p ([\w,-]+)", text).group(1).split(",")
    fn = E.apply_passes(D.parse_module(text), tuple(run))
    filecheck_lite.check(D.print_func(fn), text)


def test_filecheck_lite_semantics():
    out = "a b\nsh_gemm(x, 1)\nnext line\nz"
    filecheck_lite.check(out, "// CHECK: sh_gemm({{.*}}, 1)\n// CHECK-NEXT: next   line\n// CHECK-NOT: nothing")
    with pytest.raises(AssertionError):
        filecheck_lite.check(out, "// CHECK: sh_gemm\n// CHECK-NEXT: z")
    with pytest.raises(AssertionError):
        filecheck_lite.check(out, "// CHECK: a b\n// CHECK-NOT: next\n// CHECK: z")


def test_memref_geometry():
    mt = D.parse_memref('memref<64x256xf16, strided<[256, 1], offset: 16384>, "hbm_west">')
    assert mt.geom() == (64, 256, 256, 16384) and mt.space == "hbm_west" and mt.nbytes == 64 * 256 * 2
    assert D.parse_memref('memref<1x768xf16, "hbm_west">').geom() == (1, 768, 768, 0)
    assert D.parse_attrs('eps = 1.0e-6 : f32, cluster = -1 : i32, pipeline, tag = "P"') == {
        "eps": 9.999999974752427e-07, "cluster": -1, "pipeline": True, "tag": "P"}


def _calls(c: str) -> dict[str, int]:
    kernel = c.split("static void siglip_encoder(void) {")[1].split("static void siglip_encoder_checks")[0]
    out: dict[str, int] = {}
    for m in re.finditer(r"\b(sh_\w+)\(", kernel):
        out[m.group(1)] = out.get(m.group(1), 0) + 1
    return out


def test_siglip_frontend_module_per_head():
    """frontend/siglip.py output (S=256, 12 heads, per-head attention): every op lowers to one library call."""
    c = E.emit_c((MLIR / "siglip_s256_perhead.mlir").read_text())
    k = _calls(c)
    assert k["sh_layernorm"] == 2 and k["sh_transpose"] == 1 and k["sh_softmax_rows"] == 12
    assert k["sh_gemm"] == 4 + 2 + 24 and k["sh_add_bias"] == 6 and k["sh_gelu"] == 1 and k["sh_add"] == 2
    assert "unsupported" not in c
    # per-head views: q head 1 at element offset 64 (128 B), kT head 1 at 64 * 256 elements
    assert "sh_gemm((hb3 + 128), (hb6 + 32768), (hb7 + 131072), 256, 256, 64, 768, 256, 256, &cfg, 1); }" in c
    inputs = c.split("static void siglip_encoder_inputs(void) {")[1].split("static void siglip_encoder(void)")[0]
    assert inputs.count("sh_test_fill_fp16(") == 17     # x + 16 parameters, before the timer


def test_siglip_frontend_module_fused_two_layers():
    c = E.emit_c((MLIR / "siglip_s64_fused_l2.mlir").read_text())
    k = _calls(c)
    assert k["sh_attention_q"] == 2 and k["sh_layernorm"] == 4 and k["sh_gemm"] == 12
    # q_block attribute (the frontend's mirror of the library rule) selects sh_attention_q; scale 1/sqrt(64)
    assert "sh_attention_q(hb3, hb4, hb5, hb6, 64, 128, 2, 128, 128, 128, 128, 0.125f, SH_ALL, 64);" in c


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_emitted_program_compiles_and_links(tmp_path):
    """The generated main.c builds against include/sh_ops.h and links with libsh_ops_cuda.so (no run)."""
    lib = ROOT / "softhier-mlir_b200" / "lib"
    if not (lib / "libsh_ops_cuda.so").exists():
        pytest.skip("library not built")
    src = tmp_path / "main.c"
    src.write_text(E.emit_c((MLIR / "siglip_s256_perhead.mlir").read_text()))
    r = subprocess.run(["gcc", "-O1", "-Wall", "-Wno-unused-variable", "-Werror", "-I", str(ROOT / "include"), str(src), "-L", str(lib),
                        "-lsh_ops_cuda", "-o", str(tmp_path / "main")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
