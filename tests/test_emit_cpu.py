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
# a checkout of the reference (runwangdl/softhier-mlir), named by SOFTHIER_REF; its FileCheck suite is skipped without it
REF = Path(os.environ["SOFTHIER_REF"]) if os.environ.get("SOFTHIER_REF") else None
FC = REF / "tests" / "filecheck" if REF else None
MLIR = Path(__file__).resolve().parent / "golden" / "mlir"
# translate tests of the operator library and the decoder ops (the others exercise TCDM / expert / training ops)
HOT_TRANSLATE = ["gemm512_translate.mlir", "gemm_nonconst_translate.mlir", "hbm_ops_translate.mlir",
                 "attention_translate.mlir", "loop_translate.mlir", "mark_translate.mlir", "gemm_xmcast_translate.mlir",
                 "llm_translate.mlir"]
OPT = ["distribute_summa.mlir", "pipeline_gemm.mlir", "linalg_gemm512.mlir"]
needs_ref = pytest.mark.skipif(FC is None or not FC.exists(), reason="SOFTHIER_REF names no reference checkout")


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


def test_fuse_epilogues_pass():
    """fuse-epilogues: gemm + add_bias (+ gelu | + residual add) -> one sh_cuda_gemm; the SigLIP layer goes from 16
    calls to 9; buffers that later ops read before a GEMM overwrites them are left unfused."""
    c = E.emit_c((MLIR / "siglip_s256_fused.mlir").read_text(), ("fuse-epilogues",))
    k = _calls(c)
    assert k == {"sh_cuda_gemm": 6, "sh_layernorm": 2, "sh_attention_q": 1, "sh_barrier_global": 1,
                 "sh_hbm_addr": k["sh_hbm_addr"], "sh_cluster_id": 4, "sh_is_first_core": 4, "sh_printf": 4,
                 "sh_cycles": 4}
    assert "sh_cuda_gemm(hb2, hb14, hb3, 256, 768, 768, 768, 768, 768, hb20, 0, 768, SH_EPI_BIAS, 0);" in c
    # o projection: h = x + (o wo + bo); FC1: g = gelu(ln2 w1 + b1); FC2: out = h + (g w2 + b2)
    assert "sh_cuda_gemm(hb6, hb17, hb8, 256, 768, 768, 768, 768, 768, hb23, hb1, 768, SH_EPI_BIAS | SH_EPI_RESIDUAL, 0);" in c
    assert "sh_cuda_gemm(hb9, hb18, hb11, 256, 3072, 768, 768, 3072, 3072, hb24, 0, 3072, SH_EPI_BIAS | SH_EPI_GELU, 0);" in c
    assert "sh_cuda_gemm(hb11, hb19, hb13, 256, 768, 3072, 3072, 768, 768, hb25, hb8, 768, SH_EPI_BIAS | SH_EPI_RESIDUAL, 0);" in c
    # two stacked layers: the second layer's GEMMs overwrite ao / f1 / f2 before reading them, so both layers fuse
    k2 = _calls(E.emit_c((MLIR / "siglip_s64_fused_l2.mlir").read_text(), ("fuse-epilogues",)))
    assert k2["sh_cuda_gemm"] == 12 and "sh_add" not in k2 and "sh_gelu" not in k2 and "sh_add_bias" not in k2
    # a dump of the pre-GELU buffer keeps the GELU separate (bias still fuses in place)
    t = (MLIR / "siglip_s256_fused.mlir").read_text()
    dump = ('    softhier.dump_samples %f1 {tag = "F1", seed = 5 : i32, n = 8 : i32} : '
            'memref<256x3072xf16, "hbm_west">\n    func.return')
    k3 = _calls(E.emit_c(t.replace("    func.return", dump, 1), ("fuse-epilogues",)))
    assert k3["sh_gelu"] == 1 and k3["sh_cuda_gemm"] == 6


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
@pytest.mark.parametrize("passes", [(), ("fuse-epilogues",)])
def test_emitted_program_compiles_and_links(tmp_path, passes):
    """The generated main.c builds against include/ and links with libsh_ops_cuda.so (no run)."""
    lib = ROOT / "softhier-mlir_b200" / "lib"
    if not (lib / "libsh_ops_cuda.so").exists():
        pytest.skip("library not built")
    src = tmp_path / "main.c"
    src.write_text(E.emit_c((MLIR / "siglip_s256_perhead.mlir").read_text(), passes))
    r = subprocess.run(["gcc", "-O1", "-Wall", "-Wno-unused-variable", "-Werror", "-I", str(ROOT / "include"), str(src), "-L", str(lib),
                        "-lsh_ops_cuda", "-o", str(tmp_path / "main")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_looped_encoder_lowering(tmp_path):
    """scf.for lowering of a compact multi-layer module (tests/looped_module.py): the layer loop becomes a C for loop,
    every indexed parameter buffer `offset + i * stride`, the nested GELU loop indexed column views of FC1's output,
    and the indexed dump appends the layer number (the rules of the reference's loop_translate.mlir:26-37); the
    program compiles and links against the library."""
    import looped_module as LM
    S, D, F, H, NL = 64, 128, 256, 2, 3
    act, poff, stride, base = LM.layout(S, D, F)
    c = E.emit_c(LM.looped_encoder(S, D, F, H, NL))
    body = c.split("static void looped_encoder(void) {")[1]
    assert "for (uint32_t i1 = 0; i1 < 3; i1 += 1) {" in body
    assert f"sh_hbm_addr((uint64_t){base + poff['w1']} + (uint64_t)(i1) * {stride}u);" in body
    assert "for (uint32_t i2 = 0; i2 < 4; i2 += 1) {" in body
    # gelu over column block i2 of f1 (hb10) into g (hb11): 64 columns = 128 bytes per block
    assert "sh_gelu((hb11 + (uint64_t)(i2) * 128u), (hb10 + (uint64_t)(i2) * 128u), 64, 64, 256, SH_ALL);" in body
    assert 'sh_test_dump_samples_idx(hb1, 64, 128, 128, 7, 32, "L", (uint32_t)((i1 + 1)));' in body
    assert body.count("sh_gemm(") == 6 and "unsupported" not in c
    lib = ROOT / "softhier-mlir_b200" / "lib"
    if shutil.which("gcc") is None or not (lib / "libsh_ops_cuda.so").exists():
        pytest.skip("no C compiler or library")
    src = tmp_path / "main.c"
    src.write_text(c)
    r = subprocess.run(["gcc", "-O1", "-Wall", "-Wno-unused-variable", "-Werror", "-I", str(ROOT / "include"),
                        str(src), "-L", str(lib), "-lsh_ops_cuda", "-o", str(tmp_path / "main")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
