"""Frontend modules lowered by emit_cuda and run on the GPU: the reference's siglip-mlir flow (frontend ->
translate -> run -> sampled dumps vs siglip_ref, tests/gvsoc/run.py:329-368) and its KAT examples."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import golden
from oracle import lcg, siglip
from softhier_cuda import emit_cuda as E

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
MLIR = Path(__file__).resolve().parent / "golden" / "mlir"
TAGS = {"X": "x", "LN1": "ln1", "Q": "q", "K": "k", "KT": "kT", "V": "v", "O": "o", "H": "h", "G": "g", "OUT": "out"}


def _run(rt, text, capfd, passes=()):
    rt.reset()
    prog = E.Program(text, rt, passes)
    capfd.readouterr()
    assert prog.run() == 0
    rt.check()
    return prog, capfd.readouterr().out


@pytest.mark.parametrize("passes", [(), ("fuse-epilogues",)])
@pytest.mark.parametrize("name", ["siglip_s256_perhead.mlir", "siglip_s256_fused.mlir"])
def test_siglip_layer_module_matches_reference(gpu_lib, capfd, name, passes):
    """Config 3 lowered from frontend/siglip.py: sampled dumps within the reference's 0.05 / 0.05 (run.py:360-365)
    against siglip_ref's own values, and every full tensor against the oracle; unfused and with the GEMM epilogues
    fused."""
    prog, out = _run(gpu_lib, (MLIR / name).read_text(), capfd, passes)
    got = lcg.parse_samples(out)
    g = golden("siglip_s256.npz")
    tags = [t for t in TAGS if t in got]
    assert {"X", "LN1", "Q", "K", "V", "O", "H", "G", "OUT"} <= set(tags)
    for tag in tags:
        pos = g[f"{tag}_pos"]
        want = np.zeros((int(pos[:, 0].max()) + 1, int(pos[:, 1].max()) + 1), np.float32)
        want[pos[:, 0], pos[:, 1]] = g[f"{tag}_val"]
        assert [(r, c) for r, c, _ in got[tag]] == [tuple(p) for p in pos.tolist()], tag
        bad, err = lcg.compare_samples(got[tag], want, 0.05, 0.05)
        assert bad == 0, (tag, err)
    assert "[Performance Counter]: Execution period is" in out
    ref = siglip.layer_reference(256, 768, 3072, 12)
    for tag, buf in TAGS.items():
        if tag == "KT" and "fused" in name:
            continue
        t = prog.tensor(buf).astype(np.float32)
        err = np.abs(t - ref[tag])
        assert np.all(err <= 0.05 + 0.05 * np.abs(ref[tag])), (tag, float(err.max()))


@pytest.mark.parametrize("passes", [(), ("fuse-epilogues",)])
def test_two_layer_fused_module(gpu_lib, capfd, passes):
    """Two stacked layers (frontend seeds 100 * layer), small shape with explicit 64^3 GEMM tiles."""
    prog, out = _run(gpu_lib, (MLIR / "siglip_s64_fused_l2.mlir").read_text(), capfd, passes)
    x, p0 = siglip.lcg_layer_inputs(64, 128, 256, 0)
    _, p1 = siglip.lcg_layer_inputs(64, 128, 256, 1)
    want = siglip.encoder_reference(x, [p0, p1], 2, scale=0.125)
    got = prog.tensor("out").astype(np.float32)
    err = np.abs(got - want)
    assert np.all(err <= 0.05 + 0.05 * np.abs(want)), float(err.max())


KAT = """builtin.module {
  func.func @kat(%M) {
    %x = softhier.hbm_buffer {offset = 4096 : i32} : memref<%Mx%Mxf16, "hbm_west">
    %w = softhier.hbm_buffer {offset = %WOFF : i32} : memref<%Mx%Mxf16, "hbm_south">
    %z = softhier.hbm_buffer {offset = %ZOFF : i32} : memref<%Mx%Mxf16, "hbm_west">
    softhier.hbm_fill_col_parity %x {even_bits = 15360 : i32, odd_bits = %ODD : i32} : memref<%Mx%Mxf16, "hbm_west">
    softhier.hbm_fill %w {value_bits = %WBITS : i32} : memref<%Mx%Mxf16, "hbm_south">
    linalg.matmul ins(%x, %w : memref<%Mx%Mxf16, "hbm_west">, memref<%Mx%Mxf16, "hbm_south">) outs(%z : memref<%Mx%Mxf16, "hbm_west">)
    softhier.hbm_check_const %z {value_bits = %ZBITS : i32, tol = 16 : i32} : memref<%Mx%Mxf16, "hbm_west">
    func.return
  }
}
"""


def _kat(M: int, odd: int, wbits: int, zbits: int) -> str:
    b = M * M * 2
    t = KAT.replace("func.func @kat(%M)", f"func.func @kat{M}()")
    for k, v in (("%WOFF", 4096 + b), ("%ZOFF", 4096 + 2 * b), ("%ODD", odd), ("%WBITS", wbits), ("%ZBITS", zbits),
                 ("%M", M)):
        t = t.replace(k, str(v))
    return t


@pytest.mark.parametrize("M,odd,wbits,zbits,passes", [
    (512, 15360, 6144, 15360, ("linalg-to-softhier",)),                       # X = 1, W = 1/512 -> Z = 1
    (512, 14336, 6144, 14848, ("linalg-to-softhier", "pipeline-gemm")),      # col parity 1 / 0.5 -> Z = 0.75
    (1024, 15360, 5120, 15360, ("linalg-to-softhier", "distribute-summa")),  # SUMMA schedule, W = 1/1024 -> 1
])
def test_kat_modules_in_process(gpu_lib, capfd, M, odd, wbits, zbits, passes):
    _, out = _run(gpu_lib, _kat(M, odd, wbits, zbits), capfd, passes)
    assert f"KAT{M}_CHECK ok={M * M}/{M * M} KAT{M}_PASS" in out


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_emitted_c_program_runs(tmp_path):
    """The generated main.c, compiled against include/ and linked with libsh_ops_cuda.so, runs as its own process
    (the reference's flow: emit -> build -> run -> parse stdout)."""
    lib = ROOT / "softhier-mlir_b200" / "lib"
    src = tmp_path / "main.c"
    src.write_text(E.emit_c(_kat(1024, 15360, 5120, 15360), ("linalg-to-softhier", "distribute-summa")))
    exe = tmp_path / "main"
    r = subprocess.run(["gcc", "-O1", "-I", str(ROOT / "include"), str(src), "-L", str(lib), "-lsh_ops_cuda",
                        f"-Wl,-rpath,{lib}", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "KAT1024_CHECK ok=1048576/1048576 KAT1024_PASS" in r.stdout
    assert "[Performance Counter]: Execution period is" in r.stdout
    assert "[sh_" not in r.stdout


@pytest.mark.parametrize("S,D,F,H,NL", [(64, 128, 256, 2, 3), (256, 768, 3072, 12, 2)])
def test_looped_encoder_module_on_gpu(gpu_lib, capfd, S, D, F, H, NL):
    """A looped multi-layer module (scf.for over layers with indexed parameter buffers, a nested loop over indexed
    GELU column views; tests/looped_module.py) run through emit_cuda.Program: the residual stream after every layer
    (indexed dumps L1..Ln) and the final output match the stacked oracle layers with the reference's LCG
    parameters (frontend seeds 100 * layer) within the reference's 0.05 / 0.05 (run.py:360-365)."""
    import looped_module as LM
    rt = gpu_lib
    rt.reset()
    text = LM.looped_encoder(S, D, F, H, NL)
    prog = E.Program(text, rt)
    act, poff, stride, base = LM.layout(S, D, F)
    x, _ = siglip.lcg_layer_inputs(S, D, F, 0)
    params = [siglip.lcg_layer_inputs(S, D, F, li)[1] for li in range(NL)]
    rt.put(rt.lib.sh_hbm_addr(act["x"]), x)
    for li, p in enumerate(params):
        for name in LM.PARAMS:
            rt.put(rt.lib.sh_hbm_addr(base + li * stride + poff[name]), p[name])
    capfd.readouterr()
    assert prog.run() == 0
    rt.check()
    out = capfd.readouterr().out
    got = lcg.parse_samples(out)
    cur = x
    scale = 1.0 / np.sqrt(D // H)
    for li in range(NL):
        cur = siglip.layer_reference_arrays(cur, params[li], H, scale=scale)["OUT"]
        tag = f"L{li + 1}"
        assert len(got[tag]) == 32, tag
        bad, err = lcg.compare_samples(got[tag], cur, 0.05, 0.05)
        assert bad == 0, (tag, err)
        assert f"[mark] layer{li + 1} " in out
    final = prog.tensor("x").astype(np.float32)
    err = np.abs(final - cur)
    assert np.all(err <= 0.05 + 0.05 * np.abs(cur)), float(err.max())
