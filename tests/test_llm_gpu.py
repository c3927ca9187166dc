"""Llama-style decoder ops (runtime/sh_llm.inc.c) on the GPU against the reference's numpy twins (tests/golden/llm.npz)
and the oracle restatement (oracle/llm.py)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import lcg, llm, ops

pytestmark = pytest.mark.gpu
A = 0xFFFFFFFF


def _ulps(a: np.ndarray, b: np.ndarray) -> int:
    ia = a.astype(np.float16).view(np.int16).astype(np.int32)
    ib = b.astype(np.float16).view(np.int16).astype(np.int32)
    return int(np.abs(ia - ib).max())


def _h(g, k):
    return g[k].view(np.float16)


def test_rmsnorm_rope_silu_pixel_shuffle_match_reference(gpu_lib):
    rt, lib, g = gpu_lib, gpu_lib.lib, golden("llm.npz")
    rt.reset()
    x, gm = _h(g, "rms_x"), _h(g, "rms_g")
    dx, dg, dy = rt.upload(x), rt.upload(gm), rt.alloc(*x.shape)
    lib.sh_rmsnorm(dy, dx, dg, x.shape[0], x.shape[1], x.shape[1], 1e-5, A)
    assert _ulps(rt.get(dy, *x.shape), _h(g, "rms_y")) <= 1

    xr, tab = _h(g, "rope_x"), _h(g, "rope_tab")
    dx, dt, dy = rt.upload(xr), rt.upload(tab), rt.alloc(*xr.shape)
    lib.sh_rope(dy, dx, dt, xr.shape[0], xr.shape[1], xr.shape[1], tab.shape[1], 64, A)
    assert _ulps(rt.get(dy, *xr.shape), _h(g, "rope_y")) <= 1

    a, b = _h(g, "silu_a"), _h(g, "silu_b")
    da, db, dy = rt.upload(a), rt.upload(b), rt.alloc(*a.shape)
    lib.sh_silu_mul(dy, da, db, a.shape[0], a.shape[1], a.shape[1], A)
    assert _ulps(rt.get(dy, *a.shape), _h(g, "silu_y")) <= 2

    ps = _h(g, "ps_x")
    dx, dy = rt.upload(ps), rt.alloc(4, 16 * 32)
    lib.sh_pixel_shuffle(dy, dx, 8, 32, 4, A)
    np.testing.assert_array_equal(rt.get(dy, 4, 512).view(np.uint16), g["ps_y"])      # data movement: bit-exact
    rt.check()


def test_softmax_masked_against_oracle(gpu_lib):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    R, C = 96, 200
    x = lcg.normal_fp16(R, C, 51)
    rng = np.random.default_rng(5)
    tq = rng.integers(0, 4, R).astype(np.uint16)
    tk = rng.integers(0, 4, C).astype(np.uint16)
    tq[[3, 50]] = llm.PAD
    tk[[7, 8, 199]] = llm.PAD
    dx, dy = rt.upload(x), rt.alloc(R, C)
    dtq, dtk = rt.alloc_bytes(R * 2), rt.alloc_bytes(C * 2)
    rt.put_bytes(dtq, tq.tobytes())
    rt.put_bytes(dtk, tk.tobytes())
    lib.sh_softmax_masked(dy, dx, R, C, C, 0.3, dtq, dtk, A)
    got = rt.get(dy, R, C).astype(np.float32)
    want = llm.softmax_masked(x, 0.3, tq, tk, rounding=False)
    assert np.abs(got - want).max() <= 2e-3
    assert np.all(got[np.asarray(tq)[:, None] < tk[None, :]] == 0)
    rt.check()


def test_gqa_masked_attention_matches_reference(gpu_lib):
    """GQA (3 query heads on 1 key/value head) with a padding-token mask, against the reference twin on the rows of
    non-PAD queries and the oracle on PAD query rows (uniform)."""
    rt, lib, g = gpu_lib, gpu_lib.lib, golden("llm.npz")
    rt.reset()
    q, k, v, tok = _h(g, "gqa_q"), _h(g, "gqa_k"), _h(g, "gqa_v"), g["gqa_tok"]
    S = q.shape[0]
    dq, dk, dv, do = rt.upload(q), rt.upload(k), rt.upload(v), rt.alloc(S, q.shape[1])
    dt = rt.alloc_bytes(S * 2)
    rt.put_bytes(dt, tok.astype(np.uint16).tobytes())
    assert lib.sh_attention_gqa(dq, dk, dv, do, S, 192, 3, 1, 192, 64, 64, 192, 0.125, dt, A) == 0
    got = rt.get(do, S, 192).astype(np.float32)
    rows = tok != llm.PAD
    want = _h(g, "gqa_o").astype(np.float32)
    assert np.abs(got[rows] - want[rows]).max() <= 2e-2
    ora = llm.attention_gqa(q, k, v, 3, 1, 0.125, tok, rounding=False)
    assert np.abs(got - ora).max() <= 2e-2
    rt.check()


@pytest.mark.parametrize("S,H,Hkv,masked", [(256, 6, 2, False), (200, 4, 1, False), (96, 4, 2, True)])
def test_gqa_and_head_masked_shapes(gpu_lib, S, H, Hkv, masked):
    """dh = 64: unmasked GQA runs on the tensor-core kernel (K / V head h / (H / Hkv)); masked on the CUDA cores."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    dh = 64
    q = lcg.normal_fp16(S, H * dh, 61)
    k = lcg.normal_fp16(S, Hkv * dh, 62)
    v = lcg.normal_fp16(S, Hkv * dh, 63)
    tok = None
    dt = 0
    if masked:
        tok = (np.arange(S) // 8).astype(np.uint16)      # block-causal classes
        tok[[10, 11]] = llm.PAD
        dt = rt.alloc_bytes(S * 2)
        rt.put_bytes(dt, tok.tobytes())
    dq, dk, dv, do = rt.upload(q), rt.upload(k), rt.upload(v), rt.alloc(S, H * dh)
    assert lib.sh_attention_gqa(dq, dk, dv, do, S, H * dh, H, Hkv, H * dh, Hkv * dh, Hkv * dh, H * dh, 0.125, dt,
                                A) == 0
    got = rt.get(do, S, H * dh).astype(np.float32)
    want = llm.attention_gqa(q, k, v, H, Hkv, 0.125, tok, rounding=False)
    err, rel = ops.max_abs_and_rel_l2(got, want)
    assert err <= 2e-2 and rel <= 5e-3, (err, rel)
    if masked:   # one head through sh_attention_head_masked (head 1 reads key / value head 1 // (H / Hkv))
        kvh = 1 // (H // Hkv)
        do1 = rt.alloc(S, dh)
        assert lib.sh_attention_head_masked(dq + 2 * dh, dk + 2 * kvh * dh, dv + 2 * kvh * dh, do1, S, dh, H * dh,
                                            Hkv * dh, Hkv * dh, dh, 0.125, dt, A) == 0
        np.testing.assert_allclose(rt.get(do1, S, dh).astype(np.float32), want[:, dh:2 * dh], atol=2e-2)
    rt.check()


def test_llm_errors(gpu_lib, capfd):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    x = rt.alloc(64, 128)
    assert lib.sh_attention_gqa(x, x, x, x, 64, 128, 2, 3, 128, 128, 128, 128, 0.125, 0, A) == -1   # H % Hkv
    lib.sh_rope(x, x, x, 64, 128, 128, 64, 12, A)                                                   # dh % 8
    cap = capfd.readouterr()
    assert "[sh_attention_gqa] bad D=128 H=2 Hkv=3" in cap.out + cap.err
    assert "[sh_rope]" in cap.out + cap.err
    assert lib.sh_cuda_last_error() == -1
    rt.check()


DECODER = """builtin.module {
  func.func @dec() {
    %x   = softhier.hbm_buffer {offset = 65536 : i32}  : memref<128x192xf16, "hbm_west">
    %g   = softhier.hbm_buffer {offset = 131072 : i32} : memref<1x192xf16, "hbm_west">
    %ln  = softhier.hbm_buffer {offset = 139264 : i32} : memref<128x192xf16, "hbm_west">
    %tab = softhier.hbm_buffer {offset = 196608 : i32} : memref<128x64xf16, "hbm_west">
    %tok = softhier.hbm_buffer {offset = 229376 : i32} : memref<128xi16, "hbm_west">
    %kv  = softhier.hbm_buffer {offset = 233472 : i32} : memref<128x128xf16, "hbm_west">
    %o   = softhier.hbm_buffer {offset = 270336 : i32} : memref<128x192xf16, "hbm_west">
    %m   = softhier.hbm_buffer {offset = 327680 : i32} : memref<128x192xf16, "hbm_west">
    %k = softhier.view %kv : memref<128x128xf16, "hbm_west"> -> memref<128x64xf16, strided<[128, 1], offset: 0>, "hbm_west">
    %v = softhier.view %kv : memref<128x128xf16, "hbm_west"> -> memref<128x64xf16, strided<[128, 1], offset: 64>, "hbm_west">
    softhier.hbm_fill_lcg %x {seed = 71 : i32, lo = -64 : i32, hi = 64 : i32, scale = 0.03125 : f32} : memref<128x192xf16, "hbm_west">
    softhier.hbm_fill_lcg %g {seed = 72 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x192xf16, "hbm_west">
    softhier.hbm_fill_lcg %tab {seed = 73 : i32, lo = -32 : i32, hi = 32 : i32, scale = 0.03125 : f32} : memref<128x64xf16, "hbm_west">
    softhier.hbm_fill_lcg %kv {seed = 74 : i32, lo = -32 : i32, hi = 32 : i32, scale = 0.03125 : f32} : memref<128x128xf16, "hbm_west">
    softhier.rmsnorm %x, %g -> %ln {eps = 1.0e-5 : f32, cluster = -1 : i32} : memref<128x192xf16, "hbm_west">, memref<1x192xf16, "hbm_west"> -> memref<128x192xf16, "hbm_west">
    softhier.rope %ln, %tab -> %ln {head_dim = 64 : i32, cluster = -1 : i32} : memref<128x192xf16, "hbm_west">, memref<128x64xf16, "hbm_west"> -> memref<128x192xf16, "hbm_west">
    softhier.attention %ln, %k, %v, %tok -> %o {scale = 0.125 : f32, heads = 3 : i32, kv_heads = 1 : i32, cluster = -1 : i32}
        : memref<128x192xf16, "hbm_west">, memref<128x64xf16, strided<[128, 1], offset: 0>, "hbm_west">, memref<128x64xf16, strided<[128, 1], offset: 64>, "hbm_west">, memref<128xi16, "hbm_west"> -> memref<128x192xf16, "hbm_west">
    softhier.silu_mul %o, %x -> %m {cluster = -1 : i32} : memref<128x192xf16, "hbm_west">, memref<128x192xf16, "hbm_west"> -> memref<128x192xf16, "hbm_west">
    func.return
  }
}
"""


def test_decoder_module_through_emit_cuda(gpu_lib, capfd):
    """A decoder block in the dialect (rmsnorm -> rope -> masked GQA attention on a strided K|V buffer -> silu-mul),
    lowered by emit_cuda and run in-process, against the oracle chain."""
    from softhier_cuda import emit_cuda as E
    rt = gpu_lib
    rt.reset()
    prog = E.Program(DECODER, rt)
    assert prog.run_phase("prologue") == 0
    tok = (np.arange(128) // 16).astype(np.uint16)
    tok[[9, 100]] = llm.PAD
    rt.put_bytes(prog.address("tok")[0], tok.tobytes())
    assert prog.run_phase("kernel") == 0
    rt.check()
    x, g, tab, kv = (prog.tensor(n).astype(np.float32) for n in ("x", "g", "tab", "kv"))
    ln = llm.rope(llm.rmsnorm(x, g), tab, 64)
    o = llm.attention_gqa(ln, kv[:, :64], kv[:, 64:], 3, 1, 0.125, tok, rounding=False)
    want = llm.silu_mul(llm.r16(o), x, rounding=False)
    got = prog.tensor("m").astype(np.float32)
    err, rel = ops.max_abs_and_rel_l2(got, want)
    assert err <= 2e-2 and rel <= 5e-3, (err, rel)
