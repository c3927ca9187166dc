"""Fused attention through the C ABI against the reference's attention_reference (golden) and the oracle."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import lcg, ops

pytestmark = pytest.mark.gpu
A = 0xFFFFFFFF


def _check(got, want, atol=0.05, rtol=0.05):
    got = np.asarray(got, np.float32)
    err = np.abs(got - want)
    assert np.all(err <= atol + rtol * np.abs(want)), float(err.max())


@pytest.mark.parametrize("S,D,H", [(64, 128, 2), (256, 768, 12)])
def test_attention_matches_reference_golden(gpu_lib, S, D, H):
    """tests/gvsoc/run.py attention case: LCG q/k/v (seeds 21-23), scale 0.125, tol 0.05 (run.py:963)."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    q = lcg.fill_fp16(S, D, 21, -8, 8, 0.125)
    k = lcg.fill_fp16(S, D, 22, -8, 8, 0.125)
    v = lcg.fill_fp16(S, D, 23, -16, 16, 0.125)
    dq, dk, dv = rt.upload(q), rt.upload(k), rt.upload(v)
    do = rt.alloc(S, D)
    lib.sh_test_fill_int_fp16(do, S, D, D, 24, 7, 7)    # poison (attention/main.c fills o with 7.0)
    assert lib.sh_attention(dq, dk, dv, do, S, D, H, D, D, D, D, 0.125, A) == 0
    rt.check()
    want = golden("attention.npz")[f"{S}_{D}_{H}_o"].view(np.float16).astype(np.float32)
    got = rt.get(do, S, D)
    _check(got, want)
    err, rel = ops.max_abs_and_rel_l2(got, ops.attention(q, k, v, H, 0.125, rounding=False))
    assert err <= 2e-2 and rel <= 5e-3, (err, rel)


def test_attention_packed_qkv_layout(gpu_lib):
    """attention_translate.mlir: q / k / v are column slices of one [S, 3D] buffer (ld 2304)."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    S, D, H = 256, 768, 12
    qkv = lcg.normal_fp16(S, 3 * D, 9)
    base = rt.upload(qkv)
    do = rt.alloc(S, D)
    assert lib.sh_attention(base, base + 2 * D, base + 4 * D, do, S, D, H, 3 * D, 3 * D, 3 * D, D, 0.125, A) == 0
    rt.check()
    want = ops.attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], H, 0.125, rounding=False)
    got = rt.get(do, S, D)
    err, rel = ops.max_abs_and_rel_l2(got, want)
    assert err <= 2e-2 and rel <= 5e-3, (err, rel)
    # sh_attention_q with an explicit q block gives the same numbers
    do2 = rt.alloc(S, D)
    assert lib.sh_attention_q(base, base + 2 * D, base + 4 * D, do2, S, D, H, 3 * D, 3 * D, 3 * D, D, 0.125, A, 64) == 0
    rt.check()
    assert np.array_equal(rt.get(do2, S, D), got)


@pytest.mark.parametrize("S,dh,H,B", [(256, 64, 12, 4), (200, 64, 2, 3), (1024, 64, 2, 1), (96, 32, 4, 2),
                                      (128, 128, 2, 2), (52, 16, 1, 1), (300, 64, 2, 2)])
@pytest.mark.parametrize("sign", [1.0, -1.0])
def test_attention_batched_shapes(gpu_lib, S, dh, H, B, sign):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    D = dh * H
    q, k, v = (lcg.normal_fp16(B * S, D, s) for s in (1, 2, 3))
    dq, dk, dv = rt.upload(q), rt.upload(k), rt.upload(v)
    do = rt.alloc(B * S, D)
    scale = sign / np.sqrt(dh)
    assert lib.sh_cuda_attention_batched(dq, dk, dv, do, S, D, H, D, D, D, D, scale, B) == 0
    rt.check()
    got = rt.get(do, B * S, D)
    for b in range(B):
        sl = slice(b * S, (b + 1) * S)
        want = ops.attention(q[sl], k[sl], v[sl], H, scale, rounding=False)
        err, rel = ops.max_abs_and_rel_l2(got[sl], want)
        assert err <= 2e-2 and rel <= 5e-3, (b, err, rel)


@pytest.mark.parametrize("S,H,B,scale", [(132, 3, 2, 0.125), (4, 1, 3, 0.125), (256, 12, 2, -0.125),
                                          (200, 2, 2, -0.3), (128, 4, 3, 0.125)])
def test_attention_single_block_cases(gpu_lib, S, H, B, scale):
    """Edge cases of the tensor-core kernel at S <= 256: a second query tile with 4 valid rows and 4 valid keys in
    the second key block (S = 132), tiny S, a negative softmax scale (the row max of s * scale is the minimum of s,
    and masked keys must still get p = 0), and one query tile only (S = 128); nothing is written outside the output
    columns."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    D = 64 * H
    q, k, v = (lcg.normal_fp16(B * S, D, s) for s in (31, 32, 33))
    dq, dk, dv = rt.upload(q), rt.upload(k), rt.upload(v)
    do = rt.alloc(B * S, D + 64)
    rt.view(do, B * S, D + 64).fill_(3.0)
    assert lib.sh_cuda_attention_batched(dq, dk, dv, do, S, D, H, D, D, D, D + 64, scale, B) == 0
    rt.check()
    got = rt.get(do, B * S, D + 64)
    assert (got[:, D:] == 3.0).all()              # nothing written outside the output columns
    for b in range(B):
        sl = slice(b * S, (b + 1) * S)
        want = ops.attention(q[sl], k[sl], v[sl], H, scale, rounding=False)
        err, rel = ops.max_abs_and_rel_l2(got[sl, :D], want)
        assert err <= 2e-2 and rel <= 5e-3, (b, err, rel)


def test_attention_head_and_errors(gpu_lib, capfd):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    S, D = 128, 64
    q, k, v = (lcg.normal_fp16(S, D, s) for s in (4, 5, 6))
    dq, dk, dv, do = rt.upload(q), rt.upload(k), rt.upload(v), rt.alloc(S, D)
    assert lib.sh_attention_head(dq, dk, dv, do, S, D, D, D, D, D, 0.125, 0) == 0
    rt.check()
    err, rel = ops.max_abs_and_rel_l2(rt.get(do, S, D), ops.attention(q, k, v, 1, 0.125, rounding=False))
    assert err <= 2e-2 and rel <= 5e-3
    capfd.readouterr()
    assert lib.sh_attention(dq, dk, dv, do, S, 100, 3, D, D, D, D, 0.125, A) == -1     # D % H
    assert "[sh_attention] D=100 not divisible by H=3" in capfd.readouterr().out
    assert lib.sh_attention_q(dq, dk, dv, do, S, D, 1, D, D, D, D, 0.125, A, 48) == -1  # sq does not divide S
    assert lib.sh_attention(dq, dk, dv, do, 130, D, 1, D, D, D, D, 0.125, A) == -1     # S % 4
    lib.sh_cuda_last_error()
