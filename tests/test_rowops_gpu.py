"""Row / elementwise ops through the C ABI against the oracle (tests/gvsoc/run.py:136-173 semantics)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import lcg, ops

pytestmark = pytest.mark.gpu
A = 0xFFFFFFFF


def _tol_ok(got, want, atol=2e-2, rtol=2e-2):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    return np.all(np.abs(got - want) <= atol + rtol * np.abs(want)), float(np.abs(got - want).max())


def _baseline_err(got, want):
    err, rel = ops.max_abs_and_rel_l2(np.asarray(got, np.float32), want)
    assert err <= 2e-2 and rel <= 5e-3, (err, rel)


@pytest.mark.parametrize("rows,cols", [(256, 768), (256, 3072), (37, 100), (5, 8), (3, 4096), (2, 5000)])
def test_rowops_match_oracle(gpu_lib, rows, cols):
    rt = gpu_lib
    lib = rt.lib
    rt.reset()
    x = lcg.normal_fp16(rows, cols, 11)
    b = lcg.normal_fp16(rows, cols, 12)
    g = lcg.normal_fp16(1, cols, 13, 1.0, 0.02)
    be = lcg.normal_fp16(1, cols, 14, 0.0, 0.02)
    dx, db, dg, dbe = (rt.upload(a) for a in (x, b, g, be))
    outs = {k: rt.alloc(rows, cols) for k in ("ln", "sm", "ge", "ad", "bi", "sc")}
    lib.sh_layernorm(outs["ln"], dx, dg, dbe, rows, cols, cols, 1e-6, A)
    lib.sh_softmax_rows(outs["sm"], dx, rows, cols, cols, 0.125, A)
    lib.sh_gelu(outs["ge"], dx, rows, cols, cols, A)
    lib.sh_add(outs["ad"], dx, db, rows, cols, cols, A)
    lib.sh_add_bias(outs["bi"], dx, dbe, rows, cols, cols, A)
    lib.sh_scale(outs["sc"], dx, rows, cols, cols, 0.125, A)
    tr = rt.alloc(cols, rows)
    lib.sh_transpose(tr, dx, rows, cols, cols, rows, A)
    rt.check()
    ref = {"ln": ops.layernorm(x, g, be, 1e-6), "sm": ops.softmax_rows(x, 0.125), "ge": ops.gelu(x),
           "ad": ops.add(x, b), "bi": ops.add_bias(x, be), "sc": ops.scale(x, 0.125)}
    for k, want in ref.items():
        got = rt.get(outs[k], rows, cols)
        ok, err = _tol_ok(got, want)
        assert ok, (k, err)
        _baseline_err(got, want)
    assert (rt.get(tr, cols, rows).view(np.uint16) == x.T.view(np.uint16)).all()


def test_rowops_reference_rowops_case(gpu_lib):
    """The reference's own rowops test data (run.py:138-158: LCG x/b/g/be, eps 1e-5, softmax 0.5, scale 0.3)."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    R, C = 256, 768
    x = lcg.fill_fp16(R, C, 11, -16, 16, 0.125)
    b = lcg.fill_fp16(R, C, 12, -16, 16, 0.125)
    g = lcg.fill_fp16(1, C, 13, 1, 8, 0.25)
    be = lcg.fill_fp16(1, C, 14, -4, 4, 0.25)
    dx, db, dg, dbe = (rt.upload(a) for a in (x, b, g, be))
    o = {k: rt.alloc(R, C) for k in ("LN", "SM", "GELU", "ADD", "BIAS", "SCALE")}
    lib.sh_layernorm(o["LN"], dx, dg, dbe, R, C, C, 1e-5, A)
    lib.sh_softmax_rows(o["SM"], dx, R, C, C, 0.5, A)
    lib.sh_gelu(o["GELU"], dx, R, C, C, A)
    lib.sh_add(o["ADD"], dx, db, R, C, C, A)
    lib.sh_add_bias(o["BIAS"], dx, dbe, R, C, C, A)
    lib.sh_scale(o["SCALE"], dx, R, C, C, 0.3, A)
    rt.check()
    ref = {"LN": ops.layernorm(x, g, be, 1e-5), "SM": ops.softmax_rows(x, 0.5), "GELU": ops.gelu(x),
           "ADD": ops.add(x, b), "BIAS": ops.add_bias(x, be), "SCALE": ops.scale(x, 0.3)}
    for k, want in ref.items():
        ok, err = _tol_ok(rt.get(o[k], R, C), want)
        assert ok, (k, err)


def test_rowops_strided_views_and_in_place(gpu_lib):
    """Views with a leading dim > cols and odd element offsets take the element-wise path; outputs may alias."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    R, LD = 64, 768
    full = lcg.normal_fp16(R, LD, 5)
    base = rt.upload(full)
    for off, cols in [(64, 64), (3, 61), (128, 256)]:
        view = base + 2 * off
        want = ops.gelu(full[:, off:off + cols])
        lib.sh_gelu(view, view, R, cols, LD, A)       # in place, strided
        rt.check()
        got = rt.get(view, R, cols, LD)
        ok, err = _tol_ok(got, want)
        assert ok, (off, cols, err)
        rt.put(view, full[:, off:off + cols], LD)     # restore
    # layernorm + softmax in place on a strided view
    v = base + 2 * 128
    lib.sh_softmax_rows(v, v, R, 256, LD, -0.7, A)    # negative scale
    rt.check()
    ok, err = _tol_ok(rt.get(v, R, 256, LD), ops.softmax_rows(full[:, 128:384], -0.7))
    assert ok, err


def test_add_layernorm_fused(gpu_lib):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    R, C = 300, 768
    a, b = lcg.normal_fp16(R, C, 1), lcg.normal_fp16(R, C, 2)
    g, be = lcg.normal_fp16(1, C, 3, 1.0, 0.02), lcg.normal_fp16(1, C, 4, 0.0, 0.02)
    da, db, dg, dbe = (rt.upload(t) for t in (a, b, g, be))
    h, y = rt.alloc(R, C), rt.alloc(R, C)
    lib.sh_cuda_add_layernorm(h, y, da, db, dg, dbe, R, C, C, 1e-6)
    rt.check()
    hr = ops.r16(ops.add(a, b))
    assert (rt.get(h, R, C) == hr.astype(np.float16)).all()
    ok, err = _tol_ok(rt.get(y, R, C), ops.layernorm(hr, g, be, 1e-6))
    assert ok, err


@pytest.mark.parametrize("rows", [1, 3, 301])
@pytest.mark.parametrize("cols,ld", [(528, 528), (640, 648), (768, 768), (768, 1024)])
def test_layernorm_two_rows_per_warp(gpu_lib, rows, cols, ld):
    """528-768 columns run two rows per warp (16 lanes per row): an odd row count leaves the second half of the last
    warp past the end (it still takes part in the shuffles), a leading dim above cols leaves a gap between rows that
    must stay untouched; plain and fused with the residual add."""
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    a, b = lcg.normal_fp16(rows, ld, 11), lcg.normal_fp16(rows, ld, 12)
    g, be = lcg.normal_fp16(1, cols, 13, 1.0, 0.1), lcg.normal_fp16(1, cols, 14, 0.0, 0.1)
    da, db, dg, dbe = (rt.upload(t) for t in (a, b, g, be))
    sentinel = np.full((rows, ld), 7.0, np.float16)
    y, h, y2 = rt.upload(sentinel), rt.upload(sentinel), rt.upload(sentinel)
    lib.sh_layernorm(y, da, dg, dbe, rows, cols, ld, 1e-6, A)
    lib.sh_cuda_add_layernorm(h, y2, da, db, dg, dbe, rows, cols, ld, 1e-6)
    rt.check()
    got, hs, got2 = (rt.get(p, rows, ld) for p in (y, h, y2))
    ok, err = _tol_ok(got[:, :cols], ops.layernorm(a[:, :cols], g, be, 1e-6))
    assert ok, err
    hr = ops.r16(ops.add(a[:, :cols], b[:, :cols]))
    assert (hs[:, :cols] == hr.astype(np.float16)).all()
    ok, err = _tol_ok(got2[:, :cols], ops.layernorm(hr, g, be, 1e-6))
    assert ok, err
    for t in (got, hs, got2):   # the columns between cols and ld are not written
        assert (t[:, cols:] == 7.0).all()


def test_transpose_ragged_and_strided(gpu_lib):
    rt, lib = gpu_lib, gpu_lib.lib
    rt.reset()
    for rows, cols, lds, ldd in [(256, 3072, 3072, 256), (65, 130, 131, 70), (1, 7, 7, 1), (129, 64, 64, 129)]:
        x = lcg.fill_fp16(rows, lds, rows + cols, -1024, 1023, 1 / 1024)
        src = rt.upload(x)
        dst = rt.alloc(cols, ldd)
        lib.sh_transpose(dst, src, rows, cols, lds, ldd, A)
        rt.check()
        got = rt.get(dst, cols, rows, ldd)
        assert (got.view(np.uint16) == x[:, :cols].T.view(np.uint16)).all(), (rows, cols)
