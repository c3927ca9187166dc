"""The batched encoder driver (7 library calls per layer) against the SigLIP layer oracle."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import ops, siglip
from softhier_cuda import encoder

pytestmark = pytest.mark.gpu


def test_layer_reference_lcg_data_s256(gpu_lib):
    """Config 3 with the reference's own LCG data: OUT within the reference's 0.05 tolerance (run.py:321)."""
    x, p = siglip.lcg_layer_inputs(256, 768, 3072, 0)
    want = siglip.layer_reference_arrays(x, p, 12)["OUT"]
    got = encoder.run_layer_once(gpu_lib, x, p, 12, 1e-6, 0.125).astype(np.float32)
    err = np.abs(got - want)
    assert np.all(err <= 0.05 + 0.05 * np.abs(want)), float(err.max())


def test_layer_baseline_distributions_s256(gpu_lib):
    """Config 3 with BASELINE's inputs: x N(0,1), weights N(0,0.02), zero biases, gamma 1 / beta 0."""
    from oracle import lcg
    x = lcg.normal_fp16(256, 768, 7)
    p = siglip.baseline_layer_params(768, 3072, 1)
    want = siglip.layer_reference_arrays(x, p, 12, scale=0.125, rounding=False)["OUT"]
    got = encoder.run_layer_once(gpu_lib, x, p, 12, 1e-6, 0.125).astype(np.float32)
    err, rel = ops.max_abs_and_rel_l2(got, want)
    assert err <= 2e-2 and rel <= 5e-3, (err, rel)


def test_batched_two_layers(gpu_lib):
    from oracle import lcg
    rt = gpu_lib
    rt.reset()
    B, S, D, F, H = 3, 64, 128, 256, 2
    layers = [siglip.baseline_layer_params(D, F, 10 + i) for i in range(2)]
    x = lcg.normal_fp16(B * S, D, 3)
    ws = [encoder.upload_layer(rt, p) for p in layers]
    act = encoder.alloc_activations(rt, B, S, D, F)
    rt.put(act.x, x)
    res = encoder.encoder_forward(rt.lib, act, ws, H, 1e-6, 1.0 / np.sqrt(D // H))
    rt.check()
    got = rt.get(res, B * S, D).astype(np.float32)
    for b in range(B):
        sl = slice(b * S, (b + 1) * S)
        want = siglip.encoder_reference(x[sl], layers, H, scale=1.0 / np.sqrt(D // H), rounding=False)
        err, rel = ops.max_abs_and_rel_l2(got[sl], want)
        assert err <= 2e-2 and rel <= 5e-3, (b, err, rel)


def _run_folded(rt, x, layers, B, S, H, scale):
    """The encoder with both LayerNorms of every layer folded into the GEMMs (sh_cuda_gemm_ln)."""
    rt.reset()
    D = x.shape[1]
    F = np.asarray(layers[0]["w1"]).shape[1]
    ws = [encoder.fold_layer_norms(rt, encoder.upload_layer(rt, p), D, F) for p in layers]
    act = encoder.alloc_activations(rt, B, S, D, F)
    stats = encoder.alloc_row_stats(rt, B * S, D)
    rt.put(act.x, x)
    sched, res = encoder.encoder_schedule_folded(rt.lib, act, ws, stats, H, 1e-6, scale)
    for kind, fn in sched:
        assert fn() == 0, kind
    rt.check()
    return rt.get(res, B * S, D).astype(np.float32), sched


def test_folded_layer_reference_lcg_data_s256(gpu_lib):
    """Config 3 with the reference's LCG data (gamma in [0.5, 1.5], beta and biases nonzero), LayerNorms folded:
    OUT within the reference's 0.05 tolerance of siglip_ref."""
    x, p = siglip.lcg_layer_inputs(256, 768, 3072, 0)
    want = siglip.layer_reference_arrays(x, p, 12)["OUT"]
    got, sched = _run_folded(gpu_lib, x, [p], 1, 256, 12, 0.125)
    assert [k for k, _ in sched] == ["row_stats", "gemm_qkv", "attention", "gemm_o", "gemm_fc1", "gemm_fc2"]
    err = np.abs(got - want)
    assert np.all(err <= 0.05 + 0.05 * np.abs(want)), float(err.max())


def test_folded_batched_two_layers(gpu_lib):
    """BASELINE-like data with random LayerNorm parameters (gamma N(1, 0.02), beta N(0, 0.02)), 3 sequences x 2
    layers: rel-L2 <= 5e-3 and max-abs <= 2e-2 per sequence against the fp32 oracle."""
    from oracle import lcg
    B, S, D, F, H = 3, 64, 128, 256, 2
    layers = []
    for i in range(2):
        p = siglip.baseline_layer_params(D, F, 20 + i)
        for j, (g, b) in enumerate((("g1", "be1"), ("g2", "be2"))):
            p[g] = lcg.normal_fp16(1, D, 300 + 10 * i + j, 1.0, 0.02)
            p[b] = lcg.normal_fp16(1, D, 400 + 10 * i + j, 0.0, 0.02)
        layers.append(p)
    x = lcg.normal_fp16(B * S, D, 5)
    scale = 1.0 / np.sqrt(D // H)
    got, _ = _run_folded(gpu_lib, x, layers, B, S, H, scale)
    for b in range(B):
        sl = slice(b * S, (b + 1) * S)
        want = siglip.encoder_reference(x[sl], layers, H, scale=scale, rounding=False)
        err, rel = ops.max_abs_and_rel_l2(got[sl], want)
        assert rel <= 5e-3 and err <= 2e-2, (b, err, rel)


def test_gemm_ln_rejects_bad_shapes(gpu_lib, capfd):
    from softhier_cuda import lib as L
    rt = gpu_lib
    rt.reset()
    x, w, z = rt.alloc(128, 96), rt.alloc(96, 128), rt.alloc(128, 128)
    c, s = rt.alloc_bytes(128 * 4), rt.alloc_bytes(128 * 8)
    # K = 96 is not a multiple of 64: no LayerNorm statistics layout for it
    assert rt.lib.sh_cuda_gemm_ln(x, w, z, 128, 128, 96, 96, 128, 128, 0, 0, 0, L.EPI_LN_IN, s, c, 1e-6, 0) == -1
    cap = capfd.readouterr()
    assert "[sh_cuda_gemm_ln]" in cap.out + cap.err
    assert rt.lib.sh_cuda_row_stats(x, 128, 96, 96, s) == -1
    assert rt.lib.sh_cuda_last_error() == -1      # reported, and cleared by reading it
    rt.check()
