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
    assert err <= 2e-2 * max(1.0, float(np.abs(want).max()) / 4) and rel <= 5e-3, (err, rel)


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
        assert rel <= 5e-3, (b, err, rel)
