"""Parity of the benchmarked configuration: the 12-layer SigLIP-base encoder at batch 512.

The encoder runs exactly as bench.py sets it up (softhier_cuda.encoder.synthetic_encoder: weights and input
generated on the GPU by the library's N(mean, std) fill) and through the same 7-launch layer schedule, on the full
512 x 256-token batch. The test then checks:
  * the generated inputs: every weight matrix of all 12 layers and the input rows of the sampled sequences are
    bit-identical to the oracle's generator (oracle.lcg.normal_fp16), so the oracle sees the bench's exact data;
  * the output: sampled sequences (first, second, middle, last) against the fp32 numpy encoder
    (oracle.siglip.encoder_reference, no fp16 rounding points: the fp32 result north_star names), after every
    layer, with the flat bound max-abs <= 2e-2 and rel-L2 <= 5e-3 on the final output.
Reference: softhier_mlir/testing/siglip_ref.py:20-45 (one layer), frontend/siglip.py:168 (layers stacked).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import lcg, ops, siglip
from softhier_cuda import encoder

pytestmark = pytest.mark.gpu

S, D, F, H, LAYERS, B = 256, 768, 3072, 12, 12, 512
EPS, SCALE = 1e-6, 0.125
SAMPLED = (0, 1, 255, 511)
MAX_ABS, REL_L2 = 2e-2, 5e-3


def _oracle_params(layer: int) -> dict[str, np.ndarray]:
    sd = encoder.synthetic_weight_seeds(layer)
    wqkv = lcg.normal_fp16(D, 3 * D, sd["wqkv"], 0.0, 0.02)
    p = {"wq": wqkv[:, :D], "wk": wqkv[:, D:2 * D], "wv": wqkv[:, 2 * D:],
         "wo": lcg.normal_fp16(D, D, sd["wo"], 0.0, 0.02), "w1": lcg.normal_fp16(D, F, sd["w1"], 0.0, 0.02),
         "w2": lcg.normal_fp16(F, D, sd["w2"], 0.0, 0.02)}
    z = lambda c: np.zeros((1, c), np.float16)  # noqa: E731
    o = lambda c: np.ones((1, c), np.float16)   # noqa: E731
    p.update(bq=z(D), bk=z(D), bv=z(D), bo=z(D), b1=z(F), b2=z(D), g1=o(D), be1=z(D), g2=o(D), be2=z(D))
    return p, wqkv


@pytest.mark.parametrize("fold", ["none", "ln1"])
def test_encoder_config5_matches_fp32_oracle(gpu_lib, fold):
    """fold = "ln1": LN1 folded into the QKV GEMM (bench.py --ln-fold ln1), row statistics from FC2's epilogue."""
    import torch

    from softhier_cuda.runtime import Runtime
    M = B * S
    arena = (11 * M * D + M * F + LAYERS * (7 * D * D + 3 * D * F + 16 * F)) * 2 + (160 << 20)
    rt = Runtime(0, arena)          # its own arena; gpu_lib's is bound again at the end
    try:
        lib = rt.lib
        layers, act, x_in = encoder.synthetic_encoder(rt, B, S, D, F, LAYERS, encoder.INPUT_SEED0)
        rt.check()
        # the generated data are the oracle's, bit for bit
        params = []
        for li, w in enumerate(layers):
            p, wqkv = _oracle_params(li)
            for name, addr, want in (("wqkv", w.wqkv, wqkv), ("wo", w.wo, p["wo"]), ("w1", w.w1, p["w1"]),
                                     ("w2", w.w2, p["w2"])):
                got = rt.get(addr, *want.shape)
                assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), (li, name)
            for name, addr, n, code in (("bqkv", w.bqkv, 3 * D, 0), ("g1", w.g1, D, 0x3C00), ("b1", w.b1, F, 0)):
                assert (rt.get(addr, 1, n).view(np.uint16) == code).all(), (li, name)
            params.append(p)
        xs = {}
        for b in SAMPLED:
            want = lcg.normal_fp16(S, D, encoder.INPUT_SEED0, 0.0, 1.0, row0=b * S)
            got = rt.get(x_in + b * S * D * 2, S, D)
            assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), b
            xs[b] = want

        # the encoder, layer by layer, on the whole batch; sampled sequences read back after every layer
        cur, nxt = x_in, act.out
        ref = {b: xs[b].astype(np.float32) for b in SAMPLED}
        growth = []
        if fold == "ln1":
            folded = [encoder.fold_layer_norm1(rt, w, D) for w in layers]
            stats_x = encoder.alloc_row_stats(rt, M, D)[0]
            assert lib.sh_cuda_row_stats(x_in, M, D, D, stats_x) == 0
        for li, w in enumerate(layers):
            ops_l = (encoder.layer_ops(lib, act, w, H, EPS, SCALE, cur, nxt) if fold == "none" else
                     encoder.layer_ops_ln1_folded(lib, act, folded[li], stats_x, H, EPS, SCALE, cur, nxt))
            for kind, fn in ops_l:
                assert fn() == 0, (li, kind)
            rt.check()
            errs = []
            for b in SAMPLED:
                ref[b] = siglip.layer_reference_arrays(ref[b], params[li], H, EPS, rounding=False,
                                                       scale=SCALE)["OUT"]
                got = rt.get(nxt + b * S * D * 2, S, D).astype(np.float32)
                errs.append(ops.max_abs_and_rel_l2(got, ref[b]) + (float(np.abs(ref[b]).max()),))
            growth.append((li, max(e[0] for e in errs), max(e[1] for e in errs), max(e[2] for e in errs)))
            cur, nxt = nxt, (act.x if nxt == act.out else act.out)
        for li, err, rel, amax in growth:
            print(f"layer {li + 1:2d}: max-abs {err:.4g}  rel-L2 {rel:.4g}  max|ref| {amax:.3g}")
        final_err, final_rel = growth[-1][1], growth[-1][2]
        assert final_err <= MAX_ABS and final_rel <= REL_L2, growth[-1]
    finally:
        del rt
        torch.cuda.synchronize()
        gpu_lib.activate()
