"""SigLIP / ViT pre-LN encoder-layer reference (TEST INFRASTRUCTURE ONLY).

`layer_reference_arrays` follows softhier_mlir/testing/siglip_ref.py:20-45 step for step
(fp32 math on fp16 data, `r16` after every op the device stores, per-head attention with the
scores rounded before scaling), but takes the input and parameters as arrays so BASELINE's
N(0, 0.02) weights can be used. `lcg_layer_inputs` reproduces the reference's own parameter
scheme (siglip_ref.py:12-18 == frontend/siglip.py:110-124, seeds 1..17 + 100 * layer), so
`layer_reference(S, D, F, H)` equals the reference's `layer_reference` bit for bit (pinned by
tests/golden/siglip_*.npz).

Parameter layout: weights are [in, out] (X . W convention), biases / gamma / beta are 1 x cols.
"""
from __future__ import annotations

import numpy as np

from . import lcg
from .ops import f32, gelu, layernorm, r16, softmax_rows

PARAM_NAMES = ("wq", "wk", "wv", "wo", "w1", "w2", "bq", "bk", "bv", "bo", "b1", "b2", "g1", "be1", "g2", "be2")


def lcg_layer_inputs(S: int, D: int, F: int, layer: int = 0) -> tuple[np.ndarray, dict[str, np.ndarray]]:
    """The input x and layer `layer`'s parameters as the reference's frontend fills them (fp16)."""
    s0 = 100 * layer
    f = lcg.fill_fp16
    x = f(S, D, 1, -16, 16, 0.125)
    p = {
        "wq": f(D, D, 2 + s0, -8, 8, 1 / 128), "wk": f(D, D, 3 + s0, -8, 8, 1 / 128),
        "wv": f(D, D, 4 + s0, -8, 8, 1 / 128), "wo": f(D, D, 5 + s0, -8, 8, 1 / 128),
        "w1": f(D, F, 6 + s0, -8, 8, 1 / 128), "w2": f(F, D, 7 + s0, -8, 8, 1 / 256),
        "bq": f(1, D, 8 + s0, -4, 4, 0.0625), "bk": f(1, D, 9 + s0, -4, 4, 0.0625),
        "bv": f(1, D, 10 + s0, -4, 4, 0.0625), "bo": f(1, D, 11 + s0, -4, 4, 0.0625),
        "b1": f(1, F, 12 + s0, -4, 4, 0.0625), "b2": f(1, D, 13 + s0, -4, 4, 0.0625),
        "g1": f(1, D, 14 + s0, 2, 6, 0.25), "be1": f(1, D, 15 + s0, -4, 4, 0.125),
        "g2": f(1, D, 16 + s0, 2, 6, 0.25), "be2": f(1, D, 17 + s0, -4, 4, 0.125),
    }
    return x, p


def baseline_layer_params(D: int, F: int, seed: int, gamma_beta: str = "identity") -> dict[str, np.ndarray]:
    """BASELINE's synthetic weights: N(0, 0.02) matrices (one LCG seed per matrix, derived from
    `seed`), zero biases, gamma = 1 and beta = 0 ("identity"). fp16."""
    ws = {nm: lcg.normal_fp16(r, c, seed * 64 + i, 0.0, 0.02)
          for i, (nm, r, c) in enumerate([("wq", D, D), ("wk", D, D), ("wv", D, D), ("wo", D, D),
                                          ("w1", D, F), ("w2", F, D)])}
    z = lambda c: np.zeros((1, c), np.float16)  # noqa: E731
    o = lambda c: np.ones((1, c), np.float16)   # noqa: E731
    ws.update(bq=z(D), bk=z(D), bv=z(D), bo=z(D), b1=z(F), b2=z(D), g1=o(D), be1=z(D), g2=o(D), be2=z(D))
    return ws


def layer_reference_arrays(x, p: dict, heads: int, eps: float = 1e-6, rounding: bool = True,
                           scale: float = 0.125) -> dict[str, np.ndarray]:
    """One pre-LN encoder layer on one sequence x [S, D]; returns every tensor the reference
    dumps (X, LN1, Q, K, KT, P0, V, O0, O6, O, H, G, OUT) as float32.
    rounding=False drops every r16 (the pure-fp32 variant). `scale` is the softmax scale; the
    reference hard-codes 0.125 (siglip_ref.py:34), the frontend emits 1/sqrt(dh)."""
    rr = r16 if rounding else (lambda a: a)
    x = f32(x)
    P = {k: f32(v) for k, v in p.items()}
    S, D = x.shape
    dh = D // heads
    ln1 = rr(layernorm(x, P["g1"], P["be1"], eps))
    q = rr(rr(ln1 @ P["wq"]) + P["bq"])
    k = rr(rr(ln1 @ P["wk"]) + P["bk"])
    v = rr(rr(ln1 @ P["wv"]) + P["bv"])
    o = np.zeros((S, D), np.float32)
    p0 = None
    for h in range(heads):
        sl = slice(h * dh, (h + 1) * dh)
        s = rr(q[:, sl] @ k[:, sl].T) * np.float32(scale)
        pr = rr(softmax_rows(s, 1.0))
        if h == 0:
            p0 = pr
        o[:, sl] = rr(pr @ v[:, sl])
    ao = rr(rr(o @ P["wo"]) + P["bo"])
    hres = rr(x + ao)
    ln2 = rr(layernorm(hres, P["g2"], P["be2"], eps))
    f1 = rr(rr(ln2 @ P["w1"]) + P["b1"])
    g = rr(gelu(f1))
    f2 = rr(rr(g @ P["w2"]) + P["b2"])
    out = rr(hres + f2)
    o6 = o[:, 6 * dh:7 * dh] if heads > 6 else o[:, :0]
    return {"X": x, "LN1": ln1, "Q": q, "K": k, "KT": k.T, "P0": p0, "V": v, "O0": o[:, :dh], "O6": o6,
            "O": o, "H": hres, "G": g, "OUT": out}


def layer_reference(S: int, D: int, F: int, H: int) -> dict[str, np.ndarray]:
    """The reference's LCG-data layer (siglip_ref.layer_reference equivalent)."""
    x, p = lcg_layer_inputs(S, D, F, 0)
    return layer_reference_arrays(x, p, H)


def encoder_reference(x, layers: list[dict], heads: int, eps: float = 1e-6, rounding: bool = True,
                      scale: float = 0.125) -> np.ndarray:
    """Stacked layers on one sequence: the output of layer L is the input of layer L+1
    (frontend/siglip.py:168). Returns the last OUT (float32)."""
    cur = f32(x)
    for p in layers:
        cur = layer_reference_arrays(cur, p, heads, eps, rounding, scale)["OUT"]
    return cur
