"""numpy references of the hot-path operators (TEST INFRASTRUCTURE ONLY).

Each function restates the formula the reference checks its device results against:
  - row ops: tests/gvsoc/run.py:152-158 (layernorm with population variance, softmax(scale x)
    with the row max subtracted, tanh-GELU, add, add_bias, scale, transpose);
  - GEMM: fp32 `x @ w (+ z)` (tests/gvsoc/run.py:118; on-device sampled check sh_test.inc.c:32-51);
  - attention: per head, s = r16(q k^T) * scale, p = r16(softmax(s)), o = r16(p v)
    (tests/gvsoc/run.py:921-934; siglip_ref.py:31-37).
All math is float32 on float32 copies of fp16 inputs; `r16` is the fp16 store rounding the
reference applies after every op that writes HBM (siglip_ref.py:24-25).
"""
from __future__ import annotations

import numpy as np

GELU_C = np.float32(0.7978845608)     # sqrt(2/pi) as written in run.py:155 / siglip_ref.py:42
GELU_K = np.float32(0.044715)


def f32(a) -> np.ndarray:
    return np.asarray(a).astype(np.float32)


def r16(a) -> np.ndarray:
    """Round to fp16 and back (the device stores every intermediate as fp16)."""
    return np.asarray(a).astype(np.float16).astype(np.float32)


def layernorm(x, gamma, beta, eps: float) -> np.ndarray:
    x = f32(x)
    mean = x.mean(1, keepdims=True)
    var = x.var(1, keepdims=True)
    return (x - mean) / np.sqrt(var + np.float32(eps)) * f32(gamma).reshape(1, -1) + f32(beta).reshape(1, -1)


def softmax_rows(x, scale: float) -> np.ndarray:
    t = f32(x) * np.float32(scale)
    e = np.exp(t - t.max(1, keepdims=True))
    return e / e.sum(1, keepdims=True)


def gelu(x) -> np.ndarray:
    x = f32(x)
    return np.float32(0.5) * x * (np.float32(1) + np.tanh(GELU_C * (x + GELU_K * x ** 3)))


def add(a, b) -> np.ndarray:
    return f32(a) + f32(b)


def add_bias(x, bias) -> np.ndarray:
    return f32(x) + f32(bias).reshape(1, -1)


def scale(x, s: float) -> np.ndarray:
    return f32(x) * np.float32(s)


def transpose(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x).T)


def gemm(x, w, z=None) -> np.ndarray:
    out = f32(x) @ f32(w)
    return out if z is None else out + f32(z)


def attention(q, k, v, heads: int, scale: float, rounding: bool = True) -> np.ndarray:
    """Multi-head non-causal attention over column slices; q, k, v are [S, H*dh].
    rounding=True keeps the reference's fp16 rounding points, False is the pure-fp32 variant."""
    rr = r16 if rounding else (lambda a: a)
    q, k, v = f32(q), f32(k), f32(v)
    S, D = q.shape
    dh = D // heads
    o = np.zeros((S, D), np.float32)
    for h in range(heads):
        sl = slice(h * dh, (h + 1) * dh)
        s = rr(q[:, sl] @ k[:, sl].T) * np.float32(scale)
        p = np.exp(s - s.max(1, keepdims=True))
        p = rr(p / p.sum(1, keepdims=True))
        o[:, sl] = rr(p @ v[:, sl])
    return o


def max_abs_and_rel_l2(got, want) -> tuple[float, float]:
    """The two error figures BASELINE's tolerance is stated in: max |got - want| and
    ||got - want||_2 / ||want||_2 (float64)."""
    g = np.asarray(got, dtype=np.float64)
    w = np.asarray(want, dtype=np.float64)
    d = g - w
    denom = np.linalg.norm(w)
    return float(np.abs(d).max(initial=0.0)), float(np.linalg.norm(d) / denom) if denom else float(np.linalg.norm(d))
