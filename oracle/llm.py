"""CPU restatement of the reference's Llama-style decoder ops (test infrastructure only: the checker, never the
product path).

Semantics follow runtime/sh_ops.h:277-304 (the header contract of runtime/sh_llm.inc.c) and the numpy twins the
reference checks its device programs against (frontend/smolvla_expert.py:151-197, frontend/smolvla.py:473-503);
tests/golden/llm.npz holds outputs of those twins, and tests/test_oracle.py pins this file to them.
"""
from __future__ import annotations

import numpy as np

PAD = 0xFFFF          # SH_LLM_PAD (sh_ops.h:283): token class of a padding position


def r16(a) -> np.ndarray:
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def rmsnorm(x, g, eps: float = 1e-5, rounding: bool = True) -> np.ndarray:
    """y = x / sqrt(mean(x^2) + eps) * gamma per row (sh_ops.h:284; smolvla_expert.py:156-158)."""
    x = np.asarray(x, np.float32)
    y = x * (1.0 / np.sqrt((x * x).mean(1, keepdims=True) + eps)) * np.asarray(g, np.float32)
    return r16(y) if rounding else y


def rope(x, table, dh: int, rounding: bool = True) -> np.ndarray:
    """Rotate-half RoPE on every dh-column head of each row; table row = cos[dh/2] | sin[dh/2] of that row's
    position (sh_ops.h:285-288; smolvla_expert.py:161-169)."""
    x, t = np.asarray(x, np.float32), np.asarray(table, np.float32)
    half = dh // 2
    c, s = t[:, :half], t[:, half:dh]
    y = np.empty_like(x)
    for h0 in range(0, x.shape[1], dh):
        a, b = x[:, h0:h0 + half], x[:, h0 + half:h0 + dh]
        y[:, h0:h0 + half] = a * c - b * s
        y[:, h0 + half:h0 + dh] = b * c + a * s
    return r16(y) if rounding else y


def silu_mul(a, b, rounding: bool = True) -> np.ndarray:
    """y = silu(a) * b = a b / (1 + e^-a) (sh_ops.h:289; the gate of smolvla_expert.py np_layer)."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    y = a / (1 + np.exp(-a)) * b
    return r16(y) if rounding else y


def mask_allowed(tok_q, tok_k) -> np.ndarray:
    """Query i may attend key j iff tok_k[j] <= tok_q[i] as unsigned 16-bit classes (sh_ops.h:278-282), so PAD
    keys are never attended by a non-PAD query."""
    tq = np.asarray(tok_q, np.uint16).astype(np.uint32)
    tk = np.asarray(tok_k, np.uint16).astype(np.uint32)
    return tk[None, :] <= tq[:, None]


def softmax_masked(x, scale: float, tok_q, tok_k, rounding: bool = True) -> np.ndarray:
    """softmax(scale x + mask) per row; a PAD query row gets uniform probabilities (sh_ops.h:290-292)."""
    x = np.asarray(x, np.float32) * np.float32(scale)
    allowed = mask_allowed(tok_q, tok_k)
    s = np.where(allowed, x, -np.inf)
    pad_q = np.asarray(tok_q, np.uint16) == PAD
    s[pad_q, :] = 0.0
    e = np.exp(s - s.max(1, keepdims=True))
    y = e / e.sum(1, keepdims=True)
    return r16(y) if rounding else y


def attention_gqa(q, k, v, heads: int, kv_heads: int, scale: float, tok=None, rounding: bool = True) -> np.ndarray:
    """Grouped-query self-attention: query head h uses key/value head h // (heads / kv_heads); optional token
    mask (tok: one class per position, the same array for queries and keys); PAD query rows average every value
    row (sh_ops.h:293-300). With rounding, fp16 rounding where the device stores fp16 (scores, exponentials, the
    unnormalised P V), as in smolvla_expert.py:172-190."""
    q, k, v = (np.asarray(t, np.float32) for t in (q, k, v))
    S = q.shape[0]
    dh = q.shape[1] // heads
    grp = heads // kv_heads
    rr = r16 if rounding else (lambda a: np.asarray(a, np.float32))
    allowed = np.ones((S, S), bool) if tok is None else mask_allowed(tok, tok)
    pad_q = np.zeros(S, bool) if tok is None else (np.asarray(tok, np.uint16) == PAD)
    o = np.zeros((S, heads * dh), np.float32)
    for h in range(heads):
        kv = h // grp
        s = rr(q[:, h * dh:(h + 1) * dh] @ k[:, kv * dh:(kv + 1) * dh].T) * scale
        s = np.where(allowed, s, -np.inf)
        s[pad_q, :] = 0.0
        e = rr(np.exp(s - s.max(1, keepdims=True)))
        o[:, h * dh:(h + 1) * dh] = rr(rr(e @ v[:, kv * dh:(kv + 1) * dh]) / e.sum(1, keepdims=True))
    return o


def pixel_shuffle(x, grid: int, s: int) -> np.ndarray:
    """Output token (gr, gb) of the (grid/s)^2 grid = the s x s block of patch tokens rows gr*s.., cols gb*s..,
    row-major, each D wide (sh_ops.h:301-303; smolvla.py:481-486). Data movement only."""
    x = np.asarray(x)
    D = x.shape[1]
    g = grid // s
    out = np.empty((g * g, s * s * D), x.dtype)
    for gr in range(g):
        for gb in range(g):
            for i in range(s):
                for j in range(s):
                    out[gr * g + gb, (i * s + j) * D:(i * s + j + 1) * D] = x[(gr * s + i) * grid + gb * s + j]
    return out
