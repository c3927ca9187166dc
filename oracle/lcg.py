"""Restatement of the reference's LCG test-data generator (TEST INFRASTRUCTURE ONLY).

Reference algorithm (runtime/sh_test.inc.c:2-13, host twin softhier_mlir/testing/lcg.py:13-59):
    state = seed ^ 0x9E3779B9
    repeat:  state = state * 1664525 + 1013904223  (mod 2**32);  draw = state >> 8
    element = fp16_rne(float32(lo + draw % (hi - lo + 1)) * float32(scale))   (row-major)
Sample positions (sh_test.inc.c:18-25, lcg.py:73-76): two draws per sample, i = d0 % rows,
j = d1 % cols. The "<tag> r c hex" dump line format is sh_test.inc.c:23 / lcg.py:79-91.

The stream is produced here by log-step doubling (the k-step affine map is squared each
round), so a 100 M-element tensor costs a few numpy passes; the reference uses a fixed
4096-lane leapfrog. Both are exact in uint32 arithmetic, so the bytes are identical; the
golden vectors in tests/golden pin that.

`uniform_fp16` / `normal_fp16` are the input distributions BASELINE asks for. Uniform is
exactly `fill_fp16(.., -1024, 1023, 1/1024)` (reference semantics); the normal generator is an
EXTENSION defined by this repository (the reference's LCG only yields scaled integers):
Box-Muller over consecutive draw pairs, float64 math, RNE to fp16.
"""
from __future__ import annotations

import re

import numpy as np

LCG_A = 1664525
LCG_C = 1013904223
SEED_XOR = 0x9E3779B9
_MASK = 0xFFFFFFFF


def _compose(a1: int, c1: int, a2: int, c2: int) -> tuple[int, int]:
    """Affine map x -> a2 * (a1 * x + c1) + c2 (mod 2**32): apply (a1, c1) first."""
    return (a2 * a1) & _MASK, (a2 * c1 + c2) & _MASK


def lcg_states(seed: int, n: int) -> np.ndarray:
    """The n successive 32-bit LCG states after seeding (state_1 .. state_n), uint32."""
    out = np.empty(n, dtype=np.uint32)
    if n == 0:
        return out
    s0 = (int(seed) ^ SEED_XOR) & _MASK
    out[0] = (s0 * LCG_A + LCG_C) & _MASK
    filled = 1
    step_a, step_c = LCG_A, LCG_C           # map advancing a state by `filled` steps
    with np.errstate(over="ignore"):
        while filled < n:
            take = min(filled, n - filled)
            out[filled:filled + take] = out[:take] * np.uint32(step_a) + np.uint32(step_c)
            step_a, step_c = _compose(step_a, step_c, step_a, step_c)
            filled += take
    return out


def lcg_draws(seed: int, n: int) -> np.ndarray:
    """The n successive draws (state >> 8) of the device LCG, uint32 in [0, 2**24)."""
    return lcg_states(seed, n) >> np.uint32(8)


def lcg_draws_scalar(seed: int, n: int) -> np.ndarray:
    """Plain sequential loop over the recurrence; used to self-check `lcg_draws`."""
    s = (int(seed) ^ SEED_XOR) & _MASK
    out = np.empty(n, dtype=np.uint32)
    for i in range(n):
        s = (s * LCG_A + LCG_C) & _MASK
        out[i] = s >> 8
    return out


def fill_fp16(rows: int, cols: int, seed: int, lo: int, hi: int, scale: float = 1.0) -> np.ndarray:
    """sh_test_fill_fp16 (sh_test.inc.c:4-13): integers in [lo, hi] times scale, fp16 RNE, row-major."""
    span = int(hi) - int(lo) + 1
    ints = (lcg_draws(seed, rows * cols) % np.uint32(span)).astype(np.int64) + int(lo)
    return (ints.astype(np.float32) * np.float32(scale)).astype(np.float16).reshape(rows, cols)


def const_fp16(rows: int, cols: int, bits: int) -> np.ndarray:
    """sh_test_fill_const_fp16 (sh_test.inc.c:74-76): every element is the fp16 code `bits`."""
    return np.full((rows, cols), int(bits) & 0xFFFF, dtype=np.uint16).view(np.float16)


def colparity_fp16(rows: int, cols: int, even_bits: int, odd_bits: int) -> np.ndarray:
    """sh_test_fill_colparity_fp16 (sh_test.inc.c:77-79): even / odd columns get two fp16 codes."""
    codes = np.empty(cols, dtype=np.uint16)
    codes[0::2] = int(even_bits) & 0xFFFF
    codes[1::2] = int(odd_bits) & 0xFFFF
    return np.tile(codes, (rows, 1)).view(np.float16)


def sample_positions(rows: int, cols: int, seed: int, nsamples: int) -> list[tuple[int, int]]:
    """(i, j) sequence of sh_test_dump_samples (sh_test.inc.c:18-25): draws alternate row / column."""
    d = lcg_draws(seed, 2 * nsamples).astype(np.int64)
    return list(zip((d[0::2] % rows).tolist(), (d[1::2] % cols).tolist()))


_LINE = re.compile(r"^(\S+) (\d+) (\d+) ([0-9a-fA-F]{4})$")


def parse_samples(text: str) -> dict[str, list[tuple[int, int, float]]]:
    """Collect "<tag> r c hex" lines (sh_test.inc.c:23) into {tag: [(r, c, value)]}."""
    out: dict[str, list[tuple[int, int, float]]] = {}
    for line in text.splitlines():
        m = _LINE.match(line.strip())
        if m:
            code = np.array([int(m.group(4), 16)], dtype=np.uint16).view(np.float16)[0]
            out.setdefault(m.group(1), []).append((int(m.group(2)), int(m.group(3)), float(code)))
    return out


def compare_samples(samples, ref: np.ndarray, atol: float, rtol: float) -> tuple[int, float]:
    """(mismatches, max abs error) of sampled values against a reference array, with the
    reference's acceptance rule |got - want| <= atol + rtol * |want| (lcg.py:93-106)."""
    bad, worst = 0, 0.0
    for r, c, got in samples:
        want = float(ref[r, c])
        err = abs(got - want)
        worst = max(worst, err)
        if err > atol + rtol * abs(want):
            bad += 1
    return bad, worst


# ---- BASELINE input distributions -------------------------------------------------------

def uniform_fp16(rows: int, cols: int, seed: int) -> np.ndarray:
    """uniform [-1, 1) as k/1024 (exact reference semantics: fill_fp16(.., -1024, 1023, 1/1024))."""
    return fill_fp16(rows, cols, seed, -1024, 1023, 1.0 / 1024)


def normal_fp16(rows: int, cols: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """N(mean, std) fp16 from the LCG stream (extension of this repository): draw pairs (d0, d1)
    give u = (d + 0.5) / 2**24 in (0, 1); z = sqrt(-2 ln u0) cos(2 pi u1) (float64), then
    mean + std * z rounded RNE to fp16. One pair per element."""
    n = rows * cols
    d = lcg_draws(seed, 2 * n).astype(np.float64)
    u0 = (d[0::2] + 0.5) / float(1 << 24)
    u1 = (d[1::2] + 0.5) / float(1 << 24)
    z = np.sqrt(-2.0 * np.log(u0)) * np.cos(2.0 * np.pi * u1)
    return (mean + std * z).astype(np.float16).reshape(rows, cols)
