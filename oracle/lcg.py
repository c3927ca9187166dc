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
Box-Muller over consecutive draw pairs with ln / cos as fixed series of correctly rounded
float32 operations, RNE to fp16 - a definition every implementation reproduces bit for bit.
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


def _jump(n: int) -> tuple[int, int]:
    """The affine map (a, c) that advances a state by n steps (square-and-multiply)."""
    acc, p = (1, 0), (LCG_A, LCG_C)
    while n:
        if n & 1:
            acc = _compose(acc[0], acc[1], p[0], p[1])
        p = _compose(p[0], p[1], p[0], p[1])
        n >>= 1
    return acc


def lcg_states(seed: int, n: int, skip: int = 0) -> np.ndarray:
    """The n successive 32-bit LCG states after seeding (state_1 .. state_n), uint32; with `skip`, the states
    state_{skip+1} .. state_{skip+n} (the stream jumped ahead by `skip` draws)."""
    out = np.empty(n, dtype=np.uint32)
    if n == 0:
        return out
    s0 = (int(seed) ^ SEED_XOR) & _MASK
    if skip:
        a, c = _jump(int(skip))
        s0 = (a * s0 + c) & _MASK
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


def lcg_draws(seed: int, n: int, skip: int = 0) -> np.ndarray:
    """The n successive draws (state >> 8) of the device LCG, uint32 in [0, 2**24), after `skip` draws."""
    return lcg_states(seed, n, skip) >> np.uint32(8)


def lcg_draws_scalar(seed: int, n: int) -> np.ndarray:
    """Plain sequential loop over the recurrence; used to self-check `lcg_draws`."""
    s = (int(seed) ^ SEED_XOR) & _MASK
    out = np.empty(n, dtype=np.uint32)
    for i in range(n):
        s = (s * LCG_A + LCG_C) & _MASK
        out[i] = s >> 8
    return out


def fill_fp16(rows: int, cols: int, seed: int, lo: int, hi: int, scale: float = 1.0, row0: int = 0) -> np.ndarray:
    """sh_test_fill_fp16 (sh_test.inc.c:4-13): integers in [lo, hi] times scale, fp16 RNE, row-major. With `row0`,
    rows row0 .. row0 + rows - 1 of that matrix."""
    span = int(hi) - int(lo) + 1
    ints = (lcg_draws(seed, rows * cols, row0 * cols) % np.uint32(span)).astype(np.int64) + int(lo)
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

def uniform_fp16(rows: int, cols: int, seed: int, row0: int = 0) -> np.ndarray:
    """uniform [-1, 1) as k/1024 (exact reference semantics: fill_fp16(.., -1024, 1023, 1/1024))."""
    return fill_fp16(rows, cols, seed, -1024, 1023, 1.0 / 1024, row0)


_h = lambda x: np.float32(float.fromhex(x))  # noqa: E731  (exact fp32 constants)
_SQRT2, _LN2 = _h("0x1.6a09e6p+0"), _h("0x1.62e43p-1")
_ATANH = [_h(x) for x in ("0x1.3b13b2p-4", "0x1.745d18p-4", "0x1.c71c72p-4", "0x1.24924ap-3", "0x1.99999ap-3",
                          "0x1.555556p-2")]                      # 1/13, 1/11, ..., 1/3
_COS = [_h(x) for x in ("-0x1.a6d1f2p-16", "0x1.e1f506p-11", "-0x1.55d3c8p-6", "0x1.03c1f0p-2", "-0x1.3bd3ccp+0")]
_SIN = [_h(x) for x in ("-0x1.e3075p-19", "0x1.507834p-13", "-0x1.32d2ccp-8", "0x1.466bc6p-4", "-0x1.4abbcep-1",
                        "0x1.921fb6p+0")]
_ONE, _TWO, _HALF = np.float32(1.0), np.float32(2.0), np.float32(0.5)


def ln_exact(u: np.ndarray) -> np.ndarray:
    """ln u (float32, u in (0, 1], normal) as the fixed sequence of correctly rounded fp32 operations of the
    library's generator: u = m 2^e with m in [sqrt(1/2), sqrt(2)), ln u = e ln2 + 2 atanh(t), t = (m-1)/(m+1),
    atanh(t) = t + t^3/3 + ... + t^13/13 in Horner form."""
    b = u.astype(np.float32).view(np.uint32)
    e = (b >> np.uint32(23)).astype(np.int32) - 127
    m = ((b & np.uint32(0x7FFFFF)) | np.uint32(0x3F800000)).view(np.float32)
    big = m > _SQRT2
    m = np.where(big, m * _HALF, m)
    e = e + big.astype(np.int32)
    t = (m - _ONE) / (m + _ONE)
    t2 = t * t
    p = np.full_like(t, _ATANH[0])
    for c in _ATANH[1:]:
        p = c + t2 * p
    lnm = (t + t * (t2 * p)) * _TWO
    return e.astype(np.float32) * _LN2 + lnm


def cos2pi_exact(u: np.ndarray) -> np.ndarray:
    """cos(2 pi u) (float32, u in [0, 1]): 4u = q + r, q = rint(4u), |r| <= 1/2; the quadrant q mod 4 selects
    +-cos / +-sin of (pi/2) r, each a Taylor polynomial in r (to r^10 / r^11) of correctly rounded fp32 steps."""
    x = u.astype(np.float32) * np.float32(4.0)
    q = np.rint(x)
    r = x - q
    r2 = r * r
    c = np.full_like(r, _COS[0])
    for k in _COS[1:]:
        c = k + r2 * c
    c = _ONE + r2 * c
    sn = np.full_like(r, _SIN[0])
    for k in _SIN[1:]:
        sn = k + r2 * sn
    sn = r * sn
    qi = q.astype(np.int32) & 3
    return np.select([qi == 0, qi == 1, qi == 2], [c, -sn, -c], sn).astype(np.float32)


def normal_fp16(rows: int, cols: int, seed: int, mean: float = 0.0, std: float = 1.0, row0: int = 0) -> np.ndarray:
    """N(mean, std) fp16 from the LCG stream (an extension of this repository; the reference's LCG only yields
    scaled integers). One draw pair (d0, d1) per element, row-major: u = (float32(d) + 0.5) * 2^-24,
    z = sqrt(-2 ln u0) * cos(2 pi u1) with ln_exact / cos2pi_exact, value = fp16_rne(mean + std * z), every step
    one correctly rounded float32 operation. The library's generators (sh_cuda_fill_normal_fp16 on the device,
    sh_cuda_host_fill_normal_fp16 on the host) perform the same operations, so the bits agree. With `row0`, rows
    row0 .. row0 + rows - 1 of that matrix (the stream jumped ahead by 2 * row0 * cols draws)."""
    n = rows * cols
    d = lcg_draws(seed, 2 * n, 2 * row0 * cols)
    k = np.float32(2.0 ** -24)
    u0 = (d[0::2].astype(np.float32) + _HALF) * k
    u1 = (d[1::2].astype(np.float32) + _HALF) * k
    z = np.sqrt(np.float32(-2.0) * ln_exact(u0)) * cos2pi_exact(u1)
    v = np.float32(mean) + np.float32(std) * z
    return v.astype(np.float16).reshape(rows, cols)
