"""Batched SigLIP / ViT pre-LN encoder on the library's C ABI (the workload of frontend/siglip.py:133-168, run over
a batch of B sequences of S tokens at once).

Per layer, 7 launches on device-resident activations [B*S, D] (row-major fp16):
    ln1 = LN(x)                                   sh_layernorm
    qkv = ln1 . [wq|wk|wv] + [bq|bk|bv]           sh_cuda_gemm, bias epilogue (one N = 3D GEMM; q/k/v are the
                                                  column slices the attention reads with ld = 3D, the packed
                                                  layout of tests/filecheck/attention_translate.mlir)
    o   = attention(q, k, v) per sequence, head   sh_cuda_attention_batched
    h   = x + o . wo + bo                         sh_cuda_gemm, bias + residual epilogue
    ln2 = LN(h)                                   sh_layernorm
    g   = gelu(ln2 . w1 + b1)                     sh_cuda_gemm, bias + GELU epilogue
    out = h + g . w2 + b2                         sh_cuda_gemm, bias + residual epilogue
This is the reference layer (siglip_ref.py:20-45) with the frontend's add_bias / gelu / add ops folded into the
GEMM epilogues, so each intermediate is rounded to fp16 once instead of after every op.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import numpy as np

from . import lib as L
from .runtime import Runtime


@dataclass
class LayerWeights:
    wqkv: int
    bqkv: int
    wo: int
    bo: int
    w1: int
    b1: int
    w2: int
    b2: int
    g1: int
    be1: int
    g2: int
    be2: int


@dataclass
class Activations:
    B: int
    S: int
    D: int
    F: int
    x: int
    ln1: int
    qkv: int
    o: int
    h: int
    ln2: int
    g: int
    out: int
    extra: dict = field(default_factory=dict)


def upload_layer(rt: Runtime, p: dict) -> LayerWeights:
    """Parameters in the reference's layout (weights [in, out], 1 x cols rows) -> device; q/k/v weights and biases
    are concatenated along the output columns."""
    f16 = lambda a: np.asarray(a, dtype=np.float16)  # noqa: E731
    wqkv = np.concatenate([f16(p["wq"]), f16(p["wk"]), f16(p["wv"])], axis=1)
    bqkv = np.concatenate([f16(p["bq"]), f16(p["bk"]), f16(p["bv"])], axis=1)
    up = rt.upload
    return LayerWeights(wqkv=up(wqkv), bqkv=up(bqkv), wo=up(p["wo"]), bo=up(p["bo"]), w1=up(p["w1"]), b1=up(p["b1"]),
                        w2=up(p["w2"]), b2=up(p["b2"]), g1=up(p["g1"]), be1=up(p["be1"]), g2=up(p["g2"]),
                        be2=up(p["be2"]))


# ---- the benchmark's synthetic encoder --------------------------------------------------------------
WEIGHT_SEED0, WEIGHT_SEED_STRIDE, INPUT_SEED0 = 7000, 16, 100


def synthetic_weight_seeds(layer: int) -> dict[str, int]:
    """LCG seeds of layer `layer`'s N(0, 0.02) matrices ([wq|wk|wv] is one 768 x 2304 matrix, filled row-major)."""
    s = WEIGHT_SEED0 + WEIGHT_SEED_STRIDE * layer
    return {"wqkv": s, "wo": s + 1, "w1": s + 2, "w2": s + 3}


def synthetic_encoder(rt: Runtime, B: int, S: int, D: int, F: int, nlayers: int,
                      input_seed: int) -> tuple[list[LayerWeights], Activations, int]:
    """Device weights, activations and input of the synthetic encoder, generated on the GPU with the library's
    N(mean, std) fill (sh_cuda_fill_normal_fp16, bit-identical to its host definition): per layer N(0, 0.02)
    matrices with the seeds of synthetic_weight_seeds, zero biases, gamma 1, beta 0; the input x [B*S, D] is
    N(0, 1) from `input_seed`. Returns (layers, activations, x address)."""
    lib = rt.lib
    layers = []
    for li in range(nlayers):
        a = rt.alloc
        w = LayerWeights(wqkv=a(D, 3 * D), bqkv=a(1, 3 * D), wo=a(D, D), bo=a(1, D), w1=a(D, F), b1=a(1, F),
                         w2=a(F, D), b2=a(1, D), g1=a(1, D), be1=a(1, D), g2=a(1, D), be2=a(1, D))
        sd = synthetic_weight_seeds(li)
        lib.sh_cuda_fill_normal_fp16(w.wqkv, D, 3 * D, 3 * D, sd["wqkv"], 0.0, 0.02)
        lib.sh_cuda_fill_normal_fp16(w.wo, D, D, D, sd["wo"], 0.0, 0.02)
        lib.sh_cuda_fill_normal_fp16(w.w1, D, F, F, sd["w1"], 0.0, 0.02)
        lib.sh_cuda_fill_normal_fp16(w.w2, F, D, D, sd["w2"], 0.0, 0.02)
        for b, n in ((w.bqkv, 3 * D), (w.bo, D), (w.b1, F), (w.b2, D), (w.be1, D), (w.be2, D)):
            lib.sh_test_fill_const_fp16(b, 1, n, n, 0x0000)
        for g in (w.g1, w.g2):
            lib.sh_test_fill_const_fp16(g, 1, D, D, 0x3C00)
        layers.append(w)
    act = alloc_activations(rt, B, S, D, F)
    x_in = rt.alloc(B * S, D)
    lib.sh_cuda_fill_normal_fp16(x_in, B * S, D, D, input_seed, 0.0, 1.0)
    return layers, act, x_in


def alloc_activations(rt: Runtime, B: int, S: int, D: int, F: int) -> Activations:
    M = B * S
    a = rt.alloc
    return Activations(B=B, S=S, D=D, F=F, x=a(M, D), ln1=a(M, D), qkv=a(M, 3 * D), o=a(M, D), h=a(M, D),
                       ln2=a(M, D), g=a(M, F), out=a(M, D))


def layer_ops(lib, act: Activations, w: LayerWeights, heads: int, eps: float, scale: float, x: int,
              out: int) -> list[tuple[str, Callable[[], int]]]:
    """The 7 library calls of one layer as (kind, enqueue) pairs; enqueue() returns the call's return code."""
    B, S, D, F = act.B, act.S, act.D, act.F
    M = B * S
    A = L.SH_ALL

    def ln1():
        lib.sh_layernorm(act.ln1, x, w.g1, w.be1, M, D, D, eps, A)
        return 0

    def ln2():
        lib.sh_layernorm(act.ln2, act.h, w.g2, w.be2, M, D, D, eps, A)
        return 0

    return [
        ("layernorm", ln1),
        ("gemm_qkv", lambda: lib.sh_cuda_gemm(act.ln1, w.wqkv, act.qkv, M, 3 * D, D, D, 3 * D, 3 * D, w.bqkv, 0, 0,
                                              L.EPI_BIAS, 0)),
        ("attention", lambda: lib.sh_cuda_attention_batched(act.qkv, act.qkv + 2 * D, act.qkv + 4 * D, act.o, S, D,
                                                            heads, 3 * D, 3 * D, 3 * D, D, scale, B)),
        ("gemm_o", lambda: lib.sh_cuda_gemm(act.o, w.wo, act.h, M, D, D, D, D, D, w.bo, x, D,
                                            L.EPI_BIAS | L.EPI_RESIDUAL, 0)),
        ("layernorm", ln2),
        ("gemm_fc1", lambda: lib.sh_cuda_gemm(act.ln2, w.w1, act.g, M, F, D, D, F, F, w.b1, 0, 0,
                                              L.EPI_BIAS | L.EPI_GELU, 0)),
        ("gemm_fc2", lambda: lib.sh_cuda_gemm(act.g, w.w2, out, M, D, F, F, D, D, w.b2, act.h, D,
                                              L.EPI_BIAS | L.EPI_RESIDUAL, 0)),
    ]


# ---- LayerNorm folded into the GEMMs ----------------------------------------------------------------------------------
@dataclass
class FoldedWeights:
    """A layer with LN1 folded into the QKV GEMM and LN2 into FC1 (sh_cuda_gemm_ln): w' = diag(gamma) w,
    colsum = 1^T w' (fp32), bias' = beta w + bias (fp16)."""
    wqkv: int
    cqkv: int
    dqkv: int
    wo: int
    bo: int
    w1: int
    c1: int
    d1: int
    w2: int
    b2: int


def fold_layer_norms(rt: Runtime, w: LayerWeights, D: int, F: int) -> FoldedWeights:
    """Device-side weight transform (setup, not per step): both folds are GEMMs / row scalings on the library."""
    lib, a = rt.lib, rt.alloc
    ones = a(1, D)
    lib.sh_test_fill_const_fp16(ones, 1, D, D, 0x3C00)
    out = {}
    for tag, wt, bias, g, be, n in (("qkv", w.wqkv, w.bqkv, w.g1, w.be1, 3 * D), ("1", w.w1, w.b1, w.g2, w.be2, F)):
        wp, c, d = a(D, n), rt.alloc_bytes(4 * n), a(1, n)
        rc = lib.sh_cuda_scale_rows(wp, wt, D, n, n, n, g)
        rc = rc or lib.sh_cuda_gemm(ones, wp, c, 1, n, D, D, n, n, 0, 0, 0, L.EPI_F32_OUT, 1)
        rc = rc or lib.sh_cuda_gemm(be, wt, d, 1, n, D, D, n, n, bias, 0, 0, L.EPI_BIAS, 1)
        if rc:
            raise RuntimeError(f"folding LayerNorm into the {tag} GEMM failed: {rc}")
        out[tag] = (wp, c, d)
    return FoldedWeights(wqkv=out["qkv"][0], cqkv=out["qkv"][1], dqkv=out["qkv"][2], wo=w.wo, bo=w.bo,
                         w1=out["1"][0], c1=out["1"][1], d1=out["1"][2], w2=w.w2, b2=w.b2)


@dataclass
class Ln1FoldedWeights:
    """A layer with only LN1 folded into the QKV GEMM (sh_cuda_gemm_ln); LN2 stays a separate kernel."""
    wqkv: int
    cqkv: int
    dqkv: int
    wo: int
    bo: int
    w1: int
    b1: int
    w2: int
    b2: int
    g2: int
    be2: int


def fold_layer_norm1(rt: Runtime, w: LayerWeights, D: int) -> Ln1FoldedWeights:
    """The LN1 half of fold_layer_norms: w' = diag(g1) wqkv, colsum = 1^T w' (fp32), bias' = be1 wqkv + bqkv."""
    lib, a = rt.lib, rt.alloc
    ones = a(1, D)
    lib.sh_test_fill_const_fp16(ones, 1, D, D, 0x3C00)
    n = 3 * D
    wp, c, d = a(D, n), rt.alloc_bytes(4 * n), a(1, n)
    rc = lib.sh_cuda_scale_rows(wp, w.wqkv, D, n, n, n, w.g1)
    rc = rc or lib.sh_cuda_gemm(ones, wp, c, 1, n, D, D, n, n, 0, 0, 0, L.EPI_F32_OUT, 1)
    rc = rc or lib.sh_cuda_gemm(w.be1, w.wqkv, d, 1, n, D, D, n, n, w.bqkv, 0, 0, L.EPI_BIAS, 1)
    if rc:
        raise RuntimeError(f"folding LayerNorm 1 into the QKV GEMM failed: {rc}")
    return Ln1FoldedWeights(wqkv=wp, cqkv=c, dqkv=d, wo=w.wo, bo=w.bo, w1=w.w1, b1=w.b1, w2=w.w2, b2=w.b2, g2=w.g2,
                            be2=w.be2)


def layer_ops_ln1_folded(lib, act: Activations, w: Ln1FoldedWeights, stats_x: int, heads: int, eps: float,
                         scale: float, x: int, out: int) -> list[tuple[str, Callable[[], int]]]:
    """The 6 launches of one layer with LN1 folded into the QKV GEMM: x's row statistics are in stats_x (written by
    the previous layer's FC2 epilogue, or sh_cuda_row_stats for the first layer), and this layer's FC2 writes those of
    its output there for the next layer. The O projection and FC1 keep their plain epilogues (their epilogues have
    no slack for the LayerNorm arithmetic)."""
    B, S, D, F = act.B, act.S, act.D, act.F
    M = B * S
    A = L.SH_ALL
    g = lib.sh_cuda_gemm_ln

    def ln2():
        lib.sh_layernorm(act.ln2, act.h, w.g2, w.be2, M, D, D, eps, A)
        return 0

    return [
        ("gemm_qkv", lambda: g(x, w.wqkv, act.qkv, M, 3 * D, D, D, 3 * D, 3 * D, w.dqkv, 0, 0,
                               L.EPI_BIAS | L.EPI_LN_IN, stats_x, w.cqkv, eps, 0)),
        ("attention", lambda: lib.sh_cuda_attention_batched(act.qkv, act.qkv + 2 * D, act.qkv + 4 * D, act.o, S, D,
                                                            heads, 3 * D, 3 * D, 3 * D, D, scale, B)),
        ("gemm_o", lambda: lib.sh_cuda_gemm(act.o, w.wo, act.h, M, D, D, D, D, D, w.bo, x, D,
                                            L.EPI_BIAS | L.EPI_RESIDUAL, 0)),
        ("layernorm", ln2),
        ("gemm_fc1", lambda: lib.sh_cuda_gemm(act.ln2, w.w1, act.g, M, F, D, D, F, F, w.b1, 0, 0,
                                              L.EPI_BIAS | L.EPI_GELU, 0)),
        ("gemm_fc2", lambda: g(act.g, w.w2, out, M, D, F, F, D, D, w.b2, act.h, D,
                               L.EPI_BIAS | L.EPI_RESIDUAL | L.EPI_STATS_OUT, 0, 0, eps, stats_x)),
    ]


def encoder_schedule_ln1_folded(lib, act: Activations, layers: list[Ln1FoldedWeights], stats_x: int, heads: int,
                                eps: float, scale: float, x_in: int | None = None,
                                x_out: int | None = None) -> tuple[list[tuple[str, Callable[[], int]]], int]:
    """encoder_schedule with LN1 folded: one sh_cuda_row_stats of the input, then 6 launches per layer."""
    M, D = act.B * act.S, act.D
    cur = act.x if x_in is None else x_in
    nxt = act.out
    sched = [("row_stats", lambda x0=cur: lib.sh_cuda_row_stats(x0, M, D, D, stats_x))]
    for i, w in enumerate(layers):
        dst = x_out if (x_out is not None and i == len(layers) - 1) else nxt
        sched += layer_ops_ln1_folded(lib, act, w, stats_x, heads, eps, scale, cur, dst)
        cur, nxt = dst, (act.x if nxt == act.out else act.out)
    return sched, cur


def alloc_row_stats(rt: Runtime, M: int, D: int) -> tuple[int, int]:
    """(stats of the residual stream x, stats of h): D / 64 fp32 (sum, sum of squares) pairs per row each."""
    return rt.alloc_bytes(M * (D // 64) * 8), rt.alloc_bytes(M * (D // 64) * 8)


def layer_ops_folded(lib, act: Activations, w: FoldedWeights, stats: tuple[int, int], heads: int, eps: float,
                     scale: float, x: int, out: int) -> list[tuple[str, Callable[[], int]]]:
    """The 5 launches of one layer with both LayerNorms folded: x's row statistics are in stats[0] (written by the
    previous layer's FC2, or sh_cuda_row_stats for the first), the O projection writes h's into stats[1]."""
    B, S, D, F = act.B, act.S, act.D, act.F
    M = B * S
    sx, sh = stats
    g = lib.sh_cuda_gemm_ln
    return [
        ("gemm_qkv", lambda: g(x, w.wqkv, act.qkv, M, 3 * D, D, D, 3 * D, 3 * D, w.dqkv, 0, 0,
                               L.EPI_BIAS | L.EPI_LN_IN, sx, w.cqkv, eps, 0)),
        ("attention", lambda: lib.sh_cuda_attention_batched(act.qkv, act.qkv + 2 * D, act.qkv + 4 * D, act.o, S, D,
                                                            heads, 3 * D, 3 * D, 3 * D, D, scale, B)),
        ("gemm_o", lambda: g(act.o, w.wo, act.h, M, D, D, D, D, D, w.bo, x, D,
                             L.EPI_BIAS | L.EPI_RESIDUAL | L.EPI_STATS_OUT, 0, 0, eps, sh)),
        ("gemm_fc1", lambda: g(act.h, w.w1, act.g, M, F, D, D, F, F, w.d1, 0, 0,
                               L.EPI_BIAS | L.EPI_GELU | L.EPI_LN_IN, sh, w.c1, eps, 0)),
        ("gemm_fc2", lambda: g(act.g, w.w2, out, M, D, F, F, D, D, w.b2, act.h, D,
                               L.EPI_BIAS | L.EPI_RESIDUAL | L.EPI_STATS_OUT, 0, 0, eps, sx)),
    ]


def encoder_schedule_folded(lib, act: Activations, layers: list[FoldedWeights], stats: tuple[int, int], heads: int,
                            eps: float, scale: float, x_in: int | None = None,
                            x_out: int | None = None) -> tuple[list[tuple[str, Callable[[], int]]], int]:
    """encoder_schedule with the LayerNorms folded: one sh_cuda_row_stats of the input, then 5 launches per layer."""
    M, D = act.B * act.S, act.D
    cur = act.x if x_in is None else x_in
    nxt = act.out
    sched = [("row_stats", lambda x0=cur: lib.sh_cuda_row_stats(x0, M, D, D, stats[0]))]
    for i, w in enumerate(layers):
        dst = x_out if (x_out is not None and i == len(layers) - 1) else nxt
        sched += layer_ops_folded(lib, act, w, stats, heads, eps, scale, cur, dst)
        cur, nxt = dst, (act.x if nxt == act.out else act.out)
    return sched, cur


def op_work(kind: str, B: int, S: int, D: int, F: int, heads: int) -> tuple[float, float]:
    """(algorithmic FLOPs, algorithmic HBM bytes) of one launch of `kind` (fp16 = 2 B per element)."""
    M = B * S
    if kind == "layernorm":
        return 8.0 * M * D, 2.0 * (2 * M * D + 2 * D)
    if kind == "gemm_qkv":
        return 2.0 * M * D * 3 * D, 2.0 * (M * D + D * 3 * D + M * 3 * D + 3 * D)
    if kind == "gemm_o":
        return 2.0 * M * D * D, 2.0 * (M * D + D * D + 2 * M * D + D)
    if kind == "gemm_fc1":
        return 2.0 * M * D * F, 2.0 * (M * D + D * F + M * F + F)
    if kind == "gemm_fc2":
        return 2.0 * M * F * D, 2.0 * (M * F + F * D + 2 * M * D + D)
    if kind == "attention":
        return 4.0 * B * S * S * D, 2.0 * 4 * M * D
    if kind == "row_stats":
        return 3.0 * M * D, 2.0 * M * D + 8.0 * M * (D // 64)
    raise KeyError(kind)


def layer_forward(lib, act: Activations, w: LayerWeights, heads: int, eps: float, scale: float,
                  x: int | None = None, out: int | None = None) -> int:
    """Enqueue one layer on the library stream: reads x (default act.x), writes out (default act.out).
    Returns 0 or the first nonzero return code."""
    x = act.x if x is None else x
    out = act.out if out is None else out
    for _, fn in layer_ops(lib, act, w, heads, eps, scale, x, out):
        rc = fn()
        if rc:
            return rc
    return 0


def encoder_schedule(lib, act: Activations, layers: list[LayerWeights], heads: int, eps: float, scale: float,
                     x_in: int | None = None, x_out: int | None = None) -> tuple[list[tuple[str, Callable[[], int]]], int]:
    """Every call of a full forward pass and the address the result lands in. Layer 0 reads x_in (default act.x),
    later layers ping-pong the residual stream between act.out and act.x, so x_in is never overwritten when it is a
    separate buffer; x_out, when given, receives the last layer's output instead of the ping-pong buffer."""
    cur = act.x if x_in is None else x_in
    nxt = act.out
    sched = []
    for i, w in enumerate(layers):
        dst = x_out if (x_out is not None and i == len(layers) - 1) else nxt
        sched += layer_ops(lib, act, w, heads, eps, scale, cur, dst)
        cur, nxt = dst, (act.x if nxt == act.out else act.out)
    return sched, cur


def encoder_forward(lib, act: Activations, layers: list[LayerWeights], heads: int, eps: float, scale: float,
                    x_in: int | None = None) -> int:
    """All layers (see encoder_schedule). Returns the address of the result."""
    sched, res = encoder_schedule(lib, act, layers, heads, eps, scale, x_in)
    for kind, fn in sched:
        rc = fn()
        if rc:
            raise RuntimeError(f"encoder {kind} failed with {rc}")
    return res


def launches_per_layer() -> int:
    return 7


def run_layer_once(rt: Runtime, x: np.ndarray, p: dict, heads: int, eps: float = 1e-6,
                   scale: float = 0.125) -> np.ndarray:
    """One layer on one sequence (host arrays in, host array out)."""
    S, D = x.shape
    F = np.asarray(p["w1"]).shape[1]
    rt.reset()
    w = upload_layer(rt, p)
    act = alloc_activations(rt, 1, S, D, F)
    rt.put(act.x, x)
    rc = layer_forward(rt.lib, act, w, heads, eps, scale)
    if rc:
        raise RuntimeError(f"layer_forward returned {rc}")
    return rt.get(act.out, S, D)
