"""A looped multi-layer SigLIP encoder module in the softhier dialect (shared by the CPU and GPU loop tests).

The compact form of a stacked encoder (the frontend's layer, frontend/siglip.py:133-168, inside `scf.for`): every
layer parameter is an indexed `softhier.hbm_buffer %L {offset, stride}` (layer L's copy at offset + L * stride), the
GELU runs over indexed column views of FC1's output in a nested loop, the layer's output is written back into %x so
the next iteration reads it, and an indexed `dump_samples` prints the residual stream after every layer. The lowering
rules follow the reference's translate test tests/filecheck/loop_translate.mlir:26-37 (scf.for -> C for loop,
indexed buffer / view address = offset + index * stride, indexed dump appends the index to the tag).
"""
from __future__ import annotations

PARAMS = ("wq", "wk", "wv", "wo", "w1", "w2", "bq", "bk", "bv", "bo", "b1", "b2", "g1", "be1", "g2", "be2")


def _mt(r: int, c: int) -> str:
    return f'memref<{r}x{c}xf16, "hbm_west">'


def param_shapes(D: int, F: int) -> dict[str, tuple[int, int]]:
    sh = {"wq": (D, D), "wk": (D, D), "wv": (D, D), "wo": (D, D), "w1": (D, F), "w2": (F, D), "b1": (1, F)}
    for n in ("bq", "bk", "bv", "bo", "b2", "g1", "be1", "g2", "be2"):
        sh[n] = (1, D)
    return sh


def layout(S: int, D: int, F: int) -> tuple[dict[str, int], dict[str, int], int, int]:
    """(activation offsets, parameter offsets inside one layer's block, layer block bytes, weights base)."""
    off, act = 0x1000, {}
    for name, (r, c) in (("x", (S, D)), ("ln1", (S, D)), ("q", (S, D)), ("k", (S, D)), ("v", (S, D)), ("o", (S, D)),
                         ("ao", (S, D)), ("h", (S, D)), ("ln2", (S, D)), ("f1", (S, F)), ("g", (S, F)),
                         ("f2", (S, D))):
        act[name] = off
        off += (r * c * 2 + 4095) // 4096 * 4096
    base, poff, p = off, {}, 0
    for name in PARAMS:
        r, c = param_shapes(D, F)[name]
        poff[name] = p
        p += (r * c * 2 + 4095) // 4096 * 4096
    return act, poff, p, base


def looped_encoder(S: int, D: int, F: int, H: int, layers: int, gelu_block: int = 64, seed: int = 7,
                   nsamples: int = 32) -> str:
    act, poff, stride, base = layout(S, D, F)
    sh = param_shapes(D, F)
    A = _mt(S, D)
    L = []
    e = L.append
    e("builtin.module {")
    e("  func.func @looped_encoder() {")
    e("    %c0 = arith.constant 0 : index")
    e("    %c1 = arith.constant 1 : index")
    e(f"    %cL = arith.constant {layers} : index")
    e(f"    %cG = arith.constant {F // gelu_block} : index")
    for name, o in act.items():
        r, c = (S, F) if name in ("f1", "g") else (S, D)
        e(f"    %{name} = softhier.hbm_buffer {{offset = {o} : i32}} : {_mt(r, c)}")
    e("    scf.for %L = %c0 to %cL step %c1 {")
    e("      %L1 = arith.addi %L, %c1 : index")
    for name in PARAMS:
        r, c = sh[name]
        e(f"      %{name} = softhier.hbm_buffer %L {{offset = {base + poff[name]} : i32, stride = {stride} : i32}}"
          f" : {_mt(r, c)}")
    gemm = 'fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32'
    row = _mt(1, D)
    e(f"      softhier.layernorm %x, %g1, %be1 -> %ln1 {{eps = 1.0e-6 : f32, cluster = -1 : i32}} : {A}, {row}, {row}"
      f" -> {A}")
    for t in ("q", "k", "v"):
        e(f"      softhier.gemm %ln1, %w{t} into %{t} {{{gemm}}} : {A}, {_mt(D, D)}, {A}")
        e(f"      softhier.add_bias %{t}, %b{t} -> %{t} {{cluster = -1 : i32}} : {A}, {row} -> {A}")
    e(f"      softhier.attention %q, %k, %v -> %o {{scale = {1.0 / (D // H) ** 0.5} : f32, heads = {H} : i32, "
      f"cluster = -1 : i32}} : {A}, {A}, {A} -> {A}")
    e(f"      softhier.gemm %o, %wo into %ao {{{gemm}}} : {A}, {_mt(D, D)}, {A}")
    e(f"      softhier.add_bias %ao, %bo -> %ao {{cluster = -1 : i32}} : {A}, {row} -> {A}")
    e(f"      softhier.add %x, %ao -> %h {{cluster = -1 : i32}} : {A}, {A} -> {A}")
    e(f"      softhier.layernorm %h, %g2, %be2 -> %ln2 {{eps = 1.0e-6 : f32, cluster = -1 : i32}} : {A}, {row}, "
      f"{row} -> {A}")
    e(f"      softhier.gemm %ln2, %w1 into %f1 {{{gemm}}} : {A}, {_mt(D, F)}, {_mt(S, F)}")
    e(f"      softhier.add_bias %f1, %b1 -> %f1 {{cluster = -1 : i32}} : {_mt(S, F)}, {_mt(1, F)} -> {_mt(S, F)}")
    vt = f'memref<{S}x{gelu_block}xf16, strided<[{F}, 1], offset: 0>, "hbm_west">'
    e("      scf.for %j = %c0 to %cG step %c1 {")
    e(f"        %f1j = softhier.view %f1, %j {{stride = {gelu_block} : i32}} : {_mt(S, F)} -> {vt}")
    e(f"        %gj = softhier.view %g, %j {{stride = {gelu_block} : i32}} : {_mt(S, F)} -> {vt}")
    e(f"        softhier.gelu %f1j -> %gj {{cluster = -1 : i32}} : {vt} -> {vt}")
    e("      }")
    e(f"      softhier.gemm %g, %w2 into %f2 {{{gemm}}} : {_mt(S, F)}, {_mt(F, D)}, {A}")
    e(f"      softhier.add_bias %f2, %b2 -> %f2 {{cluster = -1 : i32}} : {A}, {row} -> {A}")
    e(f"      softhier.add %h, %f2 -> %x {{cluster = -1 : i32}} : {A}, {A} -> {A}")
    e('      softhier.mark %L1 {tag = "layer"}')
    e(f'      softhier.dump_samples %x, %L1 {{seed = {seed} : i32, n = {nsamples} : i32, tag = "L"}} : {A}')
    e("    }")
    e("    func.return")
    e("  }")
    e("}")
    return "\n".join(L) + "\n"
