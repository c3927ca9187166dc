builtin.module {
  func.func @siglip_encoder() {
    %x = softhier.hbm_buffer {offset = 4096 : i32} : memref<256x768xf16, "hbm_west">
    %ln1 = softhier.hbm_buffer {offset = 397312 : i32} : memref<256x768xf16, "hbm_west">
    %q = softhier.hbm_buffer {offset = 790528 : i32} : memref<256x768xf16, "hbm_west">
    %k = softhier.hbm_buffer {offset = 1183744 : i32} : memref<256x768xf16, "hbm_west">
    %v = softhier.hbm_buffer {offset = 1576960 : i32} : memref<256x768xf16, "hbm_west">
    %o = softhier.hbm_buffer {offset = 1970176 : i32} : memref<256x768xf16, "hbm_west">
    %ao = softhier.hbm_buffer {offset = 2363392 : i32} : memref<256x768xf16, "hbm_west">
    %h = softhier.hbm_buffer {offset = 2756608 : i32} : memref<256x768xf16, "hbm_west">
    %ln2 = softhier.hbm_buffer {offset = 3149824 : i32} : memref<256x768xf16, "hbm_west">
    %f1 = softhier.hbm_buffer {offset = 3543040 : i32} : memref<256x3072xf16, "hbm_west">
    %g = softhier.hbm_buffer {offset = 5115904 : i32} : memref<256x3072xf16, "hbm_west">
    %f2 = softhier.hbm_buffer {offset = 6688768 : i32} : memref<256x768xf16, "hbm_west">
    %out = softhier.hbm_buffer {offset = 7081984 : i32} : memref<256x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %x {seed = 1 : i32, lo = -16 : i32, hi = 16 : i32, scale = 0.125 : f32} : memref<256x768xf16, "hbm_west">
    %wq0 = softhier.hbm_buffer {offset = 7475200 : i32} : memref<768x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %wq0 {seed = 2 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<768x768xf16, "hbm_west">
    %wk0 = softhier.hbm_buffer {offset = 8654848 : i32} : memref<768x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %wk0 {seed = 3 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<768x768xf16, "hbm_west">
    %wv0 = softhier.hbm_buffer {offset = 9834496 : i32} : memref<768x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %wv0 {seed = 4 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<768x768xf16, "hbm_west">
    %wo0 = softhier.hbm_buffer {offset = 11014144 : i32} : memref<768x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %wo0 {seed = 5 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<768x768xf16, "hbm_west">
    %w10 = softhier.hbm_buffer {offset = 12193792 : i32} : memref<768x3072xf16, "hbm_west">
    softhier.hbm_fill_lcg %w10 {seed = 6 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<768x3072xf16, "hbm_west">
    %w20 = softhier.hbm_buffer {offset = 16912384 : i32} : memref<3072x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %w20 {seed = 7 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.00390625 : f32} : memref<3072x768xf16, "hbm_west">
    %bq0 = softhier.hbm_buffer {offset = 21630976 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %bq0 {seed = 8 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x768xf16, "hbm_west">
    %bk0 = softhier.hbm_buffer {offset = 21635072 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %bk0 {seed = 9 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x768xf16, "hbm_west">
    %bv0 = softhier.hbm_buffer {offset = 21639168 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %bv0 {seed = 10 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x768xf16, "hbm_west">
    %bo0 = softhier.hbm_buffer {offset = 21643264 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %bo0 {seed = 11 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x768xf16, "hbm_west">
    %b10 = softhier.hbm_buffer {offset = 21647360 : i32} : memref<1x3072xf16, "hbm_west">
    softhier.hbm_fill_lcg %b10 {seed = 12 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x3072xf16, "hbm_west">
    %b20 = softhier.hbm_buffer {offset = 21655552 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %b20 {seed = 13 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x768xf16, "hbm_west">
    %g10 = softhier.hbm_buffer {offset = 21659648 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %g10 {seed = 14 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x768xf16, "hbm_west">
    %be10 = softhier.hbm_buffer {offset = 21663744 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %be10 {seed = 15 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.125 : f32} : memref<1x768xf16, "hbm_west">
    %g20 = softhier.hbm_buffer {offset = 21667840 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %g20 {seed = 16 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x768xf16, "hbm_west">
    %be20 = softhier.hbm_buffer {offset = 21671936 : i32} : memref<1x768xf16, "hbm_west">
    softhier.hbm_fill_lcg %be20 {seed = 17 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.125 : f32} : memref<1x768xf16, "hbm_west">
    softhier.mark {tag = "start"}
    softhier.layernorm %x, %g10, %be10 -> %ln1 {eps = 1.0e-6 : f32, cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.gemm %ln1, %wq0 into %q {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<768x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west">
    softhier.add_bias %q, %bq0 -> %q {cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.gemm %ln1, %wk0 into %k {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<768x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west">
    softhier.add_bias %k, %bk0 -> %k {cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.gemm %ln1, %wv0 into %v {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<768x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west">
    softhier.add_bias %v, %bv0 -> %v {cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.mark {tag = "qkv0"}
    softhier.attention %q, %k, %v -> %o {scale = 0.125 : f32, heads = 12 : i32, q_block = 64 : i32, cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.group_barrier {grid_x = 4 : i32, grid_y = 4 : i32}
    softhier.mark {tag = "attn0"}
    softhier.gemm %o, %wo0 into %ao {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<768x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west">
    softhier.add_bias %ao, %bo0 -> %ao {cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.add %x, %ao -> %h {cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.layernorm %h, %g20, %be20 -> %ln2 {eps = 1.0e-6 : f32, cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.gemm %ln2, %w10 into %f1 {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<768x3072xf16, "hbm_west">, memref<256x3072xf16, "hbm_west">
    softhier.add_bias %f1, %b10 -> %f1 {cluster = -1 : i32} : memref<256x3072xf16, "hbm_west">, memref<1x3072xf16, "hbm_west"> -> memref<256x3072xf16, "hbm_west">
    softhier.gelu %f1 -> %g {cluster = -1 : i32} : memref<256x3072xf16, "hbm_west"> -> memref<256x3072xf16, "hbm_west">
    softhier.gemm %g, %w20 into %f2 {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<256x3072xf16, "hbm_west">, memref<3072x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west">
    softhier.add_bias %f2, %b20 -> %f2 {cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<1x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.add %h, %f2 -> %out {cluster = -1 : i32} : memref<256x768xf16, "hbm_west">, memref<256x768xf16, "hbm_west"> -> memref<256x768xf16, "hbm_west">
    softhier.mark {tag = "layer0"}
    softhier.dump_samples %x {seed = 200 : i32, n = 64 : i32, tag = "X"} : memref<256x768xf16, "hbm_west">
    softhier.dump_samples %ln1 {seed = 206 : i32, n = 64 : i32, tag = "LN1"} : memref<256x768xf16, "hbm_west">
    softhier.dump_samples %q {seed = 201 : i32, n = 64 : i32, tag = "Q"} : memref<256x768xf16, "hbm_west">
    softhier.dump_samples %k {seed = 207 : i32, n = 64 : i32, tag = "K"} : memref<256x768xf16, "hbm_west">
    softhier.dump_samples %v {seed = 211 : i32, n = 64 : i32, tag = "V"} : memref<256x768xf16, "hbm_west">
    softhier.dump_samples %o {seed = 202 : i32, n = 64 : i32, tag = "O"} : memref<256x768xf16, "hbm_west">
    softhier.dump_samples %h {seed = 203 : i32, n = 64 : i32, tag = "H"} : memref<256x768xf16, "hbm_west">
    softhier.dump_samples %g {seed = 204 : i32, n = 64 : i32, tag = "G"} : memref<256x3072xf16, "hbm_west">
    softhier.dump_samples %out {seed = 205 : i32, n = 64 : i32, tag = "OUT"} : memref<256x768xf16, "hbm_west">
    func.return
  }
}
