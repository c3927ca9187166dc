builtin.module {
  func.func @siglip_encoder() {
    %x = softhier.hbm_buffer {offset = 4096 : i32} : memref<64x128xf16, "hbm_west">
    %ln1 = softhier.hbm_buffer {offset = 20480 : i32} : memref<64x128xf16, "hbm_west">
    %q = softhier.hbm_buffer {offset = 36864 : i32} : memref<64x128xf16, "hbm_west">
    %k = softhier.hbm_buffer {offset = 53248 : i32} : memref<64x128xf16, "hbm_west">
    %v = softhier.hbm_buffer {offset = 69632 : i32} : memref<64x128xf16, "hbm_west">
    %kT = softhier.hbm_buffer {offset = 86016 : i32} : memref<128x64xf16, "hbm_west">
    %sc = softhier.hbm_buffer {offset = 102400 : i32} : memref<128x64xf16, "hbm_west">
    %o = softhier.hbm_buffer {offset = 118784 : i32} : memref<64x128xf16, "hbm_west">
    %ao = softhier.hbm_buffer {offset = 135168 : i32} : memref<64x128xf16, "hbm_west">
    %h = softhier.hbm_buffer {offset = 151552 : i32} : memref<64x128xf16, "hbm_west">
    %ln2 = softhier.hbm_buffer {offset = 167936 : i32} : memref<64x128xf16, "hbm_west">
    %f1 = softhier.hbm_buffer {offset = 184320 : i32} : memref<64x256xf16, "hbm_west">
    %g = softhier.hbm_buffer {offset = 217088 : i32} : memref<64x256xf16, "hbm_west">
    %f2 = softhier.hbm_buffer {offset = 249856 : i32} : memref<64x128xf16, "hbm_west">
    %out = softhier.hbm_buffer {offset = 266240 : i32} : memref<64x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %x {seed = 1 : i32, lo = -16 : i32, hi = 16 : i32, scale = 0.125 : f32} : memref<64x128xf16, "hbm_west">
    %wq0 = softhier.hbm_buffer {offset = 282624 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wq0 {seed = 2 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wk0 = softhier.hbm_buffer {offset = 315392 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wk0 {seed = 3 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wv0 = softhier.hbm_buffer {offset = 348160 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wv0 {seed = 4 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wo0 = softhier.hbm_buffer {offset = 380928 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wo0 {seed = 5 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %w10 = softhier.hbm_buffer {offset = 413696 : i32} : memref<128x256xf16, "hbm_west">
    softhier.hbm_fill_lcg %w10 {seed = 6 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x256xf16, "hbm_west">
    %w20 = softhier.hbm_buffer {offset = 479232 : i32} : memref<256x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %w20 {seed = 7 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.00390625 : f32} : memref<256x128xf16, "hbm_west">
    %bq0 = softhier.hbm_buffer {offset = 544768 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bq0 {seed = 8 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bk0 = softhier.hbm_buffer {offset = 548864 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bk0 {seed = 9 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bv0 = softhier.hbm_buffer {offset = 552960 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bv0 {seed = 10 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bo0 = softhier.hbm_buffer {offset = 557056 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bo0 {seed = 11 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %b10 = softhier.hbm_buffer {offset = 561152 : i32} : memref<1x256xf16, "hbm_west">
    softhier.hbm_fill_lcg %b10 {seed = 12 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x256xf16, "hbm_west">
    %b20 = softhier.hbm_buffer {offset = 565248 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %b20 {seed = 13 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %g10 = softhier.hbm_buffer {offset = 569344 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %g10 {seed = 14 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x128xf16, "hbm_west">
    %be10 = softhier.hbm_buffer {offset = 573440 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %be10 {seed = 15 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.125 : f32} : memref<1x128xf16, "hbm_west">
    %g20 = softhier.hbm_buffer {offset = 577536 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %g20 {seed = 16 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x128xf16, "hbm_west">
    %be20 = softhier.hbm_buffer {offset = 581632 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %be20 {seed = 17 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.125 : f32} : memref<1x128xf16, "hbm_west">
    softhier.mark {tag = "start"}
    softhier.layernorm %x, %g10, %be10 -> %ln1 {eps = 1.0e-6 : f32, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wq0 into %q {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %q, %bq0 -> %q {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wk0 into %k {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %k, %bk0 -> %k {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wv0 into %v {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %v, %bv0 -> %v {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.mark {tag = "qkv0"}
    softhier.transpose %k -> %kT {cluster = -1 : i32} : memref<64x128xf16, "hbm_west"> -> memref<128x64xf16, "hbm_west">
    %q0_0 = softhier.view %q : memref<64x128xf16, "hbm_west"> -> memref<64x64xf16, strided<[128, 1], offset: 0>, "hbm_west">
    %kT0_0 = softhier.view %kT : memref<128x64xf16, "hbm_west"> -> memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west">
    %s0_0 = softhier.view %sc : memref<128x64xf16, "hbm_west"> -> memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west">
    %v0_0 = softhier.view %v : memref<64x128xf16, "hbm_west"> -> memref<64x64xf16, strided<[128, 1], offset: 0>, "hbm_west">
    %o0_0 = softhier.view %o : memref<64x128xf16, "hbm_west"> -> memref<64x64xf16, strided<[128, 1], offset: 0>, "hbm_west">
    softhier.gemm %q0_0, %kT0_0 into %s0_0 {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 64 : i32, pipeline, cluster = 0 : i32} : memref<64x64xf16, strided<[128, 1], offset: 0>, "hbm_west">, memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west">, memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west">
    softhier.softmax %s0_0 -> %s0_0 {scale = 0.125 : f32, cluster = 0 : i32} : memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west"> -> memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west">
    softhier.gemm %s0_0, %v0_0 into %o0_0 {fmt = "fp16", tile_m = 256 : i32, tile_n = 64 : i32, tile_k = 256 : i32, pipeline, cluster = 0 : i32} : memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west">, memref<64x64xf16, strided<[128, 1], offset: 0>, "hbm_west">, memref<64x64xf16, strided<[128, 1], offset: 0>, "hbm_west">
    %q0_1 = softhier.view %q : memref<64x128xf16, "hbm_west"> -> memref<64x64xf16, strided<[128, 1], offset: 64>, "hbm_west">
    %kT0_1 = softhier.view %kT : memref<128x64xf16, "hbm_west"> -> memref<64x64xf16, strided<[64, 1], offset: 4096>, "hbm_west">
    %s0_1 = softhier.view %sc : memref<128x64xf16, "hbm_west"> -> memref<64x64xf16, strided<[64, 1], offset: 4096>, "hbm_west">
    %v0_1 = softhier.view %v : memref<64x128xf16, "hbm_west"> -> memref<64x64xf16, strided<[128, 1], offset: 64>, "hbm_west">
    %o0_1 = softhier.view %o : memref<64x128xf16, "hbm_west"> -> memref<64x64xf16, strided<[128, 1], offset: 64>, "hbm_west">
    softhier.gemm %q0_1, %kT0_1 into %s0_1 {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 64 : i32, pipeline, cluster = 1 : i32} : memref<64x64xf16, strided<[128, 1], offset: 64>, "hbm_west">, memref<64x64xf16, strided<[64, 1], offset: 4096>, "hbm_west">, memref<64x64xf16, strided<[64, 1], offset: 4096>, "hbm_west">
    softhier.softmax %s0_1 -> %s0_1 {scale = 0.125 : f32, cluster = 1 : i32} : memref<64x64xf16, strided<[64, 1], offset: 4096>, "hbm_west"> -> memref<64x64xf16, strided<[64, 1], offset: 4096>, "hbm_west">
    softhier.gemm %s0_1, %v0_1 into %o0_1 {fmt = "fp16", tile_m = 256 : i32, tile_n = 64 : i32, tile_k = 256 : i32, pipeline, cluster = 1 : i32} : memref<64x64xf16, strided<[64, 1], offset: 4096>, "hbm_west">, memref<64x64xf16, strided<[128, 1], offset: 64>, "hbm_west">, memref<64x64xf16, strided<[128, 1], offset: 64>, "hbm_west">
    softhier.group_barrier {grid_x = 4 : i32, grid_y = 4 : i32}
    softhier.mark {tag = "attn0"}
    softhier.gemm %o, %wo0 into %ao {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %ao, %bo0 -> %ao {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.add %x, %ao -> %h {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.layernorm %h, %g20, %be20 -> %ln2 {eps = 1.0e-6 : f32, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln2, %w10 into %f1 {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x256xf16, "hbm_west">, memref<64x256xf16, "hbm_west">
    softhier.add_bias %f1, %b10 -> %f1 {cluster = -1 : i32} : memref<64x256xf16, "hbm_west">, memref<1x256xf16, "hbm_west"> -> memref<64x256xf16, "hbm_west">
    softhier.gelu %f1 -> %g {cluster = -1 : i32} : memref<64x256xf16, "hbm_west"> -> memref<64x256xf16, "hbm_west">
    softhier.gemm %g, %w20 into %f2 {fmt = "fp16", tile_m = 256 : i32, tile_n = 256 : i32, tile_k = 256 : i32, pipeline, cluster = -1 : i32} : memref<64x256xf16, "hbm_west">, memref<256x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %f2, %b20 -> %f2 {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.add %h, %f2 -> %out {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.mark {tag = "layer0"}
    softhier.dump_samples %x {seed = 200 : i32, n = 64 : i32, tag = "X"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %ln1 {seed = 206 : i32, n = 64 : i32, tag = "LN1"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %q {seed = 201 : i32, n = 64 : i32, tag = "Q"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %k {seed = 207 : i32, n = 64 : i32, tag = "K"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %kT {seed = 208 : i32, n = 64 : i32, tag = "KT"} : memref<128x64xf16, "hbm_west">
    %p0view = softhier.view %sc : memref<128x64xf16, "hbm_west"> -> memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west">
    softhier.dump_samples %p0view {seed = 209 : i32, n = 64 : i32, tag = "P0"} : memref<64x64xf16, strided<[64, 1], offset: 0>, "hbm_west">
    softhier.dump_samples %v {seed = 211 : i32, n = 64 : i32, tag = "V"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %o {seed = 202 : i32, n = 64 : i32, tag = "O"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %h {seed = 203 : i32, n = 64 : i32, tag = "H"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %g {seed = 204 : i32, n = 64 : i32, tag = "G"} : memref<64x256xf16, "hbm_west">
    softhier.dump_samples %out {seed = 205 : i32, n = 64 : i32, tag = "OUT"} : memref<64x128xf16, "hbm_west">
    func.return
  }
}
