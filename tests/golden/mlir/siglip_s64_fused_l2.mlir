builtin.module {
  func.func @siglip_encoder() {
    %x = softhier.hbm_buffer {offset = 4096 : i32} : memref<64x128xf16, "hbm_west">
    %ln1 = softhier.hbm_buffer {offset = 20480 : i32} : memref<64x128xf16, "hbm_west">
    %q = softhier.hbm_buffer {offset = 36864 : i32} : memref<64x128xf16, "hbm_west">
    %k = softhier.hbm_buffer {offset = 53248 : i32} : memref<64x128xf16, "hbm_west">
    %v = softhier.hbm_buffer {offset = 69632 : i32} : memref<64x128xf16, "hbm_west">
    %o = softhier.hbm_buffer {offset = 86016 : i32} : memref<64x128xf16, "hbm_west">
    %ao = softhier.hbm_buffer {offset = 102400 : i32} : memref<64x128xf16, "hbm_west">
    %h = softhier.hbm_buffer {offset = 118784 : i32} : memref<64x128xf16, "hbm_west">
    %ln2 = softhier.hbm_buffer {offset = 135168 : i32} : memref<64x128xf16, "hbm_west">
    %f1 = softhier.hbm_buffer {offset = 151552 : i32} : memref<64x256xf16, "hbm_west">
    %g = softhier.hbm_buffer {offset = 184320 : i32} : memref<64x256xf16, "hbm_west">
    %f2 = softhier.hbm_buffer {offset = 217088 : i32} : memref<64x128xf16, "hbm_west">
    %out = softhier.hbm_buffer {offset = 233472 : i32} : memref<64x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %x {seed = 1 : i32, lo = -16 : i32, hi = 16 : i32, scale = 0.125 : f32} : memref<64x128xf16, "hbm_west">
    %wq0 = softhier.hbm_buffer {offset = 249856 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wq0 {seed = 2 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wk0 = softhier.hbm_buffer {offset = 282624 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wk0 {seed = 3 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wv0 = softhier.hbm_buffer {offset = 315392 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wv0 {seed = 4 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wo0 = softhier.hbm_buffer {offset = 348160 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wo0 {seed = 5 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %w10 = softhier.hbm_buffer {offset = 380928 : i32} : memref<128x256xf16, "hbm_west">
    softhier.hbm_fill_lcg %w10 {seed = 6 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x256xf16, "hbm_west">
    %w20 = softhier.hbm_buffer {offset = 446464 : i32} : memref<256x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %w20 {seed = 7 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.00390625 : f32} : memref<256x128xf16, "hbm_west">
    %bq0 = softhier.hbm_buffer {offset = 512000 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bq0 {seed = 8 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bk0 = softhier.hbm_buffer {offset = 516096 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bk0 {seed = 9 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bv0 = softhier.hbm_buffer {offset = 520192 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bv0 {seed = 10 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bo0 = softhier.hbm_buffer {offset = 524288 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bo0 {seed = 11 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %b10 = softhier.hbm_buffer {offset = 528384 : i32} : memref<1x256xf16, "hbm_west">
    softhier.hbm_fill_lcg %b10 {seed = 12 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x256xf16, "hbm_west">
    %b20 = softhier.hbm_buffer {offset = 532480 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %b20 {seed = 13 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %g10 = softhier.hbm_buffer {offset = 536576 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %g10 {seed = 14 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x128xf16, "hbm_west">
    %be10 = softhier.hbm_buffer {offset = 540672 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %be10 {seed = 15 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.125 : f32} : memref<1x128xf16, "hbm_west">
    %g20 = softhier.hbm_buffer {offset = 544768 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %g20 {seed = 16 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x128xf16, "hbm_west">
    %be20 = softhier.hbm_buffer {offset = 548864 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %be20 {seed = 17 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.125 : f32} : memref<1x128xf16, "hbm_west">
    %wq1 = softhier.hbm_buffer {offset = 552960 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wq1 {seed = 102 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wk1 = softhier.hbm_buffer {offset = 585728 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wk1 {seed = 103 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wv1 = softhier.hbm_buffer {offset = 618496 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wv1 {seed = 104 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %wo1 = softhier.hbm_buffer {offset = 651264 : i32} : memref<128x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %wo1 {seed = 105 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x128xf16, "hbm_west">
    %w11 = softhier.hbm_buffer {offset = 684032 : i32} : memref<128x256xf16, "hbm_west">
    softhier.hbm_fill_lcg %w11 {seed = 106 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.0078125 : f32} : memref<128x256xf16, "hbm_west">
    %w21 = softhier.hbm_buffer {offset = 749568 : i32} : memref<256x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %w21 {seed = 107 : i32, lo = -8 : i32, hi = 8 : i32, scale = 0.00390625 : f32} : memref<256x128xf16, "hbm_west">
    %bq1 = softhier.hbm_buffer {offset = 815104 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bq1 {seed = 108 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bk1 = softhier.hbm_buffer {offset = 819200 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bk1 {seed = 109 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bv1 = softhier.hbm_buffer {offset = 823296 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bv1 {seed = 110 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %bo1 = softhier.hbm_buffer {offset = 827392 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %bo1 {seed = 111 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %b11 = softhier.hbm_buffer {offset = 831488 : i32} : memref<1x256xf16, "hbm_west">
    softhier.hbm_fill_lcg %b11 {seed = 112 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x256xf16, "hbm_west">
    %b21 = softhier.hbm_buffer {offset = 835584 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %b21 {seed = 113 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.0625 : f32} : memref<1x128xf16, "hbm_west">
    %g11 = softhier.hbm_buffer {offset = 839680 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %g11 {seed = 114 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x128xf16, "hbm_west">
    %be11 = softhier.hbm_buffer {offset = 843776 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %be11 {seed = 115 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.125 : f32} : memref<1x128xf16, "hbm_west">
    %g21 = softhier.hbm_buffer {offset = 847872 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %g21 {seed = 116 : i32, lo = 2 : i32, hi = 6 : i32, scale = 0.25 : f32} : memref<1x128xf16, "hbm_west">
    %be21 = softhier.hbm_buffer {offset = 851968 : i32} : memref<1x128xf16, "hbm_west">
    softhier.hbm_fill_lcg %be21 {seed = 117 : i32, lo = -4 : i32, hi = 4 : i32, scale = 0.125 : f32} : memref<1x128xf16, "hbm_west">
    softhier.mark {tag = "start"}
    softhier.layernorm %x, %g10, %be10 -> %ln1 {eps = 1.0e-6 : f32, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wq0 into %q {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %q, %bq0 -> %q {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wk0 into %k {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %k, %bk0 -> %k {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wv0 into %v {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %v, %bv0 -> %v {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.mark {tag = "qkv0"}
    softhier.attention %q, %k, %v -> %o {scale = 0.125 : f32, heads = 2 : i32, q_block = 64 : i32, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.group_barrier {grid_x = 4 : i32, grid_y = 4 : i32}
    softhier.mark {tag = "attn0"}
    softhier.gemm %o, %wo0 into %ao {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %ao, %bo0 -> %ao {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.add %x, %ao -> %h {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.layernorm %h, %g20, %be20 -> %ln2 {eps = 1.0e-6 : f32, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln2, %w10 into %f1 {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x256xf16, "hbm_west">, memref<64x256xf16, "hbm_west">
    softhier.add_bias %f1, %b10 -> %f1 {cluster = -1 : i32} : memref<64x256xf16, "hbm_west">, memref<1x256xf16, "hbm_west"> -> memref<64x256xf16, "hbm_west">
    softhier.gelu %f1 -> %g {cluster = -1 : i32} : memref<64x256xf16, "hbm_west"> -> memref<64x256xf16, "hbm_west">
    softhier.gemm %g, %w20 into %f2 {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x256xf16, "hbm_west">, memref<256x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %f2, %b20 -> %f2 {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.add %h, %f2 -> %out {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.mark {tag = "layer0"}
    softhier.layernorm %out, %g11, %be11 -> %ln1 {eps = 1.0e-6 : f32, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wq1 into %q {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %q, %bq1 -> %q {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wk1 into %k {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %k, %bk1 -> %k {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln1, %wv1 into %v {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %v, %bv1 -> %v {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.mark {tag = "qkv1"}
    softhier.attention %q, %k, %v -> %o {scale = 0.125 : f32, heads = 2 : i32, q_block = 64 : i32, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.group_barrier {grid_x = 4 : i32, grid_y = 4 : i32}
    softhier.mark {tag = "attn1"}
    softhier.gemm %o, %wo1 into %ao {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %ao, %bo1 -> %ao {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.add %out, %ao -> %h {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.layernorm %h, %g21, %be21 -> %ln2 {eps = 1.0e-6 : f32, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.gemm %ln2, %w11 into %f1 {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<128x256xf16, "hbm_west">, memref<64x256xf16, "hbm_west">
    softhier.add_bias %f1, %b11 -> %f1 {cluster = -1 : i32} : memref<64x256xf16, "hbm_west">, memref<1x256xf16, "hbm_west"> -> memref<64x256xf16, "hbm_west">
    softhier.gelu %f1 -> %g {cluster = -1 : i32} : memref<64x256xf16, "hbm_west"> -> memref<64x256xf16, "hbm_west">
    softhier.gemm %g, %w21 into %f2 {fmt = "fp16", tile_m = 64 : i32, tile_n = 64 : i32, tile_k = 64 : i32, pipeline, cluster = -1 : i32} : memref<64x256xf16, "hbm_west">, memref<256x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west">
    softhier.add_bias %f2, %b21 -> %f2 {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<1x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.add %h, %f2 -> %out {cluster = -1 : i32} : memref<64x128xf16, "hbm_west">, memref<64x128xf16, "hbm_west"> -> memref<64x128xf16, "hbm_west">
    softhier.mark {tag = "layer1"}
    softhier.dump_samples %x {seed = 200 : i32, n = 64 : i32, tag = "X"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %ln1 {seed = 206 : i32, n = 64 : i32, tag = "LN1"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %q {seed = 201 : i32, n = 64 : i32, tag = "Q"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %k {seed = 207 : i32, n = 64 : i32, tag = "K"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %v {seed = 211 : i32, n = 64 : i32, tag = "V"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %o {seed = 202 : i32, n = 64 : i32, tag = "O"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %h {seed = 203 : i32, n = 64 : i32, tag = "H"} : memref<64x128xf16, "hbm_west">
    softhier.dump_samples %g {seed = 204 : i32, n = 64 : i32, tag = "G"} : memref<64x256xf16, "hbm_west">
    softhier.dump_samples %out {seed = 205 : i32, n = 64 : i32, tag = "OUT"} : memref<64x128xf16, "hbm_west">
    func.return
  }
}
