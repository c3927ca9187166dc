// Llama-style decoder ops of the operator library (reference: runtime/sh_llm.inc.c:100-370, declared at
// runtime/sh_ops.h:277-304): RMSNorm, rotate-half RoPE, SiLU-gated product, token-masked softmax rows and the
// SmolVLM pixel shuffle. The masked / grouped-query attention entry points live with the other attention kernels.
//
// The reference computes these in fp16 SIMD lanes with a degree-3 exp2 on TCDM-staged row blocks; here they are
// single-pass HBM kernels with fp32 arithmetic and one fp16 rounding per output: one warp per row for the row
// reductions (RMSNorm, softmax), one thread per element (pair) for the elementwise ones.
#include <math.h>

#include "sh_internal.cuh"

namespace {

constexpr int kWarps = 8;            // warps per block of the row kernels
constexpr uint32_t kPadTok = 0xFFFFu;

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// y = x rsqrt(mean x^2 + eps) gamma; one warp per row, the row read twice (the second pass from L1 / L2)
__global__ void __launch_bounds__(kWarps * 32) k_rmsnorm(__half *y, const __half *x, const __half *g, uint32_t rows,
                                                        uint32_t cols, uint32_t ld, float eps) {
    const uint32_t row = blockIdx.x * kWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const __half *xr = x + (size_t)row * ld;
    float ss = 0.f;
    for (uint32_t c = lane; c < cols; c += 32) {
        const float t = __half2float(xr[c]);
        ss = fmaf(t, t, ss);
    }
    const float rs = rsqrtf(warp_sum_f(ss) / (float)cols + eps);
    __half *yr = y + (size_t)row * ld;
    for (uint32_t c = lane; c < cols; c += 32)
        yr[c] = __float2half_rn(__half2float(xr[c]) * rs * __half2float(g[c]));
}

// rotate-half RoPE: thread per (row, head, i < dh / 2); table row = cos[dh/2] | sin[dh/2]
__global__ void __launch_bounds__(256) k_rope(__half *y, const __half *x, const __half *tab, uint32_t rows,
                                             uint32_t cols, uint32_t ld, uint32_t ldt, uint32_t dh) {
    const uint32_t half = dh >> 1, per_row = cols >> 1;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)rows * per_row) return;
    const uint32_t r = (uint32_t)(t / per_row), e = (uint32_t)(t % per_row);
    const uint32_t h = e / half, i = e % half;
    const size_t b = (size_t)r * ld + (size_t)h * dh + i;
    const float a = __half2float(x[b]), bb = __half2float(x[b + half]);
    const float c = __half2float(tab[(size_t)r * ldt + i]), s = __half2float(tab[(size_t)r * ldt + half + i]);
    y[b] = __float2half_rn(a * c - bb * s);
    y[b + half] = __float2half_rn(bb * c + a * s);
}

// y = a b / (1 + e^-a)
__global__ void __launch_bounds__(256) k_silu_mul(__half *y, const __half *a, const __half *b, uint32_t rows,
                                                 uint32_t cols, uint32_t ld) {
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)rows * cols) return;
    const size_t i = (size_t)(t / cols) * ld + (t % cols);
    const float av = __half2float(a[i]);
    y[i] = __float2half_rn(av / (1.f + __expf(-av)) * __half2float(b[i]));
}

// softmax(scale x + mask) per row: key j stays iff tok_k[j] <= tok_q[row]; a PAD query row is uniform. One warp per
// row, three passes over the row (max, sum, write).
__global__ void __launch_bounds__(kWarps * 32) k_softmax_masked(__half *y, const __half *x, uint32_t rows,
                                                               uint32_t cols, uint32_t ld, float sl2,
                                                               const uint16_t *tok_q, const uint16_t *tok_k) {
    const uint32_t row = blockIdx.x * kWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const __half *xr = x + (size_t)row * ld;
    __half *yr = y + (size_t)row * ld;
    const uint32_t tq = tok_q[row];
    if (tq == kPadTok) {
        const __half u = __float2half_rn(1.f / (float)cols);
        for (uint32_t c = lane; c < cols; c += 32) yr[c] = u;
        return;
    }
    float m = -INFINITY;
    for (uint32_t c = lane; c < cols; c += 32)
        if (tok_k[c] <= tq) m = fmaxf(m, __half2float(xr[c]) * sl2);
    m = warp_max_f(m);
    float s = 0.f;
    for (uint32_t c = lane; c < cols; c += 32)
        if (tok_k[c] <= tq) s += exp2f(__half2float(xr[c]) * sl2 - m);
    const float inv = 1.f / warp_sum_f(s);
    for (uint32_t c = lane; c < cols; c += 32)
        yr[c] = __float2half_rn(tok_k[c] <= tq ? exp2f(__half2float(xr[c]) * sl2 - m) * inv : 0.f);
}

// output token (gr, gb) = the s x s block of source tokens rows gr*s.., cols gb*s.., row-major, each D wide
__global__ void __launch_bounds__(256) k_pixel_shuffle(__half *dst, const __half *src, uint32_t grid, uint32_t D,
                                                      uint32_t s) {
    const uint32_t g = grid / s, out_cols = s * s * D;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)g * g * out_cols) return;
    const uint32_t tok = (uint32_t)(t / out_cols), e = (uint32_t)(t % out_cols);
    const uint32_t gr = tok / g, gb = tok % g, blk = e / D, d = e % D;
    const uint32_t i = blk / s, j = blk % s;
    dst[t] = src[((size_t)(gr * s + i) * grid + gb * s + j) * D + d];
}

unsigned blocks_for(uint64_t n, unsigned per) { return (unsigned)((n + per - 1) / per); }

}  // namespace

extern "C" {

void sh_rmsnorm(uint64_t y, uint64_t x, uint64_t gamma, uint32_t rows, uint32_t cols, uint32_t ld, float eps,
                uint32_t) {
    if (rows == 0 || cols == 0) return;
    if ((cols & 3) || ld < cols || !x || !y || !gamma) {   // sh_llm.inc.c:122
        sh::set_error(-1, "[sh_rmsnorm] cols %u %% 4 != 0 (ld %u)", cols, ld);
        return;
    }
    k_rmsnorm<<<blocks_for(rows, kWarps), kWarps * 32, 0, sh::stream()>>>((__half *)y, (const __half *)x,
                                                                           (const __half *)gamma, rows, cols, ld, eps);
    sh::cuda_ok(cudaGetLastError(), "sh_rmsnorm");
}

void sh_rope(uint64_t y, uint64_t x, uint64_t cos_sin, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t ld_table,
             uint32_t dh, uint32_t) {
    if (rows == 0 || cols == 0) return;
    if ((dh & 7) || dh == 0 || cols % dh || ld < cols || ld_table < dh) {   // sh_llm.inc.c:147
        sh::set_error(-1, "[sh_rope] need dh %% 8 == 0 and cols %% dh == 0 (dh=%u cols=%u)", dh, cols);
        return;
    }
    const uint64_t n = (uint64_t)rows * (cols / 2);
    k_rope<<<blocks_for(n, 256), 256, 0, sh::stream()>>>((__half *)y, (const __half *)x, (const __half *)cos_sin,
                                                          rows, cols, ld, ld_table, dh);
    sh::cuda_ok(cudaGetLastError(), "sh_rope");
}

void sh_silu_mul(uint64_t y, uint64_t a, uint64_t b, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t) {
    if (rows == 0 || cols == 0) return;
    if ((cols & 3) || ld < cols) {   // sh_llm.inc.c:170
        sh::set_error(-1, "[sh_silu_mul] cols %u %% 4 != 0", cols);
        return;
    }
    k_silu_mul<<<blocks_for((uint64_t)rows * cols, 256), 256, 0, sh::stream()>>>(
        (__half *)y, (const __half *)a, (const __half *)b, rows, cols, ld);
    sh::cuda_ok(cudaGetLastError(), "sh_silu_mul");
}

void sh_softmax_masked(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, float scale,
                       uint64_t tok_q, uint64_t tok_k, uint32_t) {
    if (rows == 0 || cols == 0) return;
    if ((cols & 3) || scale <= 0.f || ld < cols || !tok_q || !tok_k) {   // sh_llm.inc.c:244
        sh::set_error(-1, "[sh_softmax_masked] need cols %% 4 == 0 and scale > 0");
        return;
    }
    k_softmax_masked<<<blocks_for(rows, kWarps), kWarps * 32, 0, sh::stream()>>>(
        (__half *)y, (const __half *)x, rows, cols, ld, scale * 1.4426950408889634f, (const uint16_t *)tok_q,
        (const uint16_t *)tok_k);
    sh::cuda_ok(cudaGetLastError(), "sh_softmax_masked");
}

void sh_pixel_shuffle(uint64_t dst, uint64_t src, uint32_t grid, uint32_t D, uint32_t s, uint32_t) {
    if (grid == 0 || D == 0) return;
    if (s == 0 || grid % s) {
        sh::set_error(-1, "[sh_pixel_shuffle] grid %u not a multiple of the scale %u", grid, s);
        return;
    }
    const uint64_t g = grid / s, n = g * g * s * s * D;
    k_pixel_shuffle<<<blocks_for(n, 256), 256, 0, sh::stream()>>>((__half *)dst, (const __half *)src, grid, D, s);
    sh::cuda_ok(cudaGetLastError(), "sh_pixel_shuffle");
}

}  // extern "C"
