// Test helpers of the operator library (reference: runtime/sh_test.inc.c:2-115, sh_rt.inc.c:31-59; declared at
// runtime/sh_ops.h:220-240).
//
// The fills run on the GPU: each thread jumps the 32-bit LCG to the start of its chunk with the composed affine
// map (log2 steps) and then steps sequentially, so the bytes equal the reference's single-core loop exactly.
// Dumps and checks read the device tensor back and print the reference's line formats.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "sh_internal.cuh"

namespace {

constexpr uint32_t kA = 1664525u, kC = 1013904223u, kSeedXor = 0x9e3779b9u;

struct Affine {
    uint32_t a, c;
};
__host__ __device__ inline Affine compose(Affine first, Affine then) {
    return Affine{then.a * first.a, then.a * first.c + then.c};
}
// the map that advances the state by n steps
__host__ __device__ inline Affine lcg_jump(uint64_t n) {
    Affine acc{1u, 0u}, p{kA, kC};
    while (n) {
        if (n & 1) acc = compose(acc, p);
        p = compose(p, p);
        n >>= 1;
    }
    return acc;
}

constexpr uint32_t kChunk = 64;   // elements per thread

__global__ void k_fill_lcg(__half *a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, int lo, uint32_t span,
                           float scale) {
    const uint64_t total = (uint64_t)rows * cols;
    const uint64_t start = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * kChunk;
    if (start >= total) return;
    const Affine j = lcg_jump(start);
    uint32_t s = j.a * (seed ^ kSeedXor) + j.c;   // state before element `start` is drawn
    uint64_t r = start / cols, c = start - r * cols;
    const uint64_t end = start + kChunk < total ? start + kChunk : total;
    for (uint64_t i = start; i < end; ++i) {
        s = s * kA + kC;
        const int v = lo + (int)((s >> 8) % span);
        a[r * ld + c] = __float2half_rn((float)v * scale);
        if (++c == cols) {
            c = 0;
            ++r;
        }
    }
}

// ---- N(mean, std) with every step an IEEE-exact fp32 operation ------------------------------------------------
// Box-Muller over one LCG draw pair (d0, d1) per element, row-major: u = (float(d) + 0.5) * 2^-24,
// z = sqrt(-2 ln u0) * cos(2 pi u1), value = fp16_rne(mean + stdev * z). ln and cos are series of this file's own,
// from calculus: ln u = e ln2 + 2 atanh((m - 1) / (m + 1)) with u = m 2^e, m in [sqrt(1/2), sqrt(2)), atanh to
// t^13; cos(2 pi u) = +-cos / +-sin of (pi / 2) r with 4u = q + r, q = rint(4u), |r| <= 1/2, Taylor to r^10 / r^11.
// Each step is one correctly rounded add / multiply / divide / sqrt in a fixed order (the _rn intrinsics on the
// device, so nothing is contracted into an FMA; the host build disables contraction), so the host, the device and
// the test oracle's numpy float32 restatement produce the same bits.
#ifdef __CUDA_ARCH__
#define RN_ADD(a, b) __fadd_rn((a), (b))
#define RN_MUL(a, b) __fmul_rn((a), (b))
#define RN_DIV(a, b) __fdiv_rn((a), (b))
#define RN_SQRT(a) __fsqrt_rn(a)
#else
#define RN_ADD(a, b) ((a) + (b))
#define RN_MUL(a, b) ((a) * (b))
#define RN_DIV(a, b) ((a) / (b))
#define RN_SQRT(a) sqrtf(a)
#endif

__host__ __device__ inline float bits_f32(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}
__host__ __device__ inline uint32_t f32_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

// ln u for normal u in (0, 1]
__host__ __device__ inline float ln_exact(float u) {
    const uint32_t b = f32_bits(u);
    int e = (int)(b >> 23) - 127;
    float m = bits_f32((b & 0x7FFFFFu) | 0x3F800000u);   // [1, 2)
    if (m > 0x1.6a09e6p+0f) {                            // sqrt(2)
        m = RN_MUL(m, 0.5f);
        e += 1;
    }
    const float t = RN_DIV(RN_ADD(m, -1.0f), RN_ADD(m, 1.0f));
    const float t2 = RN_MUL(t, t);
    float p = 0x1.3b13b2p-4f;                    // 1/13
    p = RN_ADD(0x1.745d18p-4f, RN_MUL(t2, p));   // 1/11
    p = RN_ADD(0x1.c71c72p-4f, RN_MUL(t2, p));   // 1/9
    p = RN_ADD(0x1.24924ap-3f, RN_MUL(t2, p));   // 1/7
    p = RN_ADD(0x1.99999ap-3f, RN_MUL(t2, p));   // 1/5
    p = RN_ADD(0x1.555556p-2f, RN_MUL(t2, p));   // 1/3
    const float lnm = RN_MUL(RN_ADD(t, RN_MUL(t, RN_MUL(t2, p))), 2.0f);
    return RN_ADD(RN_MUL((float)e, 0x1.62e43p-1f), lnm);   // ln 2
}

// cos(2 pi u) for u in [0, 1]
__host__ __device__ inline float cos2pi_exact(float u) {
    const float x = RN_MUL(u, 4.0f);
    const float q = rintf(x);
    const float r = RN_ADD(x, -q);   // exact, |r| <= 1/2
    const float r2 = RN_MUL(r, r);
    float c = -0x1.a6d1f2p-16f;                  // (-1)^k (pi/2)^2k / (2k)!, k = 5 .. 1, then 1
    c = RN_ADD(0x1.e1f506p-11f, RN_MUL(r2, c));
    c = RN_ADD(-0x1.55d3c8p-6f, RN_MUL(r2, c));
    c = RN_ADD(0x1.03c1f0p-2f, RN_MUL(r2, c));
    c = RN_ADD(-0x1.3bd3ccp+0f, RN_MUL(r2, c));
    c = RN_ADD(1.0f, RN_MUL(r2, c));
    float sn = -0x1.e3075p-19f;                  // (-1)^k (pi/2)^(2k+1) / (2k+1)!, k = 5 .. 0
    sn = RN_ADD(0x1.507834p-13f, RN_MUL(r2, sn));
    sn = RN_ADD(-0x1.32d2ccp-8f, RN_MUL(r2, sn));
    sn = RN_ADD(0x1.466bc6p-4f, RN_MUL(r2, sn));
    sn = RN_ADD(-0x1.4abbcep-1f, RN_MUL(r2, sn));
    sn = RN_ADD(0x1.921fb6p+0f, RN_MUL(r2, sn));
    sn = RN_MUL(r, sn);
    switch ((int)q & 3) {
        case 0: return c;
        case 1: return -sn;
        case 2: return -c;
        default: return sn;
    }
}

__host__ __device__ inline float normal_exact(uint32_t d0, uint32_t d1, float mean, float stdev) {
    const float u0 = RN_MUL(RN_ADD((float)d0, 0.5f), 0x1p-24f);
    const float u1 = RN_MUL(RN_ADD((float)d1, 0.5f), 0x1p-24f);
    const float z = RN_MUL(RN_SQRT(RN_MUL(-2.0f, ln_exact(u0))), cos2pi_exact(u1));
    return RN_ADD(mean, RN_MUL(stdev, z));
}

__global__ void k_fill_normal(__half *a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, float mean,
                              float stdev) {
    const uint64_t total = (uint64_t)rows * cols;
    const uint64_t start = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * kChunk;
    if (start >= total) return;
    const Affine j = lcg_jump(2 * start);
    uint32_t s = j.a * (seed ^ kSeedXor) + j.c;
    uint64_t r = start / cols, c = start - r * cols;
    const uint64_t end = start + kChunk < total ? start + kChunk : total;
    for (uint64_t i = start; i < end; ++i) {
        s = s * kA + kC;
        const uint32_t d0 = s >> 8;
        s = s * kA + kC;
        a[r * ld + c] = __float2half_rn(normal_exact(d0, s >> 8, mean, stdev));
        if (++c == cols) {
            c = 0;
            ++r;
        }
    }
}

// sub-block [row0.., col0..] of a global gcols-wide LCG matrix: element (r, c) is draw (row0 + r) * gcols + col0 + c
__global__ void k_fill_lcg_block(__half *a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, int lo,
                                 uint32_t span, float scale, uint64_t row0, uint64_t col0, uint64_t gcols) {
    const uint32_t chunks = (cols + kChunk - 1) / kChunk;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)rows * chunks) return;
    const uint32_t r = (uint32_t)(t / chunks), c0 = (uint32_t)(t - (uint64_t)r * chunks) * kChunk;
    const uint64_t start = (row0 + r) * gcols + col0 + c0;
    const Affine j = lcg_jump(start);
    uint32_t s = j.a * (seed ^ kSeedXor) + j.c;
    const uint32_t end = c0 + kChunk < cols ? c0 + kChunk : cols;
    for (uint32_t c = c0; c < end; ++c) {
        s = s * kA + kC;
        const int v = lo + (int)((s >> 8) % span);
        a[(size_t)r * ld + c] = __float2half_rn((float)v * scale);
    }
}

__global__ void k_fill_parity(uint16_t *a, uint32_t rows, uint32_t cols, uint32_t ld, uint16_t even, uint16_t odd) {
    const uint64_t total = (uint64_t)rows * cols;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / cols, c = i - r * cols;
        a[r * ld + c] = (c & 1) ? odd : even;
    }
}

uint32_t host_lcg(uint32_t *s) {
    *s = *s * kA + kC;
    return *s >> 8;
}

bool read_elem(uint64_t a, uint64_t idx, uint16_t *out) {
    return sh::cuda_ok(cudaMemcpy(out, (const void *)(a + idx * 2), 2, cudaMemcpyDeviceToHost), "sh_test read");
}

}  // namespace

extern "C" {

float sh_fp16_to_f32(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

uint16_t sh_f32_to_fp16(float f) {   // round to nearest even, like the reference's software conversion
    __half_raw r = __half_raw(__float2half_rn(f));
    return r.x;
}

void sh_test_fill_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, int lo, int hi,
                       float scale) {
    if (rows == 0 || cols == 0) return;
    const uint64_t total = (uint64_t)rows * cols;
    const uint64_t threads = (total + kChunk - 1) / kChunk;
    const uint32_t grid = (uint32_t)((threads + 255) / 256);
    k_fill_lcg<<<grid, 256, 0, sh::stream()>>>((__half *)a, rows, cols, ld, seed, lo, (uint32_t)(hi - lo + 1), scale);
    sh::cuda_ok(cudaGetLastError(), "sh_test_fill_fp16");
}

void sh_cuda_fill_normal_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, float mean,
                              float stdev) {
    if (rows == 0 || cols == 0) return;
    const uint64_t total = (uint64_t)rows * cols;
    const uint64_t threads = (total + kChunk - 1) / kChunk;
    const uint32_t grid = (uint32_t)((threads + 255) / 256);
    k_fill_normal<<<grid, 256, 0, sh::stream()>>>((__half *)a, rows, cols, ld, seed, mean, stdev);
    sh::cuda_ok(cudaGetLastError(), "sh_cuda_fill_normal_fp16");
}

void sh_cuda_host_fill_normal_fp16(uint16_t *dst, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, float mean,
                                   float stdev) {
    if (!dst) return;
    uint32_t s = seed ^ kSeedXor;
    for (uint32_t r = 0; r < rows; ++r)
        for (uint32_t c = 0; c < cols; ++c) {
            const uint32_t d0 = host_lcg(&s);
            const uint32_t d1 = host_lcg(&s);
            dst[(size_t)r * ld + c] = sh_f32_to_fp16(normal_exact(d0, d1, mean, stdev));
        }
}

void sh_cuda_fill_lcg_block(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, int lo, int hi,
                            float scale, uint64_t row0, uint64_t col0, uint64_t gcols) {
    if (rows == 0 || cols == 0) return;
    const uint64_t threads = (uint64_t)rows * ((cols + kChunk - 1) / kChunk);
    const uint32_t grid = (uint32_t)((threads + 255) / 256);
    k_fill_lcg_block<<<grid, 256, 0, sh::stream()>>>((__half *)a, rows, cols, ld, seed, lo, (uint32_t)(hi - lo + 1),
                                                     scale, row0, col0, gcols);
    sh::cuda_ok(cudaGetLastError(), "sh_cuda_fill_lcg_block");
}

void sh_test_fill_int_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, int lo, int hi) {
    sh_test_fill_fp16(a, rows, cols, ld, seed, lo, hi, 1.0f);
}

void sh_test_fill_colparity_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t even, uint32_t odd) {
    if (rows == 0 || cols == 0) return;
    k_fill_parity<<<1024, 256, 0, sh::stream()>>>((uint16_t *)a, rows, cols, ld, (uint16_t)even, (uint16_t)odd);
    sh::cuda_ok(cudaGetLastError(), "sh_test_fill_colparity_fp16");
}

void sh_test_fill_const_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t bits) {
    sh_test_fill_colparity_fp16(a, rows, cols, ld, bits, bits);
}

void sh_test_dump_samples(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, uint32_t nsamples,
                          const char *tag) {
    if (!sh::cuda_ok(cudaStreamSynchronize(sh::stream()), "sh_test_dump_samples")) return;
    uint32_t s = seed ^ kSeedXor;
    for (uint32_t n = 0; n < nsamples; ++n) {
        const uint32_t i = host_lcg(&s) % rows, j = host_lcg(&s) % cols;
        uint16_t v = 0;
        if (!read_elem(a, (uint64_t)i * ld + j, &v)) return;
        printf("%s %u %u %04x\n", tag, i, j, (uint32_t)v);
    }
    fflush(stdout);
}

void sh_test_dump_samples_idx(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, uint32_t nsamples,
                              const char *tag, uint32_t idx) {
    char t[64];
    snprintf(t, sizeof t, "%s%u", tag, idx);
    sh_test_dump_samples(a, rows, cols, ld, seed, nsamples, t);
}

uint32_t sh_test_check_gemm(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx,
                            uint32_t ldw, uint32_t ldz, uint32_t nsamples, float tol, float z0, const char *tag) {
    if (!sh::cuda_ok(cudaStreamSynchronize(sh::stream()), "sh_test_check_gemm")) return nsamples;
    uint32_t s = 0xC0FFEEu, bad = 0;
    float maxdiff = 0.f;
    std::vector<uint16_t> xr(K), wc(K);
    for (uint32_t n = 0; n < nsamples; ++n) {
        const uint32_t i = (n * 7919u + host_lcg(&s)) % M, j = (n * 104729u + host_lcg(&s)) % N;
        if (!sh::cuda_ok(cudaMemcpy(xr.data(), (const void *)(x + (uint64_t)i * ldx * 2), K * 2, cudaMemcpyDeviceToHost),
                         "sh_test_check_gemm") ||
            !sh::cuda_ok(cudaMemcpy2D(wc.data(), 2, (const void *)(w + (uint64_t)j * 2), (size_t)ldw * 2, 2, K,
                                      cudaMemcpyDeviceToHost),
                         "sh_test_check_gemm"))
            return nsamples;
        float acc = z0;
        for (uint32_t k = 0; k < K; ++k) acc += sh_fp16_to_f32(xr[k]) * sh_fp16_to_f32(wc[k]);
        uint16_t zv = 0;
        if (!read_elem(z, (uint64_t)i * ldz + j, &zv)) return nsamples;
        const float got = sh_fp16_to_f32(zv);
        const float d = fabsf(got - acc);
        if (d > maxdiff) maxdiff = d;
        if (d > tol) {
            if (bad < 4) printf("  mismatch z[%u,%u] got %f want %f\n", i, j, got, acc);
            ++bad;
        }
    }
    printf("%s samples=%u bad=%u maxdiff=%f %s\n", tag, nsamples, bad, maxdiff, bad ? "FAIL" : "PASS");
    fflush(stdout);
    return bad;
}

uint32_t sh_test_check_const_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t bits, uint32_t tol,
                                  const char *tag) {
    if (!sh::cuda_ok(cudaStreamSynchronize(sh::stream()), "sh_test_check_const_fp16")) return 0;
    std::vector<uint16_t> h((size_t)rows * cols);
    if (rows && cols &&
        !sh::cuda_ok(cudaMemcpy2D(h.data(), (size_t)cols * 2, (const void *)a, (size_t)ld * 2, (size_t)cols * 2, rows,
                                  cudaMemcpyDeviceToHost),
                     "sh_test_check_const_fp16"))
        return 0;
    uint32_t ok = 0;
    for (size_t i = 0; i < h.size(); ++i) {
        int d = (int)h[i] - (int)bits;
        if (d < 0) d = -d;
        if ((uint32_t)d <= tol) ++ok;
    }
    printf("%s_CHECK ok=%u/%u %s_%s\n", tag, ok, rows * cols, tag, ok == rows * cols ? "PASS" : "FAIL");
    fflush(stdout);
    return ok;
}

}  // extern "C"
