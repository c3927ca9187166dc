// Row-wise / elementwise fp16 ops on HBM tensors (reference: runtime/sh_rowops.inc.c:383-465, declared at
// runtime/sh_ops.h:94-100).
//
// The reference stages row blocks through a cluster's TCDM and computes in fp16 SIMD lanes. Here every op is
// one pass over HBM: row ops (layernorm, softmax) give one warp a whole row held in registers (8 fp16 per
// 16-byte vector, up to 4096 columns), reduce with warp shuffles in fp32 and store fp16 RNE; elementwise
// ops stream 16-byte vectors with a grid sized to the SM count. Anything not 16-byte aligned (views with odd
// element offsets, cols % 8 != 0) takes an element-wise path with the same arithmetic.
#include "sh_internal.cuh"

namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kMaxVecPerLane = 16;   // 16 x 8 x 32 = 4096 columns in registers

struct Vec8 {
    float v[8];
};

__device__ __forceinline__ Vec8 load8(const __half *p) {
    uint4 raw = *reinterpret_cast<const uint4 *>(p);
    const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
    Vec8 r;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        r.v[2 * i] = f.x;
        r.v[2 * i + 1] = f.y;
    }
    return r;
}
__device__ __forceinline__ void store8(__half *p, const Vec8 &a) {
    uint4 raw;
    __half2 *h = reinterpret_cast<__half2 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(a.v[2 * i], a.v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(p) = raw;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---- layernorm (optionally fused with the residual add h = a + b) -------------------------------------
// The row stays in registers as fp16 (4 registers per 8 columns) and is converted on each of the three uses, so the
// kernel fits 40 registers and 6 blocks (48 rows in flight) per SM for rows up to 1024 columns: more loads in
// flight, which matters where the power cap holds the SM clock low.
__device__ __forceinline__ float sum8(const uint4 &raw) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        s += f.x + f.y;
    }
    return s;
}
__device__ __forceinline__ float sqdev8(const uint4 &raw, float mean) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        q = fmaf(f.x - mean, f.x - mean, q);
        q = fmaf(f.y - mean, f.y - mean, q);
    }
    return q;
}

// sum over the LPR lanes of a row group (LPR = 32: the warp; 16: each half-warp), every lane taking part
template <int LPR>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = LPR / 2; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Two rows per warp (LPR = 16 lanes per row) for 528-768 columns: each lane holds six 16-byte vectors of its row, as
// many bytes as the warp-per-row kernel's three, so 64 rows are in flight per SM instead of 48. Blocks of four warps
// (8 K registers) fit beside a running GEMM CTA, so with programmatic dependent launch one waits on every SM.
constexpr uint32_t kHwWarps = 4;
template <int VPL, bool ADD, int LPR = 16>
__global__ void __launch_bounds__(kHwWarps * 32, 8)
    k_layernorm_hw(__half *y, __half *h, const __half *a, const __half *b, const __half *g, const __half *be,
                    uint32_t rows, uint32_t cols, uint32_t ld, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t sub = lane % LPR;
    const uint32_t row = (blockIdx.x * kHwWarps + (threadIdx.x >> 5)) * (32 / LPR) + lane / LPR;
    // (a half-warp whose row is past the end still takes part in the shuffles)
    const bool live = row < rows;
    const uint32_t cv = cols >> 3;
    const __half *ar = a + (size_t)row * ld;
    uint4 x[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t v = sub + LPR * i;
        x[i] = make_uint4(0u, 0u, 0u, 0u);
        if (live && v < cv) x[i] = *reinterpret_cast<const uint4 *>(ar + 8 * v);
    }
    if (ADD) {   // h = fp16(a + b), stored, and normalised below
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const uint32_t v = sub + LPR * i;
            if (live && v < cv) {
                const uint4 bb = *reinterpret_cast<const uint4 *>(b + (size_t)row * ld + 8 * v);
                __half2 *xh = reinterpret_cast<__half2 *>(&x[i]);
                const __half2 *bh = reinterpret_cast<const __half2 *>(&bb);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 fa = __half22float2(xh[j]), fb = __half22float2(bh[j]);
                    xh[j] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
                }
                *reinterpret_cast<uint4 *>(h + (size_t)row * ld + 8 * v) = x[i];
            }
        }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) s += sum8(x[i]);   // zero vectors past the row add nothing
    const float inv_cols = 1.f / (float)cols;
    const float mean = group_sum<LPR>(s) * inv_cols;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
        if (sub + LPR * i < cv) q += sqdev8(x[i], mean);
    const float rstd = rsqrtf(group_sum<LPR>(q) * inv_cols + eps);
    __half *yr = y + (size_t)row * ld;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t v = sub + LPR * i;
        if (live && v < cv) {
            const uint4 gr = *reinterpret_cast<const uint4 *>(g + 8 * v), br = *reinterpret_cast<const uint4 *>(be + 8 * v);
            const __half2 *xh = reinterpret_cast<const __half2 *>(&x[i]), *gh = reinterpret_cast<const __half2 *>(&gr),
                          *bh = reinterpret_cast<const __half2 *>(&br);
            uint4 o;
            __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 fx = __half22float2(xh[j]), fg = __half22float2(gh[j]), fb = __half22float2(bh[j]);
                oh[j] = __floats2half2_rn((fx.x - mean) * rstd * fg.x + fb.x, (fx.y - mean) * rstd * fg.y + fb.y);
            }
            *reinterpret_cast<uint4 *>(yr + 8 * v) = o;
        }
    }
}

template <int VPL, bool ADD>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, VPL <= 4 ? 6 : 1) k_layernorm_vec(__half *y, __half *h, const __half *a,
                                                                          const __half *b, const __half *g,
                                                                          const __half *be, uint32_t rows,
                                                                          uint32_t cols, uint32_t ld, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
    if (row >= rows) return;
    const uint32_t cv = cols >> 3;
    const __half *ar = a + (size_t)row * ld;
    uint4 x[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t v = lane + 32 * i;
        x[i] = make_uint4(0u, 0u, 0u, 0u);
        if (v < cv) x[i] = *reinterpret_cast<const uint4 *>(ar + 8 * v);
    }
    if (ADD) {   // h = fp16(a + b), stored, and normalised below
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const uint32_t v = lane + 32 * i;
            if (v < cv) {
                const uint4 bb = *reinterpret_cast<const uint4 *>(b + (size_t)row * ld + 8 * v);
                __half2 *xh = reinterpret_cast<__half2 *>(&x[i]);
                const __half2 *bh = reinterpret_cast<const __half2 *>(&bb);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 fa = __half22float2(xh[j]), fb = __half22float2(bh[j]);
                    xh[j] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
                }
                *reinterpret_cast<uint4 *>(h + (size_t)row * ld + 8 * v) = x[i];
            }
        }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) s += sum8(x[i]);   // zero vectors past the row add nothing
    const float inv_cols = 1.f / (float)cols;
    const float mean = warp_sum(s) * inv_cols;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
        if (lane + 32 * i < cv) q += sqdev8(x[i], mean);
    const float rstd = rsqrtf(warp_sum(q) * inv_cols + eps);
    __half *yr = y + (size_t)row * ld;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t v = lane + 32 * i;
        if (v < cv) {
            const uint4 gr = *reinterpret_cast<const uint4 *>(g + 8 * v), br = *reinterpret_cast<const uint4 *>(be + 8 * v);
            const __half2 *xh = reinterpret_cast<const __half2 *>(&x[i]), *gh = reinterpret_cast<const __half2 *>(&gr),
                          *bh = reinterpret_cast<const __half2 *>(&br);
            uint4 o;
            __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 fx = __half22float2(xh[j]), fg = __half22float2(gh[j]), fb = __half22float2(bh[j]);
                oh[j] = __floats2half2_rn((fx.x - mean) * rstd * fg.x + fb.x, (fx.y - mean) * rstd * fg.y + fb.y);
            }
            *reinterpret_cast<uint4 *>(yr + 8 * v) = o;
        }
    }
}

// element-wise fallback: one warp per row, three passes over global memory (L1/L2 resident)
template <bool ADD>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) k_layernorm_any(__half *y, __half *h, const __half *a,
                                                                       const __half *b, const __half *g,
                                                                       const __half *be, uint32_t rows, uint32_t cols,
                                                                       uint32_t ld, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
    if (row >= rows) return;
    const __half *ar = a + (size_t)row * ld;
    const __half *br = ADD ? b + (size_t)row * ld : nullptr;
    __half *hr = ADD ? h + (size_t)row * ld : nullptr;
    auto xin = [&](uint32_t c) -> float {
        if (ADD) return __half2float(__float2half_rn(__half2float(ar[c]) + __half2float(br[c])));
        return __half2float(ar[c]);
    };
    float s = 0.f;
    for (uint32_t c = lane; c < cols; c += 32) s += xin(c);
    const float mean = warp_sum(s) / (float)cols;
    float q = 0.f;
    for (uint32_t c = lane; c < cols; c += 32) {
        const float d = xin(c) - mean;
        q += d * d;
    }
    const float rstd = rsqrtf(warp_sum(q) / (float)cols + eps);
    __syncwarp();
    __half *yr = y + (size_t)row * ld;
    for (uint32_t c = lane; c < cols; c += 32) {
        const float xv = xin(c);
        if (ADD) hr[c] = __float2half_rn(xv);
        yr[c] = __float2half_rn((xv - mean) * rstd * __half2float(g[c]) + __half2float(be[c]));
    }
}

// ---- softmax(scale x) per row -----------------------------------------------------------------------------
template <int VPL>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) k_softmax_vec(__half *y, const __half *x, uint32_t rows,
                                                                     uint32_t cols, uint32_t ld, float scale) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
    if (row >= rows) return;
    const uint32_t cv = cols >> 3;
    const float s2 = scale * 1.4426950408889634f;   // work in the log2 domain: e^(s x) = 2^(s log2(e) x)
    Vec8 t[VPL];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t v = lane + 32 * i;
        if (v < cv) {
            t[i] = load8(x + (size_t)row * ld + 8 * v);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                t[i].v[j] *= s2;
                m = fmaxf(m, t[i].v[j]);
            }
        }
    }
    m = warp_max(m);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        if (lane + 32 * i < cv) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                t[i].v[j] = fast_exp2(t[i].v[j] - m);
                sum += t[i].v[j];
            }
        }
    }
    const float inv = 1.f / warp_sum(sum);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t v = lane + 32 * i;
        if (v < cv) {
#pragma unroll
            for (int j = 0; j < 8; ++j) t[i].v[j] *= inv;
            store8(y + (size_t)row * ld + 8 * v, t[i]);
        }
    }
}

__global__ void __launch_bounds__(kWarpsPerBlock * 32) k_softmax_any(__half *y, const __half *x, uint32_t rows,
                                                                     uint32_t cols, uint32_t ld, float scale) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float s2 = scale * 1.4426950408889634f;
    const __half *xr = x + (size_t)row * ld;
    float m = -INFINITY;
    for (uint32_t c = lane; c < cols; c += 32) m = fmaxf(m, __half2float(xr[c]) * s2);
    m = warp_max(m);
    float sum = 0.f;
    for (uint32_t c = lane; c < cols; c += 32) sum += exp2f(__half2float(xr[c]) * s2 - m);
    const float inv = 1.f / warp_sum(sum);
    __syncwarp();
    __half *yr = y + (size_t)row * ld;
    for (uint32_t c = lane; c < cols; c += 32) yr[c] = __float2half_rn(exp2f(__half2float(xr[c]) * s2 - m) * inv);
}

// ---- wide rows (cols > 1024): one CTA of kRowThreads per row, the row in registers, block reductions ----------
constexpr int kRowThreads = 128;

template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = (l < NT / 32) ? red[l] : 0.f;
    return warp_sum(t);
}
template <int NT>
__device__ __forceinline__ float block_max(float v, float *red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = (l < NT / 32) ? red[l] : -INFINITY;
    return warp_max(t);
}

template <int VPT, bool ADD>
__global__ void __launch_bounds__(kRowThreads) k_layernorm_row(__half *y, __half *h, const __half *a, const __half *b,
                                                               const __half *g, const __half *be, uint32_t cols,
                                                               uint32_t ld, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float red[kRowThreads / 32];
    const size_t row = blockIdx.x;
    const uint32_t cv = cols >> 3;
    Vec8 x[VPT];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const uint32_t v = threadIdx.x + kRowThreads * i;
        if (v < cv) {
            x[i] = load8(a + row * ld + 8 * v);
            if (ADD) {
                Vec8 bb = load8(b + row * ld + 8 * v);
#pragma unroll
                for (int j = 0; j < 8; ++j) x[i].v[j] = __half2float(__float2half_rn(x[i].v[j] + bb.v[j]));
                store8(h + row * ld + 8 * v, x[i]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) s += x[i].v[j];
        }
    }
    const float mean = block_sum<kRowThreads>(s, red) / (float)cols;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
        if (threadIdx.x + kRowThreads * i < cv) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float d = x[i].v[j] - mean;
                q += d * d;
            }
        }
    const float rstd = rsqrtf(block_sum<kRowThreads>(q, red) / (float)cols + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const uint32_t v = threadIdx.x + kRowThreads * i;
        if (v < cv) {
            Vec8 gg = load8(g + 8 * v), bb = load8(be + 8 * v), o;
#pragma unroll
            for (int j = 0; j < 8; ++j) o.v[j] = (x[i].v[j] - mean) * rstd * gg.v[j] + bb.v[j];
            store8(y + row * ld + 8 * v, o);
        }
    }
}

template <int VPT, int NT = kRowThreads>
__global__ void __launch_bounds__(NT) k_softmax_row(__half *y, const __half *x, uint32_t cols, uint32_t ld,
                                                    float scale) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float red[kRowThreads / 32];
    const size_t row = blockIdx.x;
    const uint32_t cv = cols >> 3;
    const float s2 = scale * 1.4426950408889634f;
    Vec8 t[VPT];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const uint32_t v = threadIdx.x + NT * i;
        if (v < cv) {
            t[i] = load8(x + row * ld + 8 * v);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                t[i].v[j] *= s2;
                m = fmaxf(m, t[i].v[j]);
            }
        }
    }
    m = block_max<NT>(m, red);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
        if (threadIdx.x + NT * i < cv) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                t[i].v[j] = fast_exp2(t[i].v[j] - m);
                sum += t[i].v[j];
            }
        }
    const float inv = 1.f / block_sum<NT>(sum, red);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const uint32_t v = threadIdx.x + NT * i;
        if (v < cv) {
#pragma unroll
            for (int j = 0; j < 8; ++j) t[i].v[j] *= inv;
            store8(y + row * ld + 8 * v, t[i]);
        }
    }
}

// ---- elementwise ---------------------------------------------------------------------------------------------
enum EwOp : int { kGelu = 0, kAdd = 1, kBias = 2, kScale = 3 };

template <int OP>
__device__ __forceinline__ float ew_apply(float x, float b, float s) {
    if (OP == kGelu) return gelu_fast(x);
    if (OP == kAdd || OP == kBias) return x + b;
    return x * s;
}

// rows x cv vectors; `ld` multiple of 8; 64-bit flat index over the vectors
template <int OP>
__global__ void k_ew_vec(__half *y, const __half *x, const __half *b, uint32_t rows, uint32_t cv, uint32_t ld,
                         float s) {
    pdl_launch_dependents();
    pdl_wait();
    const uint64_t total = (uint64_t)rows * cv;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / cv, c = i - r * cv;
        const size_t off = r * ld + 8 * c;
        Vec8 a = load8(x + off), bb;
        if (OP == kAdd) bb = load8(b + off);
        if (OP == kBias) bb = load8(b + 8 * c);
#pragma unroll
        for (int j = 0; j < 8; ++j) a.v[j] = ew_apply<OP>(a.v[j], (OP == kAdd || OP == kBias) ? bb.v[j] : 0.f, s);
        store8(y + off, a);
    }
}

template <int OP>
__global__ void k_ew_any(__half *y, const __half *x, const __half *b, uint32_t rows, uint32_t cols, uint32_t ld,
                         float s) {
    pdl_launch_dependents();
    pdl_wait();
    const uint64_t total = (uint64_t)rows * cols;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / cols, c = i - r * cols;
        const size_t off = r * ld + c;
        float bv = 0.f;
        if (OP == kAdd) bv = __half2float(b[off]);
        if (OP == kBias) bv = __half2float(b[c]);
        y[off] = __float2half_rn(ew_apply<OP>(__half2float(x[off]), bv, s));
    }
}

// ---- transpose: 64 x 64 tiles through shared memory (bit-exact data movement) ------------------------------------
constexpr int TT = 64;

// Full aligned tiles: the tile is kept transposed in shared memory as 32-bit pairs, tT[c][p] = (x[2p][c], x[2p+1][c]),
// 32 words per source column, the 16-byte groups of each row XOR-swizzled by (c % 8). Warp w loads 16-byte chunk w of
// rows 2p, 2p+1 (p = lane) and writes 8 pair words (conflict-free: one row c per instruction, 32 consecutive p);
// the store phase reads 16-byte groups (8 source rows) and writes them as one vector of an output row.
__global__ void __launch_bounds__(256) k_transpose_pairs(__half *dst, const __half *src, uint32_t rows, uint32_t cols,
                                                         uint32_t ld_src, uint32_t ld_dst) {
    __shared__ __align__(16) uint32_t tT[TT * 32];
    const uint32_t r0 = blockIdx.y * TT, c0 = blockIdx.x * TT;
    const uint16_t *s16 = reinterpret_cast<const uint16_t *>(src);
    uint16_t *d16 = reinterpret_cast<uint16_t *>(dst);
    const uint32_t p = threadIdx.x & 31, q = threadIdx.x >> 5;   // row pair, 16-byte chunk (8 columns)
    const uint4 a = *reinterpret_cast<const uint4 *>(s16 + (size_t)(r0 + 2 * p) * ld_src + c0 + 8 * q);
    const uint4 b = *reinterpret_cast<const uint4 *>(s16 + (size_t)(r0 + 2 * p + 1) * ld_src + c0 + 8 * q);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t c = 8 * q + k;
        const uint32_t lo = (k & 1) ? (aw[k >> 1] >> 16) : (aw[k >> 1] & 0xFFFFu);
        const uint32_t hi = (k & 1) ? (bw[k >> 1] >> 16) : (bw[k >> 1] & 0xFFFFu);
        tT[c * 32 + (((p >> 2) ^ (c & 7)) << 2) + (p & 3)] = lo | (hi << 16);
    }
    __syncthreads();
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const uint32_t idx = threadIdx.x + 256 * it;
        const uint32_t c = idx >> 3, g = idx & 7;   // output row (source column), 16-byte group = 8 source rows
        const uint4 v = *reinterpret_cast<const uint4 *>(&tT[c * 32 + ((g ^ (c & 7)) << 2)]);
        *reinterpret_cast<uint4 *>(d16 + (size_t)(c0 + c) * ld_dst + r0 + 8 * g) = v;
    }
}
__global__ void __launch_bounds__(256) k_transpose(__half *dst, const __half *src, uint32_t rows, uint32_t cols,
                                                   uint32_t ld_src, uint32_t ld_dst, int vec) {
    __shared__ uint16_t tile[TT][TT + 2];
    const uint32_t r0 = blockIdx.y * TT, c0 = blockIdx.x * TT;
    const uint16_t *s16 = reinterpret_cast<const uint16_t *>(src);
    uint16_t *d16 = reinterpret_cast<uint16_t *>(dst);
    const bool full = (r0 + TT <= rows) && (c0 + TT <= cols);
    if (full && vec) {
        // 64 rows x 8 vectors of 8 elements: 512 vectors, 2 per thread
        for (int i = threadIdx.x; i < TT * 8; i += 256) {
            const int r = i >> 3, cv = i & 7;
            uint4 raw = *reinterpret_cast<const uint4 *>(s16 + (size_t)(r0 + r) * ld_src + c0 + 8 * cv);
            const uint16_t *e = reinterpret_cast<const uint16_t *>(&raw);
#pragma unroll
            for (int j = 0; j < 8; ++j) tile[r][8 * cv + j] = e[j];
        }
        __syncthreads();
        for (int i = threadIdx.x; i < TT * 8; i += 256) {
            const int c = i >> 3, rv = i & 7;   // output row c (a source column), 8 source rows
            uint4 raw;
            uint16_t *e = reinterpret_cast<uint16_t *>(&raw);
#pragma unroll
            for (int j = 0; j < 8; ++j) e[j] = tile[8 * rv + j][c];
            *reinterpret_cast<uint4 *>(d16 + (size_t)(c0 + c) * ld_dst + r0 + 8 * rv) = raw;
        }
    } else {
        for (int i = threadIdx.x; i < TT * TT; i += 256) {
            const uint32_t r = i / TT, c = i % TT;
            if (r0 + r < rows && c0 + c < cols) tile[r][c] = s16[(size_t)(r0 + r) * ld_src + c0 + c];
        }
        __syncthreads();
        for (int i = threadIdx.x; i < TT * TT; i += 256) {
            const uint32_t c = i / TT, r = i % TT;   // consecutive threads: consecutive source rows
            if (r0 + r < rows && c0 + c < cols) d16[(size_t)(c0 + c) * ld_dst + r0 + r] = tile[r][c];
        }
    }
}

inline bool vec_ok(uint64_t p, uint32_t ld) { return sh::aligned16(p) && (ld % 8 == 0); }

inline uint32_t ew_grid(uint64_t work, int threads) {
    const uint64_t want = (work + threads - 1) / threads;
    const uint64_t cap = (uint64_t)sh::state().num_sms * 16;
    return (uint32_t)(want < cap ? (want ? want : 1) : cap);
}

template <int OP>
void launch_ew(uint64_t y, uint64_t x, uint64_t b, uint32_t rows, uint32_t cols, uint32_t ld, float s,
               const char *name) {
    if (rows == 0 || cols == 0) return;
    if (cols > ld) {
        sh::set_error(-1, "[%s] cols %u > ld %u", name, cols, ld);
        return;
    }
    cudaStream_t st = sh::stream();
    bool vec = (cols % 8 == 0) && vec_ok(y, ld) && vec_ok(x, ld);
    if (OP == kAdd) vec = vec && vec_ok(b, ld);
    if (OP == kBias) vec = vec && sh::aligned16(b);
    if (vec) {
        const uint32_t cv = cols / 8;
        sh::launch_pdl(k_ew_vec<OP>, dim3(ew_grid((uint64_t)rows * cv, 256)), dim3(256), 0, st, (__half *)y, (const __half *)x,
                                                                        (const __half *)b, rows, cv, ld, s);
    } else {
        sh::launch_pdl(k_ew_any<OP>, dim3(ew_grid((uint64_t)rows * cols, 256)), dim3(256), 0, st, (__half *)y, (const __half *)x,
                                                                          (const __half *)b, rows, cols, ld, s);
    }
    sh::cuda_ok(cudaGetLastError(), name);
}

template <bool ADD, int VPL, int LPR = 32>
void ln_vec_launch(uint64_t y, uint64_t h, uint64_t a, uint64_t b, uint64_t g, uint64_t be, uint32_t rows,
                   uint32_t cols, uint32_t ld, float eps, cudaStream_t st) {
    const uint32_t warps = LPR == 32 ? kWarpsPerBlock : kHwWarps;
    const uint32_t rows_per_block = warps * (32 / LPR);
    const uint32_t grid = (rows + rows_per_block - 1) / rows_per_block;
    if constexpr (LPR == 32)
        sh::launch_pdl(k_layernorm_vec<VPL, ADD>, dim3(grid), dim3(warps * 32), 0, st, (__half *)y,
                       (__half *)h, (const __half *)a, (const __half *)b, (const __half *)g, (const __half *)be, rows,
                       cols, ld, eps);
    else
        sh::launch_pdl(k_layernorm_hw<VPL, ADD, LPR>, dim3(grid), dim3(warps * 32), 0, st, (__half *)y,
                       (__half *)h, (const __half *)a, (const __half *)b, (const __half *)g, (const __half *)be, rows,
                       cols, ld, eps);
}

template <bool ADD>
void launch_layernorm(uint64_t y, uint64_t h, uint64_t a, uint64_t b, uint64_t g, uint64_t be, uint32_t rows,
                      uint32_t cols, uint32_t ld, float eps, const char *name) {
    if (rows == 0 || cols == 0) return;
    if (cols > ld) {
        sh::set_error(-1, "[%s] cols %u > ld %u", name, cols, ld);
        return;
    }
    cudaStream_t st = sh::stream();
    bool vec = cols % 8 == 0 && cols <= 32u * 8u * kMaxVecPerLane && vec_ok(y, ld) && vec_ok(a, ld) &&
               sh::aligned16(g) && sh::aligned16(be);
    if (ADD) vec = vec && vec_ok(h, ld) && vec_ok(b, ld);
    if (vec && cols > 1024) {
        const uint32_t vpt = (cols / 8 + kRowThreads - 1) / kRowThreads;   // 2..4 vectors per thread
#define SH_LNR(n) \
    sh::launch_pdl(k_layernorm_row<n, ADD>, dim3(rows), dim3(kRowThreads), 0, st, (__half *)y, (__half *)h, (const __half *)a, \
                                                         (const __half *)b, (const __half *)g, (const __half *)be, cols, ld, eps)
        if (vpt <= 2) SH_LNR(2); else if (vpt <= 3) SH_LNR(3); else SH_LNR(4);
#undef SH_LNR
    } else if (vec && cols > 512 && cols <= 768) {   // two rows per warp, six vectors per lane
        ln_vec_launch<ADD, 6, 16>(y, h, a, b, g, be, rows, cols, ld, eps, st);
    } else if (vec) {
        const int vpl = (int)((cols / 8 + 31) / 32);
        switch (vpl) {
#define SH_LN_CASE(n) \
    case n: ln_vec_launch<ADD, n>(y, h, a, b, g, be, rows, cols, ld, eps, st); break;
            SH_LN_CASE(1) SH_LN_CASE(2) SH_LN_CASE(3) SH_LN_CASE(4) SH_LN_CASE(5) SH_LN_CASE(6) SH_LN_CASE(7)
            SH_LN_CASE(8) SH_LN_CASE(9) SH_LN_CASE(10) SH_LN_CASE(11) SH_LN_CASE(12) SH_LN_CASE(13) SH_LN_CASE(14)
            SH_LN_CASE(15) SH_LN_CASE(16)
#undef SH_LN_CASE
            default: break;
        }
    } else {
        const uint32_t grid = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
        sh::launch_pdl(k_layernorm_any<ADD>, dim3(grid), dim3(kWarpsPerBlock * 32), 0, st, (__half *)y, (__half *)h, (const __half *)a,
                                                                   (const __half *)b, (const __half *)g,
                                                                   (const __half *)be, rows, cols, ld, eps);
    }
    sh::cuda_ok(cudaGetLastError(), name);
}

template <int VPL>
void sm_vec_launch(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, float scale, cudaStream_t st) {
    const uint32_t grid = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
    sh::launch_pdl(k_softmax_vec<VPL>, dim3(grid), dim3(kWarpsPerBlock * 32), 0, st, (__half *)y, (const __half *)x, rows, cols, ld, scale);
}

}  // namespace

namespace {

// (sum, sum of squares) of each 64-column group of a row (one thread per group; the format sh_cuda_gemm_ln reads)
__global__ void __launch_bounds__(256) k_row_stats(const __half *x, uint32_t rows, uint32_t parts, uint32_t ld,
                                                   float2 *out) {
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)rows * parts) return;
    const uint32_t r = (uint32_t)(t / parts), g = (uint32_t)(t % parts);
    const uint4 *p = reinterpret_cast<const uint4 *>(x + (size_t)r * ld + (size_t)g * 64);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 u = __ldg(p + i);
        const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h[j]);
            s1 += f.x + f.y;
            s2 = fmaf(f.x, f.x, fmaf(f.y, f.y, s2));
        }
    }
    out[t] = make_float2(s1, s2);
}

// dst[r, c] = src[r, c] * gamma[r] (fp16)
__global__ void __launch_bounds__(256) k_scale_rows(__half *dst, const __half *src, uint32_t rows, uint32_t cols,
                                                    uint32_t lds, uint32_t ldd, const __half *gamma) {
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (uint64_t)rows * cols) return;
    const uint32_t r = (uint32_t)(t / cols), c = (uint32_t)(t % cols);
    dst[(size_t)r * ldd + c] = __float2half_rn(__half2float(src[(size_t)r * lds + c]) * __half2float(gamma[r]));
}

}  // namespace

extern "C" {

void sh_layernorm(uint64_t y, uint64_t x, uint64_t gamma, uint64_t beta, uint32_t rows, uint32_t cols, uint32_t ld,
                  float eps, uint32_t) {
    launch_layernorm<false>(y, 0, x, 0, gamma, beta, rows, cols, ld, eps, "sh_layernorm");
}

void sh_cuda_add_layernorm(uint64_t h, uint64_t y, uint64_t a, uint64_t b, uint64_t gamma, uint64_t beta,
                           uint32_t rows, uint32_t cols, uint32_t ld, float eps) {
    launch_layernorm<true>(y, h, a, b, gamma, beta, rows, cols, ld, eps, "sh_cuda_add_layernorm");
}

void sh_softmax_rows(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, float scale, uint32_t) {
    if (rows == 0 || cols == 0) return;
    if (cols > ld) {
        sh::set_error(-1, "[sh_softmax_rows] cols %u > ld %u", cols, ld);
        return;
    }
    cudaStream_t st = sh::stream();
    const bool vec = cols % 8 == 0 && cols <= 32u * 8u * kMaxVecPerLane && vec_ok(y, ld) && vec_ok(x, ld);
    if (vec && cols > 1024) {
        const uint32_t vpt = (cols / 8 + kRowThreads - 1) / kRowThreads;
#define SH_SMR(n) sh::launch_pdl(k_softmax_row<n>, dim3(rows), dim3(kRowThreads), 0, st, (__half *)y, (const __half *)x, cols, ld, scale)
        if (vpt <= 2) SH_SMR(2); else if (vpt <= 3) SH_SMR(3); else SH_SMR(4);
#undef SH_SMR
    } else if (vec) {
        switch ((int)((cols / 8 + 31) / 32)) {
#define SH_SM_CASE(n) \
    case n: sm_vec_launch<n>(y, x, rows, cols, ld, scale, st); break;
            SH_SM_CASE(1) SH_SM_CASE(2) SH_SM_CASE(3) SH_SM_CASE(4) SH_SM_CASE(5) SH_SM_CASE(6) SH_SM_CASE(7)
            SH_SM_CASE(8) SH_SM_CASE(9) SH_SM_CASE(10) SH_SM_CASE(11) SH_SM_CASE(12) SH_SM_CASE(13) SH_SM_CASE(14)
            SH_SM_CASE(15) SH_SM_CASE(16)
#undef SH_SM_CASE
            default: break;
        }
    } else {
        const uint32_t grid = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
        sh::launch_pdl(k_softmax_any, dim3(grid), dim3(kWarpsPerBlock * 32), 0, st, (__half *)y, (const __half *)x, rows, cols, ld, scale);
    }
    sh::cuda_ok(cudaGetLastError(), "sh_softmax_rows");
}

void sh_gelu(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t) {
    launch_ew<kGelu>(y, x, 0, rows, cols, ld, 0.f, "sh_gelu");
}
void sh_add(uint64_t y, uint64_t a, uint64_t b, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t) {
    launch_ew<kAdd>(y, a, b, rows, cols, ld, 0.f, "sh_add");
}
void sh_add_bias(uint64_t y, uint64_t x, uint64_t bias_row, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t) {
    launch_ew<kBias>(y, x, bias_row, rows, cols, ld, 0.f, "sh_add_bias");
}
void sh_scale(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, float s, uint32_t) {
    launch_ew<kScale>(y, x, 0, rows, cols, ld, s, "sh_scale");
}

void sh_transpose(uint64_t dst, uint64_t src, uint32_t rows, uint32_t cols, uint32_t ld_src, uint32_t ld_dst,
                  uint32_t) {
    if (rows == 0 || cols == 0) return;
    if (cols > ld_src || rows > ld_dst) {
        sh::set_error(-1, "[sh_transpose] %ux%u with ld_src %u ld_dst %u", rows, cols, ld_src, ld_dst);
        return;
    }
    const int vec = vec_ok(src, ld_src) && vec_ok(dst, ld_dst);
    if (vec && rows % TT == 0 && cols % TT == 0) {
        dim3 grid(cols / TT, rows / TT);
        k_transpose_pairs<<<grid, 256, 0, sh::stream()>>>((__half *)dst, (const __half *)src, rows, cols, ld_src,
                                                          ld_dst);
    } else {
        dim3 grid((cols + TT - 1) / TT, (rows + TT - 1) / TT);
        k_transpose<<<grid, 256, 0, sh::stream()>>>((__half *)dst, (const __half *)src, rows, cols, ld_src, ld_dst,
                                                    vec);
    }
    sh::cuda_ok(cudaGetLastError(), "sh_transpose");
}

int sh_cuda_row_stats(uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, uint64_t stats_out) {
    if (rows == 0) return 0;
    if (!x || !stats_out || cols % 64 || cols == 0 || ld < cols || !vec_ok(x, ld)) {
        sh::set_error(-1, "[sh_cuda_row_stats] %ux%u ld %u: need cols %% 64 == 0 and 16-byte aligned rows", rows,
                      cols, ld);
        return -1;
    }
    const uint64_t n = (uint64_t)rows * (cols / 64);
    k_row_stats<<<(unsigned)((n + 255) / 256), 256, 0, sh::stream()>>>((const __half *)x, rows, cols / 64, ld,
                                                                        (float2 *)stats_out);
    return sh::cuda_ok(cudaGetLastError(), "sh_cuda_row_stats") ? 0 : -1;
}

int sh_cuda_scale_rows(uint64_t dst, uint64_t src, uint32_t rows, uint32_t cols, uint32_t ld_src, uint32_t ld_dst,
                       uint64_t gamma) {
    if (rows == 0 || cols == 0) return 0;
    if (!dst || !src || !gamma || ld_src < cols || ld_dst < cols) {
        sh::set_error(-1, "[sh_cuda_scale_rows] %ux%u ld %u / %u", rows, cols, ld_src, ld_dst);
        return -1;
    }
    const uint64_t n = (uint64_t)rows * cols;
    k_scale_rows<<<(unsigned)((n + 255) / 256), 256, 0, sh::stream()>>>((__half *)dst, (const __half *)src, rows,
                                                                         cols, ld_src, ld_dst, (const __half *)gamma);
    return sh::cuda_ok(cudaGetLastError(), "sh_cuda_scale_rows") ? 0 : -1;
}

}  // extern "C"
