// GEMM of the operator library: Z[M,N] (+)= X[M,K] . W[K,N], fp16 in, fp32 accumulate, fp16 out
// (reference: runtime/sh_gemm.inc.c:17-117 sh_cfg_fill / sh_gemm_l1_bytes / sh_gemm, :127-189 sh_gemm_mesh,
// :192-344 sh_gemm_xmcast_ex; declared at runtime/sh_ops.h:54-88).
//
// The reference streams tm x tk / tk x tn tiles into TCDM and accumulates on RedMulE. Here persistent CTAs (one
// per SM, or one cluster of two per SM pair) run a warp-specialised tcgen05 pipeline:
//   warp 0     TMA producer: X tile [128 x 64] (K-major) and W tiles [64 x 64] (N-major, i.e. W as stored) per
//              stage into a ring of 128-byte-swizzled shared memory, completion on mbarriers;
//   warp 1     MMA issuer: the whole warp walks the issue loop and lane 0 issues tcgen05.mma into a tensor-memory
//              accumulator; tcgen05.commit frees each stage (in the 2-CTA kernel one commit signals both CTAs) and
//              publishes each finished accumulator;
//   warps 2-9  epilogue: tcgen05.ld the accumulator (warp w owns TMEM lane quarter w % 4 = 32 rows, and half of
//              the columns), apply the fused epilogue (accumulate / bias / GELU / residual / fp32 in or out) and
//              write fp16 through 32 x 32 staging tiles and TMA stores.
// k_gemm_tc<BN>: single CTA, 128 x BN tiles, two accumulators (the next tile's MMAs run while the epilogue drains),
//   split-K: fp32 partial tiles in a workspace, the last CTA of a tile (arrival counter) sums them in split order.
// k_gemm_tc2<BN>: a cluster of two CTAs, tcgen05.mma.cta_group::2 (M = 256), each CTA loading its half of the W
//   columns; BN = 256 with two accumulators, or BN = 512 (two N = 256 MMAs per k-step, one accumulator, 25 % fewer
//   operand bytes per MAC) for long K loops, whose short last wave may run as 256-column slices (pair_unit);
//   KS = 2 (BN = 256 without a residual, even k-block count): stages go in pairs that share one barrier.
// Tiles are taken in groups of row-tiles (tile_coords) so that concurrent CTAs share X and W in L2, and every launch
// uses programmatic dependent launch (set-up overlaps the previous kernel). The planner (make_plan, queryable as
// sh_cuda_gemm_plan) picks the kernel and tiling per shape.
// Every mbarrier wait is bounded (SH_SPIN_CYCLES): on a timeout the CTA raises the device error word, skips its
// remaining work, waits for its outstanding TMA loads and MMAs and frees its tensor memory.
// Shapes the TMA path cannot address (16-byte alignment of base or leading dimension) use a CUDA-core kernel.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <utility>

#include "sh_internal.cuh"

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kPairThreads = 352;   // the 2-CTA kernel adds warp 10: forwards the epilogue's "accumulator drained"
constexpr uint32_t kEpiWarps = 8;

constexpr uint32_t kEpiStageBytes = 8 * 4096;   // per epilogue warp: two 32 x 32 fp16 store tiles
constexpr uint32_t kGroupM = 8;                  // default row-tiles per group of the tile order

template <int BN>
struct TileCfg {
    static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
    static constexpr uint32_t kABytes = BM * BK * 2;
    static constexpr uint32_t kBBytes = BK * BN * 2;
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr uint32_t kTmemCols = 2 * BN;
    static constexpr uint32_t kSmem = kStages * kStageBytes + kEpiStageBytes + 1024 + 256;
};

struct GemmArgs {
    __half *z;
    const __half *bias;
    const __half *resid;
    uint32_t M, N, K, ldz, ldr, flags;
    uint32_t tiles_n, num_tiles, k_blocks, splits, kb_per_split;
    uint32_t group_m;    // tile order: row-tiles per group (tile_coords)
    uint32_t full_units, num_units;   // 2-CTA kernel: whole tiles below full_units, N-halves of the rest (pair_unit)
    uint32_t vec;        // epilogue may use 16-byte accesses on z / bias / resid
    uint32_t tma_store;  // fp16 Z written by TMA stores of 32 x 32 tiles staged in shared memory
    float *ws;
    uint32_t *counters;
    int *err;
    // LayerNorm folded into the GEMM (SH_EPI_LN_IN): X holds raw rows whose statistics arrive as ln_parts partial
    // (sum, sum of squares) pairs per row; t = rstd (acc - mean colsum[col]) before the bias
    const float2 *ln_stats;
    const float *ln_colsum;
    uint32_t ln_parts;
    float ln_eps;
    // SH_EPI_STATS_OUT: (sum, sum of squares) of each row's outputs per 64 columns, N / 64 pairs per row
    float2 *stats_out;
};

// Tile order of the persistent kernels: tiles are taken in groups of group_m row-tiles, and inside a group the
// column-tiles advance slowest. The CTAs that run at the same time then share a few row-blocks of X and a few
// column-blocks of W (each k-slice is fetched into L2 once per group), instead of sweeping every column-block of W
// once per wave when W is wider than L2 holds.
__device__ __forceinline__ void tile_coords(uint32_t tile, uint32_t tiles_m, uint32_t tiles_n, uint32_t group_m,
                                            uint32_t &tm, uint32_t &tn) {
    const uint32_t per_group = group_m * tiles_n;
    const uint32_t g = tile / per_group, first = g * group_m;
    const uint32_t gsz = min(group_m, tiles_m - first);
    const uint32_t w = tile - g * per_group;
    tm = first + w % gsz;
    tn = w / gsz;
}

// mean and 1 / sqrt(var + eps) of a row of K values from its partial sums (SH_EPI_LN_IN)
__device__ __forceinline__ float2 ln_row(const GemmArgs &a, uint32_t row) {
    if (!(a.flags & SH_EPI_LN_IN) || row >= a.M) return make_float2(0.f, 1.f);
    const float2 *p = a.ln_stats + (size_t)row * a.ln_parts;
    float s1[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (uint32_t i = 0; i < a.ln_parts; ++i) {
        const float2 q = p[i];
        s1[i & 3] += q.x;
        s2[i & 3] += q.y;
    }
    const float inv_k = 1.f / (float)a.K;
    const float mean = ((s1[0] + s1[1]) + (s1[2] + s1[3])) * inv_k;
    const float var = fmaxf(((s2[0] + s2[1]) + (s2[2] + s2[3])) * inv_k - mean * mean, 0.f);
    return make_float2(mean, rsqrtf(var + a.ln_eps));
}

// Barrier of the four epilogue warps on an mbarrier (count 4), so that it is bounded like every other wait.
__device__ __forceinline__ bool epi_sync(uint64_t *bar, uint32_t &phase, volatile int *abort, int *err) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    const bool ok = mbar_wait(bar, phase, abort, err);
    phase ^= 1u;
    __syncwarp();
    return ok;
}

// fused epilogue of 8 consecutive columns of one row (values in v, fp32). Z is fp16, or fp32 with SH_EPI_F32_OUT;
// SH_EPI_ACC_F32_IN adds an fp32 matrix passed as `resid` (leading dim ldr) instead of an fp16 residual.
__device__ __forceinline__ void epilogue8(const GemmArgs &a, uint32_t row, uint32_t col, float (&v)[8]) {
    if (row >= a.M || col >= a.N) return;
    const uint32_t f = a.flags;
    const bool z32 = (f & SH_EPI_F32_OUT) != 0;
    __half *zp = a.z + (size_t)row * a.ldz + col;
    float *zf = reinterpret_cast<float *>(a.z) + (size_t)row * a.ldz + col;
    const float *rf = reinterpret_cast<const float *>(a.resid) + (size_t)row * a.ldr + col;
    if (a.vec && col + 8 <= a.N) {
        if (f & SH_EPI_ACCUMULATE) {
            if (z32) {
                const float4 p0 = reinterpret_cast<const float4 *>(zf)[0], p1 = reinterpret_cast<const float4 *>(zf)[1];
                v[0] += p0.x; v[1] += p0.y; v[2] += p0.z; v[3] += p0.w;
                v[4] += p1.x; v[5] += p1.y; v[6] += p1.z; v[7] += p1.w;
            } else {
                uint4 raw = *reinterpret_cast<const uint4 *>(zp);
                const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float2 t = __half22float2(h[i]);
                    v[2 * i] += t.x;
                    v[2 * i + 1] += t.y;
                }
            }
        }
        if (f & SH_EPI_ACC_F32_IN) {
            const float4 p0 = reinterpret_cast<const float4 *>(rf)[0], p1 = reinterpret_cast<const float4 *>(rf)[1];
            v[0] += p0.x; v[1] += p0.y; v[2] += p0.z; v[3] += p0.w;
            v[4] += p1.x; v[5] += p1.y; v[6] += p1.z; v[7] += p1.w;
        }
        if (f & SH_EPI_BIAS) {
            uint4 raw = __ldg(reinterpret_cast<const uint4 *>(a.bias + col));
            const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 t = __half22float2(h[i]);
                v[2 * i] += t.x;
                v[2 * i + 1] += t.y;
            }
        }
        if (f & SH_EPI_GELU) {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = gelu_fast(v[i]);
        }
        if (f & SH_EPI_RESIDUAL) {
            uint4 raw = *reinterpret_cast<const uint4 *>(a.resid + (size_t)row * a.ldr + col);
            const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 t = __half22float2(h[i]);
                v[2 * i] += t.x;
                v[2 * i + 1] += t.y;
            }
        }
        if (z32) {
            reinterpret_cast<float4 *>(zf)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4 *>(zf)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
            uint4 out;
            __half2 *o = reinterpret_cast<__half2 *>(&out);
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            *reinterpret_cast<uint4 *>(zp) = out;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c = col + i;
            if (c >= a.N) break;
            float t = v[i];
            if (f & SH_EPI_ACCUMULATE) t += z32 ? zf[i] : __half2float(zp[i]);
            if (f & SH_EPI_ACC_F32_IN) t += rf[i];
            if (f & SH_EPI_BIAS) t += __half2float(a.bias[c]);
            if (f & SH_EPI_GELU) t = gelu_fast(t);
            if (f & SH_EPI_RESIDUAL) t += __half2float(a.resid[(size_t)row * a.ldr + c]);
            if (z32)
                zf[i] = t;
            else
                zp[i] = __float2half_rn(t);
        }
    }
}

__device__ __forceinline__ void load32(const __half *p, uint4 (&d)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = *reinterpret_cast<const uint4 *>(p + 8 * i);
}
__device__ __forceinline__ void add8(float *v, const uint4 &raw) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(h[i]);
        v[2 * i] += t.x;
        v[2 * i + 1] += t.y;
    }
}
// fused math of 32 consecutive in-range columns of one row on the 16-byte path; `res` holds the residual
__device__ __forceinline__ void epi_math32(const GemmArgs &a, uint32_t row, uint32_t col, float (&v)[32],
                                           const uint4 (&res)[4], float2 ln) {
    const uint32_t f = a.flags;
    if (f & SH_EPI_LN_IN) {
        const float4 *cs = reinterpret_cast<const float4 *>(a.ln_colsum + col);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 c = __ldg(cs + q);
            v[4 * q] = ln.y * fmaf(-ln.x, c.x, v[4 * q]);
            v[4 * q + 1] = ln.y * fmaf(-ln.x, c.y, v[4 * q + 1]);
            v[4 * q + 2] = ln.y * fmaf(-ln.x, c.z, v[4 * q + 2]);
            v[4 * q + 3] = ln.y * fmaf(-ln.x, c.w, v[4 * q + 3]);
        }
    }
    if (f & SH_EPI_ACCUMULATE) {
        uint4 old[4];
        load32(a.z + (size_t)row * a.ldz + col, old);
#pragma unroll
        for (int q = 0; q < 4; ++q) add8(v + 8 * q, old[q]);
    }
    if (f & SH_EPI_BIAS) {
#pragma unroll
        for (int q = 0; q < 4; ++q) add8(v + 8 * q, __ldg(reinterpret_cast<const uint4 *>(a.bias + col + 8 * q)));
    }
    if (f & SH_EPI_GELU) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = gelu_fast(v[i]);
    }
    if (f & SH_EPI_RESIDUAL) {
#pragma unroll
        for (int q = 0; q < 4; ++q) add8(v + 8 * q, res[q]);
    }
}

// fused math of 32 columns of one row whose loads may leave the matrix (guarded, element by element)
__device__ __forceinline__ void epi_math_guarded(const GemmArgs &a, uint32_t row, uint32_t col, float (&v)[32],
                                                 float2 ln) {
    if (row >= a.M) return;
    const uint32_t f = a.flags;
#pragma unroll
    for (int i = 0; i < 32; ++i) {   // fully unrolled: v stays in registers
        const uint32_t c = col + i;
        if (c >= a.N) continue;
        float t = v[i];
        if (f & SH_EPI_LN_IN) t = ln.y * fmaf(-ln.x, a.ln_colsum[c], t);
        if (f & SH_EPI_ACCUMULATE) t += __half2float(a.z[(size_t)row * a.ldz + c]);
        if (f & SH_EPI_BIAS) t += __half2float(a.bias[c]);
        if (f & SH_EPI_GELU) t = gelu_fast(t);
        if (f & SH_EPI_RESIDUAL) t += __half2float(a.resid[(size_t)row * a.ldr + c]);
        v[i] = t;
    }
}

// One 32-column chunk of the tile per warp (thread = row): the fused epilogue, then either the warp's 32 x 32 tile
// is staged in its shared-memory buffer (64-byte swizzle: 16-byte unit u of row r at u ^ ((r >> 1) & 3)) and written
// by one TMA store, or every thread stores its row directly (fp32 outputs, unaligned operands).
// `slot` non-null: stage in that buffer (it held this chunk's residual tile, already read; no earlier store is
// pending on it) instead of the warp's two rotating buffers.
__device__ __forceinline__ void epi_chunk(const GemmArgs &a, const CUtensorMap *mz, uint8_t *stg, uint32_t &nst,
                                          uint32_t row, uint32_t row_base, uint32_t col, float (&v)[32],
                                          const uint4 (&res)[4], uint32_t lane, float2 ln, float2 &st,
                                          uint8_t *slot = nullptr) {
    const bool inb = a.vec && row < a.M && col + 32 <= a.N;
    if (a.tma_store) {
        if (inb)
            epi_math32(a, row, col, v, res, ln);
        else
            epi_math_guarded(a, row, col, v, ln);
        if ((a.flags & SH_EPI_STATS_OUT) && row < a.M && col < a.N) {   // N % 64 == 0: whole chunks only
            float s1 = 0.f, s2 = 0.f, s1b = 0.f, s2b = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                s1 += v[i];
                s2 = fmaf(v[i], v[i], s2);
                s1b += v[i + 1];
                s2b = fmaf(v[i + 1], v[i + 1], s2b);
            }
            st.x += s1 + s1b;
            st.y += s2 + s2b;
            if (col & 32) {   // second chunk of a 64-column group
                a.stats_out[(size_t)row * (a.N / 64) + col / 64] = st;
                st = make_float2(0.f, 0.f);
            }
        }
        uint8_t *buf = slot ? slot : stg + (nst & 1u) * 2048;
        if (!slot) {
            if (lane == 0) bulk_wait_read1();     // the store issued from this buffer two chunks ago has read it
            __syncwarp();
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 out;
            __half2 *o = reinterpret_cast<__half2 *>(&out);
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i] = __floats2half2_rn(v[8 * q + 2 * i], v[8 * q + 2 * i + 1]);
            *reinterpret_cast<uint4 *>(buf + lane * 64 + ((q ^ ((lane >> 1) & 3u)) << 4)) = out;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(mz, buf, (int32_t)col, (int32_t)row_base);
            bulk_commit();
        }
        ++nst;
    } else if (inb && !(a.flags & (SH_EPI_F32_OUT | SH_EPI_ACC_F32_IN))) {
        epi_math32(a, row, col, v, res, ln);
        __half *zp = a.z + (size_t)row * a.ldz + col;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint4 out;
            __half2 *o = reinterpret_cast<__half2 *>(&out);
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i] = __floats2half2_rn(v[8 * q + 2 * i], v[8 * q + 2 * i + 1]);
            *reinterpret_cast<uint4 *>(zp + 8 * q) = out;
        }
    } else {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            float w8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w8[i] = v[8 * g + i];
            epilogue8(a, row, col + g * 8, w8);
        }
    }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
              const __grid_constant__ CUtensorMap map_z, GemmArgs a) {
    using C = TileCfg<BN>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t *smem = smem_raw + pad;
    uint8_t *epi_stage = smem + S * C::kStageBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(epi_stage + kEpiStageBytes);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;    // [2] accumulator ready for the epilogue
    uint64_t *tempty = tfull + 2;   // [2] accumulator drained by the epilogue
    uint64_t *esync = tempty + 2;   // epilogue-group barrier (split-K arrival protocol)
    uint64_t *mdone = esync + 1;    // every issued MMA has completed (exit path)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile uint32_t *last_flag = reinterpret_cast<volatile uint32_t *>(tmem_slot + 2);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiWarps);
        }
        mbar_init(esync, kEpiWarps);
        mbar_init(mdone, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t total_units = a.num_tiles * a.splits;
    // set-up above overlaps the previous kernel (programmatic dependent launch); operands only after it is done
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            prefetch_tmap(&map_x);
            prefetch_tmap(&map_w);
            uint32_t stage = 0, phase = 0;
            uint32_t armed[S];
            for (int s = 0; s < S; ++s) armed[s] = 2;   // 2 = never armed
            bool ok = true;
            for (uint32_t u = blockIdx.x; ok && u < total_units; u += gridDim.x) {
                const uint32_t tile = u / a.splits, split = u - tile * a.splits;
                uint32_t tm, tn;
                tile_coords(tile, a.num_tiles / a.tiles_n, a.tiles_n, a.group_m, tm, tn);
                const uint32_t kb0 = split * a.kb_per_split;
                const uint32_t kb1 = min(a.k_blocks, kb0 + a.kb_per_split);
                for (uint32_t kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort, a.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + stage * C::kStageBytes;
                    uint8_t *sb = sa + C::kABytes;
                    mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
                    armed[stage] = phase;
                    tma_load_2d(sa, &map_x, &full[stage], (int32_t)(kb * BK), (int32_t)(tm * BM));
#pragma unroll
                    for (int c = 0; c < BN / 64; ++c)
                        tma_load_2d(sb + c * (BK * 128), &map_w, &full[stage], (int32_t)(tn * BN + c * 64),
                                    (int32_t)(kb * BK));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // drain: every armed stage's last transaction must have landed before the CTA may exit
            for (int s = 0; s < S; ++s)
                if (armed[s] != 2) drain_wait(&full[s], armed[s]);
        }
    } else if (warp == 1) {
        {
            // ---------------- MMA issuer: the whole warp walks the loop, lane 0 issues (is0) ----------------
            const uint32_t is0 = lane == 0 ? 1u : 0u;
            constexpr uint32_t idesc = umma_idesc_f16(BM, BN, 0, 1);
            // descriptors of stage 0 built once; a stage / k-step adds its byte offset / 16 to the 14-bit address
            // field (shared-memory offsets stay below 256 KB, so the sum never carries out of the field)
            const uint64_t a_desc0 = sw128_desc(smem_u32(smem), 16, 1024);
            const uint64_t b_desc0 = sw128_desc(smem_u32(smem) + C::kABytes, BK * 128, 1024);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (uint32_t u = blockIdx.x; ok && u < total_units; u += gridDim.x) {
                const uint32_t tile = u / a.splits, split = u - tile * a.splits;
                (void)tile;
                const uint32_t kb0 = split * a.kb_per_split;
                const uint32_t kb1 = min(a.k_blocks, kb0 + a.kb_per_split);
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + acc * BN;
                for (uint32_t kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t so = (stage * C::kStageBytes) >> 4;
#pragma unroll
                    for (int j = 0; j < BK / 16; ++j)
                        umma_f16_ss_if(is0, d, a_desc0 + so + (uint64_t)(j * 2),
                                       b_desc0 + so + (uint64_t)(j * (2048 >> 4)), idesc, (kb > kb0 || j > 0) ? 1u : 0u);
                    umma_commit_if(is0, &empty[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_if(is0, &tfull[acc]);
                acc ^= 1u;
                if (acc == 0) acc_phase ^= 1u;
            }
            // exit path: tensor memory may only be freed once every issued MMA has completed
            umma_commit_if(is0, mdone);
            if (is0) drain_wait(mdone, 0);
        }
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        // warp w drains TMEM lane quarter (w % 4) = 32 rows, column half (w - 2) / 4 of the tile
        const uint32_t quarter = warp & 3u;
        const uint32_t half = (warp - 2u) >> 2;
        constexpr uint32_t HB = BN / 2;            // columns per warp
        const uint32_t row_in_tile = quarter * 32 + lane;
        const bool want_res = (a.flags & SH_EPI_RESIDUAL) != 0;
        uint8_t *stg = epi_stage + (warp - 2u) * 4096u;
        uint32_t nst = 0;    // TMA stores this warp has issued
        if (a.tma_store && lane == 0) prefetch_tmap(&map_z);
        uint32_t acc = 0, acc_phase = 0, es_phase = 0;
        for (uint32_t u = blockIdx.x; u < total_units; u += gridDim.x) {
            const uint32_t tile = u / a.splits, split = u - tile * a.splits;
            uint32_t tm, tn;
            tile_coords(tile, a.num_tiles / a.tiles_n, a.tiles_n, a.group_m, tm, tn);
            const uint32_t row = tm * BM + row_in_tile;
            const uint32_t row_base = tm * BM + quarter * 32;
            const uint32_t col0 = tn * BN + half * HB;
            // residual of the first chunk is fetched before the accumulator is ready
            uint4 res[4] = {};
            const bool res_vec = want_res && a.vec && row < a.M;
            if (res_vec && a.splits == 1 && col0 + 32 <= a.N) load32(a.resid + (size_t)row * a.ldr + col0, res);
            const float2 ln = ln_row(a, row);   // LayerNorm statistics of this row (SH_EPI_LN_IN)
            float2 st = make_float2(0.f, 0.f);
            if (!mbar_wait(&tfull[acc], acc_phase, abort, a.err)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + acc * BN + half * HB;
            // partial tile of this split: warp-interleaved so that every store (and the reducer's load) of a warp
            // covers 512 contiguous bytes: value 4 q + j of chunk c of epilogue warp e, lane l, lives at float
            // ((e * HB / 32 + c) * 8 + q) * 128 + 4 l + j of the tile-split block
            float *part = a.splits > 1 ? a.ws + ((size_t)tile * a.splits + split) * (BM * BN) +
                                             (size_t)(warp - 2u) * (HB / 32) * 1024 + lane * 4
                                       : nullptr;
#pragma unroll 1
            for (uint32_t c = 0; c < HB / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(taddr + c * 32, r);
                tmem_ld_wait();
                if (part) {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *reinterpret_cast<float4 *>(part + c * 1024 + i * 128) =
                            make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                        __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
                    continue;
                }
                const uint32_t col = col0 + c * 32;
                uint4 nres[4] = {};
                if (res_vec && c + 1 < HB / 32 && col + 64 <= a.N)
                    load32(a.resid + (size_t)row * a.ldr + col + 32, nres);   // next chunk's residual in flight
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                if (!a.tma_store || (row_base < a.M && col < a.N))
                    epi_chunk(a, &map_z, stg, nst, row, row_base, col, v, res, lane, ln, st);
#pragma unroll
                for (int i = 0; i < 4; ++i) res[i] = nres[i];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;

            if (a.splits > 1) {
                // arrival counter: the last split of this tile reduces the partials in split order. The epilogue
                // warps' partial stores are ordered before one thread's acquire-release atomic by the CTA barrier
                // (release is cumulative), and the last CTA's loads after it by the second barrier; a fence by every
                // thread is not needed.
                if (!epi_sync(esync, es_phase, abort, a.err)) break;
                if (threadIdx.x == 64) {
                    const uint32_t t = atom_add_acq_rel_gpu(&a.counters[tile], 1u);
                    const uint32_t last = (t == a.splits - 1) ? 1u : 0u;
                    if (last) a.counters[tile] = 0;   // ready for the next launch (stream order)
                    *last_flag = last;
                }
                if (!epi_sync(esync, es_phase, abort, a.err)) break;
                if (*last_flag) {
                    // sum the partial tiles in split order, 32 columns at a time with a whole split's row segment
                    // (8 x 16 B) in flight per load batch, then the same fused epilogue as an unsplit tile
                    const float *base =
                        a.ws + (size_t)tile * a.splits * (BM * BN) + (size_t)(warp - 2u) * (HB / 32) * 1024 + lane * 4;
#pragma unroll 1
                    for (uint32_t c = 0; c < HB / 32; ++c) {
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = 0.f;
#pragma unroll 2
                        for (uint32_t sp = 0; sp < a.splits; ++sp) {
                            const float *p = base + (size_t)sp * (BM * BN) + c * 1024;
                            float4 q[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i) q[i] = __ldcg(reinterpret_cast<const float4 *>(p + i * 128));
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                v[4 * i] += q[i].x;
                                v[4 * i + 1] += q[i].y;
                                v[4 * i + 2] += q[i].z;
                                v[4 * i + 3] += q[i].w;
                            }
                        }
                        const uint32_t col = col0 + c * 32;
                        uint4 res[4] = {};
                        if (res_vec && col + 32 <= a.N) load32(a.resid + (size_t)row * a.ldr + col, res);
                        epi_chunk(a, &map_z, stg, nst, row, row_base, col, v, res, lane, ln, st);
                    }
                }
                // last_flag is rewritten for the next tile only after every warp has read it
                if (!epi_sync(esync, es_phase, abort, a.err)) break;
            }
        }
        if (lane == 0 && nst) bulk_wait_all();   // the staging buffers stay live until every store completed
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// ---- 2-CTA (cta_group::2) variant: a cluster of two CTAs on two SMs computes a 256 x BN tile -------------------
// Each CTA loads its own 128 rows of the X tile and its own BN/2 columns of the W tile per stage (32 KB: 6 stages),
// both CTAs' TMA transactions complete on the leader's `full` barrier, the leader's single thread issues
// tcgen05.mma.cta_group::2 (M = 256), and its commits arrive on the `empty` / `tfull` barriers of both CTAs. Each
// CTA's tensor memory holds its own 128 rows of the accumulator (all BN columns), which its 8 epilogue warps drain
// exactly like the single-CTA kernel; they arrive on a local barrier, and warp 10 of each CTA forwards one arrive to
// the leader's `tempty` barrier (2 arrivals). Per stage and SM, W traffic is half that of the single-CTA tile. No
// split-K (the caller picks this kernel only without it).
constexpr int kPairStages = 6;

// BN = 512: 256 x 512 pair tiles from two N = 256 MMAs per k-step into one accumulator (all 512 tensor-memory
// columns): 25 % fewer operand bytes per MAC than 256 x 256, but the epilogue no longer overlaps the next tile's
// main loop, so the planner uses it for long K loops only.
// RES (BN = 256): the residual of an epilogue chunk arrives by TMA as a 32 x 32 tile in the slot its output then
// leaves from; four slots per epilogue warp (a whole 128-column half tile, loaded one tile ahead) take the shared
// memory of one load stage.
template <int BN, bool RES = false>
struct PairCfg {
    static constexpr int kStages = BN == 512 ? 4 : (RES ? kPairStages - 1 : kPairStages);
    static constexpr uint32_t kAcc = BN == 512 ? 1 : 2;          // accumulator buffers
    static constexpr uint32_t kMmaN = BN < 256 ? BN : 256;       // N of one MMA; BN / kMmaN of them per k-step
    static constexpr uint32_t kABytes = 128 * BK * 2;          // this CTA's 128 rows
    static constexpr uint32_t kBBytes = (BN / 2) * BK * 2;     // this CTA's half of every MMA's columns
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr uint32_t kTmemCols = kAcc * BN;
    static constexpr uint32_t kEpiBytes = RES ? 2 * kEpiStageBytes : kEpiStageBytes;   // per warp 4 or 2 slots of 2 KB
    static constexpr uint32_t kSmem = kStages * kStageBytes + kEpiBytes + 1024 + (RES ? 512 : 256);
};

// Work unit u of the 2-CTA kernel: whole tile u below a.full_units; past it, one kMmaN-wide column slice (h0) of
// the remaining tiles, BN / kMmaN units per tile, so that a short last wave of wide tiles runs as a fuller wave of
// narrower units. Every output element still accumulates the same MMAs in the same order.
template <int BN>
__device__ __forceinline__ void pair_unit(const GemmArgs &a, uint32_t u, uint32_t &tile, uint32_t &h0, uint32_t &nh) {
    constexpr uint32_t NH = BN / PairCfg<BN>::kMmaN;
    if (u < a.full_units) {
        tile = u;
        h0 = 0;
        nh = NH;
    } else {
        const uint32_t t = u - a.full_units;
        tile = a.full_units + t / NH;
        h0 = t % NH;
        nh = 1;
    }
}

// KS = 2: the stages go in pairs that share one full / empty barrier, so the producer waits, arms and the MMA
// thread waits, fences and commits once per two k-steps (the k-block count of every tile must be even).
template <int BN, bool RES = false, int KS = 1>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    k_gemm_tc2(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
               const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_r, GemmArgs a) {
    using C = PairCfg<BN, RES>;
    static_assert(C::kStages % KS == 0, "stage groups");
    constexpr int S = C::kStages / KS;   // barrier groups of KS stages
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t *smem = smem_raw + pad;
    uint8_t *epi_stage = smem + C::kStages * C::kStageBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(epi_stage + C::kEpiBytes);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;
    uint64_t *tempty = tfull + 2;
    uint64_t *mdone = tempty + 2;
    uint64_t *epi_done = mdone + 1;   // [2] this CTA's 8 epilogue warps have drained accumulator buffer i
    uint64_t *res_full = epi_done + 2;   // RES: [8 warps x 4 slots] a residual tile has landed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(res_full + (RES ? 32 : 0));
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);     // leader: its producer's arrive.expect_tx of both CTAs' bytes
            mbar_init(&empty[s], 1);    // both: the leader's commit
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);         // both: the leader's commit
            mbar_init(&tempty[i], 2);        // leader: warp 10 of both CTAs
            mbar_init(&epi_done[i], kEpiWarps);
        }
        if (RES)
            for (int i = 0; i < 32; ++i) mbar_init(&res_full[i], 1);
        mbar_init(mdone, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();     // both CTAs' barriers exist before any peer signal reaches them
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t total_units = a.num_units;
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&map_x);
            prefetch_tmap(&map_w);
            uint32_t stage = 0, phase = 0;
            uint32_t armed[S];
            for (int s = 0; s < S; ++s) armed[s] = 2;
            bool ok = true;
            for (uint32_t u = pair; ok && u < total_units; u += npairs) {
                uint32_t tile, h0, nh, tm, tn;
                pair_unit<BN>(a, u, tile, h0, nh);
                tile_coords(tile, a.num_tiles / a.tiles_n, a.tiles_n, a.group_m, tm, tn);
                const uint32_t stage_tx = 2 * (C::kABytes + nh * (C::kMmaN / 2) * BK * 2);   // both CTAs' bytes
                for (uint32_t kb = 0; kb < a.k_blocks; kb += KS) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort, a.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
                    if (leader) mbar_arrive_expect_tx(&full[stage], KS * stage_tx);
                    armed[stage] = phase;
#pragma unroll
                    for (int q = 0; q < KS; ++q) {
                        uint8_t *sa = smem + (stage * KS + q) * C::kStageBytes;
                        uint8_t *sb = sa + C::kABytes;
                        const int32_t k0 = (int32_t)((kb + q) * BK);
                        tma_load_2d_pair(sa, &map_x, bar, k0, (int32_t)(tm * 256 + rank * 128));
                        // 64-column boxes: MMA h reads this CTA's kMmaN / 2 columns h kMmaN + rank kMmaN / 2 ..
                        constexpr int kBoxesPerMma = C::kMmaN / 128;
#pragma unroll
                        for (int c = 0; c < BN / 128; ++c) {
                            const uint32_t h = c / kBoxesPerMma;
                            if (h < h0 || h >= h0 + nh) continue;   // a column slice loads its own MMA's boxes only
                            tma_load_2d_pair(sb + c * (BK * 128), &map_w, bar,
                                             (int32_t)(tn * BN + h * C::kMmaN + rank * (C::kMmaN / 2) +
                                                       (c % kBoxesPerMma) * 64),
                                             k0);
                        }
                    }
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // drain: a stage is free again only after the leader's MMAs read it, which is after its bytes landed
            for (int s = 0; s < S; ++s)
                if (armed[s] != 2) drain_wait(&empty[s], armed[s]);
        }
    } else if (warp == 1) {
        if (leader) {   // the whole warp walks the loop; lane 0 issues (is0)
            const uint32_t is0 = lane == 0 ? 1u : 0u;
            constexpr uint32_t idesc = umma_idesc_f16(256, C::kMmaN, 0, 1);
            constexpr uint32_t NH = BN / C::kMmaN;
            // The issue loop is one thread's dependency chain, so it does as little as possible per MMA: the
            // descriptors of stage 0 are built once and a stage / k-step only adds its offset / 16 to the 14-bit
            // address field (shared-memory offsets stay below 256 KB, so the sum never carries out of the field);
            // one commit per k-step frees the stage in both CTAs.
            const uint64_t a_desc0 = sw128_desc(smem_u32(smem), 16, 1024);
            const uint64_t b_desc0 = sw128_desc(smem_u32(smem) + C::kABytes, BK * 128, 1024);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (uint32_t u = pair; ok && u < total_units; u += npairs) {
                uint32_t tile, h0, nh;
                pair_unit<BN>(a, u, tile, h0, nh);
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort, a.err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + acc * BN;
                for (uint32_t kb = 0; kb < a.k_blocks; kb += KS) {
                    if (!mbar_wait(&full[stage], phase, abort, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int q = 0; q < KS; ++q) {
                        const uint64_t so = ((stage * KS + q) * C::kStageBytes) >> 4;
                        const uint64_t ad = a_desc0 + so, bd = b_desc0 + so;
#pragma unroll
                        for (int j = 0; j < BK / 16; ++j)
#pragma unroll
                            for (uint32_t h = 0; h < NH; ++h)
                                if (NH == 1 || (h >= h0 && h < h0 + nh))
                                    umma_f16_ss_pair_if(is0, d + h * C::kMmaN, ad + (uint64_t)(j * 2),
                                                        bd + (uint64_t)((h * (C::kMmaN / 2) * BK * 2 + j * 2048) >> 4),
                                                        idesc, (kb + q > 0 || j > 0) ? 1u : 0u);
                    }
                    umma_commit_pair_mask_if(is0, &empty[stage], 0x3);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair_mask_if(is0, &tfull[acc], 0x3);
                if (++acc == C::kAcc) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (is0) umma_commit_pair_both(mdone);   // both CTAs: every MMA the leader issued has completed
        }
        if (lane == 0) drain_wait(mdone, 0);
    } else if (warp == 10) {
        // A remote mbarrier arrive (release, cluster scope) stalls its thread for ~2000 cycles; this warp takes
        // that stall instead of the epilogue warps: it waits for the local epilogue_done barrier of the buffer and
        // forwards one arrive to the leader's tempty barrier.
        if (lane == 0) {
            const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&tempty[0]), 0),
                                               mapa_shared(smem_u32(&tempty[1]), 0)};
            uint32_t acc = 0, acc_phase = 0;
            for (uint32_t u = pair; u < total_units; u += npairs) {
                if (!mbar_wait(&epi_done[acc], acc_phase, abort, a.err)) break;
                mbar_arrive_cluster(tempty_leader[acc]);
                if (++acc == C::kAcc) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
    } else {
        const uint32_t quarter = warp & 3u;
        const uint32_t half = (warp - 2u) >> 2;
        const uint32_t row_in_tile = rank * 128 + quarter * 32 + lane;
        const bool want_res = (a.flags & SH_EPI_RESIDUAL) != 0;
        const uint32_t ew = warp - 2u;
        uint8_t *stg = epi_stage + ew * (RES ? 8192u : 4096u);
        uint32_t nst = 0;
        if (a.tma_store && lane == 0) prefetch_tmap(&map_z);
        uint32_t acc = 0, acc_phase = 0;
        // RES: the residual tiles of this warp's 32 rows x 128 columns of a unit, one TMA load per 32-column chunk
        // into slot c, issued one unit ahead (after the previous unit's stores have read the slots)
        uint32_t res_phase = 0, res_armed = 0;
        auto load_res = [&](uint32_t u) {
            uint32_t tile, h0, nh, tm, tn;
            pair_unit<BN>(a, u, tile, h0, nh);
            tile_coords(tile, a.num_tiles / a.tiles_n, a.tiles_n, a.group_m, tm, tn);
            const int32_t y = (int32_t)(tm * 256 + rank * 128 + quarter * 32);
#pragma unroll
            for (uint32_t c = 0; c < 4; ++c) {
                mbar_arrive_expect_tx(&res_full[ew * 4 + c], 2048);
                tma_load_2d(stg + c * 2048, &map_r, &res_full[ew * 4 + c], (int32_t)(tn * BN + half * 128 + c * 32), y);
            }
        };
        if (RES && lane == 0 && pair < total_units) {
            prefetch_tmap(&map_r);
            load_res(pair);
            res_armed = 1;
        }
        for (uint32_t u = pair; u < total_units; u += npairs) {
            uint32_t tile, h0, nh, tm, tn;
            pair_unit<BN>(a, u, tile, h0, nh);
            tile_coords(tile, a.num_tiles / a.tiles_n, a.tiles_n, a.group_m, tm, tn);
            const uint32_t HB = nh * (C::kMmaN / 2);   // columns per warp: this unit's columns, split in two halves
            const uint32_t row = tm * 256 + row_in_tile;
            const uint32_t row_base = tm * 256 + rank * 128 + quarter * 32;
            const uint32_t col0 = tn * BN + h0 * C::kMmaN + half * HB;
            uint4 res[4] = {};
            const bool res_vec = !RES && want_res && a.vec && row < a.M;
            if (res_vec && col0 + 32 <= a.N) load32(a.resid + (size_t)row * a.ldr + col0, res);
            const float2 ln = ln_row(a, row);
            float2 st = make_float2(0.f, 0.f);
            if (!mbar_wait(&tfull[acc], acc_phase, abort, a.err)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + acc * BN + h0 * C::kMmaN + half * HB;
            bool res_ok = true;
#pragma unroll 1
            for (uint32_t c = 0; c < HB / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(taddr + c * 32, r);
                const uint32_t col = col0 + c * 32;
                uint4 nres[4] = {};
                if (res_vec && c + 1 < HB / 32 && col + 64 <= a.N)
                    load32(a.resid + (size_t)row * a.ldr + col + 32, nres);
                uint8_t *slot = nullptr;
                if (RES) {   // this chunk's residual tile, 64-byte swizzled like the output staging
                    slot = stg + c * 2048;
                    if (!mbar_wait(&res_full[ew * 4 + c], res_phase, abort, a.err)) res_ok = false;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        res[q] = *reinterpret_cast<const uint4 *>(slot + lane * 64 + ((q ^ ((lane >> 1) & 3u)) << 4));
                }
                tmem_ld_wait();
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                if (!a.tma_store || (row_base < a.M && col < a.N))
                    epi_chunk(a, &map_z, stg, nst, row, row_base, col, v, res, lane, ln, st, slot);
                if (!RES) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) res[i] = nres[i];
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&epi_done[acc]);
            if (RES) {
                if (!res_ok) break;   // (the loads of this unit stay armed: drained below)
                res_phase ^= 1u;
                res_armed = 0;
                if (lane == 0 && u + npairs < total_units) {
                    bulk_wait_read0();   // this unit's stores have read the slots
                    load_res(u + npairs);
                    res_armed = 1;
                }
            }
            if (++acc == C::kAcc) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0 && nst) bulk_wait_all();
        if (RES && lane == 0 && res_armed)   // loads issued for a unit this warp did not reach (an abort)
            for (uint32_t c = 0; c < 4; ++c) drain_wait(&res_full[ew * 4 + c], res_phase);
    }

    __syncwarp();
    tc_fence_before();
    cluster_sync_all();     // neither CTA frees tensor memory while the pair may still use it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

// ---- CUDA-core fallback: 64 x 64 output tile, 256 threads x (4 x 4), K slabs of 16, any alignment ----------
__global__ void __launch_bounds__(256) k_gemm_simt(const __half *x, const __half *w, uint32_t ldx, uint32_t ldw,
                                                   GemmArgs a) {
    __shared__ float xs[16][64 + 1];
    __shared__ float ws[16][64 + 1];
    const uint32_t m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const uint32_t tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < a.K; k0 += 16) {
        for (int i = threadIdx.x; i < 16 * 64; i += 256) {
            const uint32_t kk = i & 15, mm = i >> 4;
            const uint32_t gm = m0 + mm, gk = k0 + kk;
            xs[kk][mm] = (gm < a.M && gk < a.K) ? __half2float(x[(size_t)gm * ldx + gk]) : 0.f;
            const uint32_t nn = i & 63, kw = i >> 6;
            const uint32_t gn = n0 + nn, gk2 = k0 + kw;
            ws[kw][nn] = (gn < a.N && gk2 < a.K) ? __half2float(w[(size_t)gk2 * ldw + gn]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float xv[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                xv[i] = xs[kk][ty * 4 + i];
                wv[i] = ws[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += xv[i] * wv[j];
        }
        __syncthreads();
    }
    GemmArgs b = a;
    b.vec = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float v[8] = {acc[i][0], acc[i][1], acc[i][2], acc[i][3], 0, 0, 0, 0};
        // columns [n0 + 4 tx, n0 + 4 tx + 4): the scalar epilogue path stops at N; clip to 4 columns here
        const uint32_t col = n0 + tx * 4;
        GemmArgs c = b;
        c.N = min(a.N, col + 4);
        epilogue8(c, m0 + ty * 4 + i, col, v);
    }
}

template <int BN>
bool set_smem_attr() {
    static bool done[sh::kMaxDevices] = {};
    const int d = sh::current_device() % sh::kMaxDevices;
    if (!done[d]) {
        if (!sh::cuda_ok(cudaFuncSetAttribute(k_gemm_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)TileCfg<BN>::kSmem),
                         "cudaFuncSetAttribute(gemm)"))
            return false;
        done[d] = true;
    }
    return true;
}

struct Plan {
    bool pair = false;            // 2-CTA kernel, 256 x pair_bn tiles
    int pair_bn = 256;
    int bn = 0;                   // 0: CUDA-core fallback
    uint32_t tiles_m = 0, tiles_n = 0, k_blocks = 0, splits = 1, kb_per_split = 0;
};

Plan make_plan(uint32_t M, uint32_t N, uint32_t K, uint32_t splits_req, int num_sms, int min_bn = 64) {
    Plan p;
    p.bn = N > 128 ? 256 : (N > 64 ? 128 : 64);
    if (p.bn < min_bn) p.bn = min_bn;
    p.tiles_m = (M + BM - 1) / BM;
    // narrower tiles when the wide ones leave most SMs idle
    while (p.bn > min_bn && (uint64_t)p.tiles_m * ((N + p.bn - 1) / p.bn) * 2 < (uint64_t)num_sms) p.bn >>= 1;
    p.tiles_n = (N + p.bn - 1) / p.bn;
    p.k_blocks = (K + BK - 1) / BK;
    const uint32_t tiles = p.tiles_m * p.tiles_n;
    uint32_t s = 1;
    if (splits_req == 0) {
        // a split costs ~1.3 us of partial-tile traffic and reduction: only K loops of 16+ blocks are split, into
        // pieces of at least 8 blocks (512^3: unsplit 5.7 us, 2 splits 6.9; 256 x 768 x 3072: unsplit 17.0, 6 splits 9.4)
        if (tiles * 2 <= (uint32_t)num_sms && p.k_blocks >= 16) {
            s = (uint32_t)num_sms / tiles;
            s = min(s, p.k_blocks / 8);
            s = min(s, 16u);
            s = max(s, 1u);
        }
    } else {
        s = min(splits_req, p.k_blocks);
    }
    p.kb_per_split = (p.k_blocks + s - 1) / s;
    p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
    // enough 256 x 256 tiles to keep every SM pair busy: the 2-CTA kernel (half the W traffic per SM)
    static const int pair_env = [] {
        const char *e = getenv("SH_GEMM_PAIR");
        return e ? atoi(e) : -1;
    }();
    if (p.splits == 1 && p.bn == 256 && pair_env != 0 &&
        (uint64_t)((M + 255) / 256) * p.tiles_n * 2 >= (uint64_t)num_sms)
        p.pair = true;
    // 256 x 512 pair tiles for long K loops when N is a multiple of 512 and the tile waves cost no more: a wide
    // tile takes ~1.5x a 256 x 256 one while the operand loads bound the main loop (SH_GEMM_PAIR_BN=256 / 512
    // forces one width; 512 still needs N % 512 == 0)
    static const int pair_bn_env = [] {
        const char *e = getenv("SH_GEMM_PAIR_BN");
        return e ? atoi(e) : 0;
    }();
    if (p.pair && N % 512 == 0 && pair_bn_env != 256) {
        // costs in half 256 x 256 tile-times: a wide tile ~3, a 256 x 256 tile 2; a wide tail of at most half the
        // SM pairs runs as 256-column slices (one 256 x 256 wave)
        const uint64_t pairs = (uint64_t)num_sms / 2, rows = (M + 255) / 256;
        const uint64_t t512 = rows * (N / 512), tail = t512 % pairs;
        const uint64_t c256 = 2 * ((rows * p.tiles_n + pairs - 1) / pairs);
        const uint64_t c512 = 3 * (t512 / pairs) + (tail == 0 ? 0 : (2 * tail <= pairs ? 2 : 3));
        if (pair_bn_env == 512 || (p.k_blocks >= 32 && c512 <= c256)) {
            p.pair_bn = 512;
            p.tiles_n = N / 512;
        }
    }
    return p;
}

template <int BN>
int launch_tc(const Plan &p, const CUtensorMap &mx, const CUtensorMap &mw, const CUtensorMap &mz, GemmArgs a,
              cudaStream_t st) {
    if (!set_smem_attr<BN>()) return -1;
    const uint32_t units = p.tiles_m * p.tiles_n * p.splits;
    const uint32_t grid = min(units, (uint32_t)sh::state().num_sms);
    return sh::cuda_ok(sh::launch_pdl(k_gemm_tc<BN>, dim3(grid), dim3(kThreads), TileCfg<BN>::kSmem, st, mx, mw, mz, a),
                       "sh_gemm launch")
               ? 0
               : -1;
}

// Work units of the 2-CTA kernel (pair_unit): whole tiles, except that a last wave of wide tiles filling at most
// half the SM pairs runs as 256-column slices, bn / 256 units per tile.
struct PairUnits {
    uint32_t full, units;
};
PairUnits pair_units(uint32_t num_tiles, uint32_t bn, uint32_t sm_pairs) {
    PairUnits r{num_tiles, num_tiles};
    const uint32_t nh = bn > 256 ? bn / 256 : 1;
    if (nh > 1 && sm_pairs > 0) {
        const uint32_t full = (num_tiles / sm_pairs) * sm_pairs, tail = num_tiles - full;
        if (tail && tail * nh <= sm_pairs) {
            r.full = full;
            r.units = full + tail * nh;
        }
    }
    return r;
}

template <int BN, bool RES = false, int KS = 1>
int launch_pair(const Plan &p, const CUtensorMap &mx, const CUtensorMap &mw, const CUtensorMap &mz,
                const CUtensorMap &mr, GemmArgs a, cudaStream_t st) {
    static bool done[sh::kMaxDevices] = {};
    const int d = sh::current_device() % sh::kMaxDevices;
    if (!done[d]) {
        if (!sh::cuda_ok(cudaFuncSetAttribute(k_gemm_tc2<BN, RES, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)PairCfg<BN, RES>::kSmem),
                         "cudaFuncSetAttribute(gemm pair)"))
            return -1;
        done[d] = true;
    }
    a.num_tiles = ((a.M + 255) / 256) * p.tiles_n;
    a.splits = 1;
    const uint32_t sm_pairs = (uint32_t)sh::state().num_sms / 2;
    const PairUnits pu = pair_units(a.num_tiles, BN, sm_pairs);
    a.full_units = pu.full;
    a.num_units = pu.units;
    const uint32_t pairs = min(a.num_units, sm_pairs);
    return sh::cuda_ok(sh::launch_pdl(k_gemm_tc2<BN, RES, KS>, dim3(2 * pairs), dim3(kPairThreads),
                                      PairCfg<BN, RES>::kSmem, st, mx, mw, mz, mr, a),
                       "sh_gemm launch (pair)")
               ? 0
               : -1;
}

// row-tiles per group of the tile order (SH_GEMM_GROUP_M overrides; 1 = plain row-major order)
uint32_t gemm_group_m() {
    static const uint32_t g = [] {
        const char *e = getenv("SH_GEMM_GROUP_M");
        const int v = e ? atoi(e) : (int)kGroupM;
        return (uint32_t)(v < 1 ? 1 : v);
    }();
    return g;
}

uint32_t smem_of(int bn) {
    return bn == 256 ? TileCfg<256>::kSmem : bn == 128 ? TileCfg<128>::kSmem : bn == 64 ? TileCfg<64>::kSmem : 0;
}

}  // namespace

namespace sh {

struct LnFold {          // the extra operands of sh_cuda_gemm_ln
    uint64_t stats;      // K / 64 (sum, sum of squares) pairs per row of X
    uint64_t colsum;     // 1 x N fp32: column sums of diag(gamma) W
    float eps;
    uint64_t stats_out;  // N / 64 pairs per output row
};

// Shared by sh_gemm / sh_gemm_mesh / sh_gemm_xmcast_ex / sh_cuda_gemm / sh_cuda_gemm_ln (`ln` non-null).
int gemm_run(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw,
             uint32_t ldz, uint64_t bias, uint64_t resid, uint32_t ldr, uint32_t flags, uint32_t splits_req,
             const char *name, const LnFold *ln) {
    if (M == 0 || N == 0) return 0;
    if (!x || !w || !z || ldx < K || ldw < N || ldz < N || ((flags & SH_EPI_BIAS) && !bias) ||
        ((flags & (SH_EPI_RESIDUAL | SH_EPI_ACC_F32_IN)) && (!resid || ldr < N)) ||
        ((flags & SH_EPI_RESIDUAL) && (flags & SH_EPI_ACC_F32_IN))) {
        set_error(-1, "[%s] bad operands: %ux%ux%u ld %u/%u/%u flags %#x", name, M, N, K, ldx, ldw, ldz, flags);
        return -1;
    }
    DeviceState &s = state();
    cudaStream_t st = s.stream;
    GemmArgs a;
    memset(&a, 0, sizeof a);
    a.z = (__half *)z;
    a.bias = (const __half *)bias;
    a.resid = (const __half *)resid;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ldz = ldz;
    a.ldr = ldr;
    a.flags = flags & (SH_EPI_ACCUMULATE | SH_EPI_BIAS | SH_EPI_GELU | SH_EPI_RESIDUAL | SH_EPI_F32_OUT |
                       SH_EPI_ACC_F32_IN);
    a.err = s.dev_err;
    a.vec = aligned16(z) && ldz % 8 == 0 && (!(flags & SH_EPI_BIAS) || aligned16(bias)) &&
            (!(flags & (SH_EPI_RESIDUAL | SH_EPI_ACC_F32_IN)) || (aligned16(resid) && ldr % 8 == 0));

    const bool tc = !(flags & SH_GEMM_SIMT) && K > 0 && aligned16(x) && aligned16(w) && ldx % 8 == 0 &&
                    ldw % 8 == 0 && encode_tiled() != nullptr;
    int min_bn = 64;
    if (ln) {
        const uint32_t lf = flags & (SH_EPI_LN_IN | SH_EPI_STATS_OUT);
        const bool ok = tc && a.vec && !(flags & (SH_EPI_F32_OUT | SH_EPI_ACC_F32_IN | SH_EPI_ACCUMULATE)) &&
                        (!(lf & SH_EPI_LN_IN) || (ln->stats && aligned16(ln->colsum) && K % 64 == 0)) &&
                        (!(lf & SH_EPI_STATS_OUT) || (ln->stats_out && N % 64 == 0));
        if (!ok) {
            set_error(-1, "[%s] LayerNorm folding needs 16-byte aligned fp16 operands, K %% 64 == 0 (LN in), "
                          "N %% 64 == 0 (stats out) and no accumulate / fp32 modes: %ux%ux%u flags %#x",
                      name, M, N, K, flags);
            return -1;
        }
        a.flags |= lf;
        a.ln_stats = (const float2 *)ln->stats;
        a.ln_colsum = (const float *)ln->colsum;
        a.ln_parts = K / 64;
        a.ln_eps = ln->eps;
        a.stats_out = (float2 *)ln->stats_out;
        splits_req = 1;
        if (lf & SH_EPI_STATS_OUT) min_bn = 128;   // each epilogue thread covers whole 64-column groups
    }
    if (!tc) {
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        if (grid.y > 65535u) {
            set_error(-1, "[%s] M = %u too large for the fallback kernel", name, M);
            return -1;
        }
        k_gemm_simt<<<grid, 256, 0, st>>>((const __half *)x, (const __half *)w, ldx, ldw, a);
        return cuda_ok(cudaGetLastError(), name) ? 0 : -1;
    }
    Plan p = make_plan(M, N, K, splits_req, s.num_sms, min_bn);
    a.tiles_n = p.tiles_n;
    a.group_m = gemm_group_m();
    a.num_tiles = p.tiles_m * p.tiles_n;
    a.k_blocks = p.k_blocks;
    a.splits = p.splits;
    a.kb_per_split = p.kb_per_split;
    if (p.splits > 1) {
        a.ws = workspace((size_t)a.num_tiles * p.splits * BM * p.bn * sizeof(float));
        a.counters = tile_counters(a.num_tiles);
        if (!a.ws || !a.counters) return -1;
    }
    CUtensorMap mx, mw, mz;
    if (!make_map_2d(&mx, (const void *)x, M, K, ldx, BM, BK, true) ||
        !make_map_2d(&mw, (const void *)w, K, N, ldw, BK, 64, true)) {
        set_error(-1, "[%s] cuTensorMapEncodeTiled failed for %ux%ux%u", name, M, N, K);
        return -1;
    }
    // fp16 results of single-pass tiles leave through TMA stores of 32 x 32 tiles (64-byte swizzled staging)
    static const bool tma_store_env = [] {   // SH_GEMM_TMA_STORE=0: every thread stores its own row instead
        const char *e = getenv("SH_GEMM_TMA_STORE");
        return !(e && atoi(e) == 0);
    }();
    a.tma_store = (tma_store_env || ln) && a.vec && p.splits == 1 &&
                  !(a.flags & (SH_EPI_F32_OUT | SH_EPI_ACC_F32_IN)) &&
                  make_map_2d_sw(&mz, (const void *)z, M, N, ldz, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    if (ln && !a.tma_store) {   // the folded epilogue runs on the staged-store path only
        set_error(-1, "[%s] cuTensorMapEncodeTiled failed for the output of %ux%ux%u", name, M, N, K);
        return -1;
    }
    if (!a.tma_store) mz = mx;   // not read by the kernel
    if (p.pair) {
        // 256 x 256 tiles with an fp16 residual and TMA-stored outputs: the residual tiles come in by TMA as well
        // (one coalesced 2 KB box per 32 x 32 chunk instead of one 16-byte load per row and thread); SH_GEMM_RES_TMA=0
        // reads them per thread instead
        static const bool res_tma_env = [] {
            const char *e = getenv("SH_GEMM_RES_TMA");
            return !(e && atoi(e) == 0);
        }();
        CUtensorMap mr;
        if (p.pair_bn == 256 && res_tma_env && a.tma_store && (a.flags & SH_EPI_RESIDUAL) &&
            make_map_2d_sw(&mr, (const void *)resid, M, N, ldr, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
            return launch_pair<256, true>(p, mx, mw, mz, mr, a, st);
        if (p.pair_bn == 512) return launch_pair<512>(p, mx, mw, mz, mx, a, st);
        // an even k-block count: one barrier round trip per two k-steps (SH_GEMM_KS=1 keeps one per k-step)
        static const bool ks2_env = [] {
            const char *e = getenv("SH_GEMM_KS");
            return !(e && atoi(e) == 1);
        }();
        if (ks2_env && a.k_blocks % 2 == 0) return launch_pair<256, false, 2>(p, mx, mw, mz, mx, a, st);
        return launch_pair<256>(p, mx, mw, mz, mx, a, st);
    }
    switch (p.bn) {
        case 256: return launch_tc<256>(p, mx, mw, mz, a, st);
        case 128: return launch_tc<128>(p, mx, mw, mz, a, st);
        default: return launch_tc<64>(p, mx, mw, mz, a, st);
    }
}

}  // namespace sh

namespace {

void cfg_fill(sh_gemm_cfg *c, const sh_gemm_cfg *in) {   // sh_gemm.inc.c:17-22: NULL / 0 fields -> defaults
    if (in)
        *c = *in;
    else {
        memset(c, 0, sizeof *c);
        c->pipeline = 1;
    }
    if (!c->tm) c->tm = 256;
    if (!c->tn) c->tn = 256;
    if (!c->tk) c->tk = 256;
}

}  // namespace

extern "C" {

uint32_t sh_gemm_l1_bytes(uint32_t M, uint32_t N, uint32_t K, const sh_gemm_cfg *) {
    Plan p = make_plan(M, N, K, 0, sh::state().num_sms ? sh::state().num_sms : 148);
    return smem_of(p.bn);
}

int sh_gemm(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw,
            uint32_t ldz, const sh_gemm_cfg *cfg, uint32_t) {
    sh_gemm_cfg c;
    cfg_fill(&c, cfg);
    if (M % c.tm || N % c.tn || K % c.tk) {
        sh::set_error(-1, "[sh_gemm] shape %ux%ux%u not divisible by tile %ux%ux%u", M, N, K, c.tm, c.tn, c.tk);
        return -1;
    }
    if (c.fmt != SH_FP16) {
        sh::set_error(-3, "[sh_gemm] fmt %u: only SH_FP16 runs on this backend", c.fmt);
        return -3;
    }
    return sh::gemm_run(x, w, z, M, N, K, ldx, ldw, ldz, 0, 0, 0, c.accumulate ? SH_EPI_ACCUMULATE : 0, 0, "sh_gemm",
                        nullptr);
}

int sh_gemm_mesh(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw,
                 uint32_t ldz, const sh_gemm_cfg *cfg) {
    sh_gemm_cfg c;
    cfg_fill(&c, cfg);
    if (c.tn != c.tm || M % c.tm || N % c.tn || K % c.tk) {
        sh::set_error(-1, "[sh_gemm_mesh] need tm==tn, M%%tm==0, N%%tn==0, K%%tk==0 (got %ux%ux%u tile %ux%ux%u)", M, N,
                      K, c.tm, c.tn, c.tk);
        return -1;
    }
    if (c.fmt != SH_FP16) {
        sh::set_error(-3, "[sh_gemm_mesh] fmt %u: only SH_FP16 runs on this backend", c.fmt);
        return -3;
    }
    return sh::gemm_run(x, w, z, M, N, K, ldx, ldw, ldz, 0, 0, 0, c.accumulate ? SH_EPI_ACCUMULATE : 0, 0,
                        "sh_gemm_mesh", nullptr);
}

uint32_t sh_gemm_xmcast_l1_bytes(uint32_t M, uint32_t N, uint32_t K, const sh_gemm_cfg *cfg, uint32_t) {
    const uint32_t rows = (cfg && cfg->tm) ? cfg->tm : M;
    if (rows == 0 || M % rows) return 0xFFFFFFFFu;
    return sh_gemm_l1_bytes(M, N, K, cfg);
}

int sh_gemm_xmcast_ex(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx,
                      uint32_t ldw, uint32_t ldz, const sh_gemm_cfg *cfg, uint32_t mode) {
    sh_gemm_cfg c;
    if (cfg)
        c = *cfg;
    else
        memset(&c, 0, sizeof c);
    const uint32_t rows = c.tm ? c.tm : M;
    int rc = 0;
    if (c.fmt & 3)
        rc = -3;
    else if (rows == 0 || M % rows || mode > SH_XM_WHOLE)
        rc = -1;
    if (rc) {
        sh::set_error(rc, "[sh_gemm_xmcast] %ux%ux%u tile %u,%u,%u mode %u: no plan (%d)", M, N, K, c.tm, c.tn, c.tk,
                      mode, rc);
        return rc;
    }
    return sh::gemm_run(x, w, z, M, N, K, ldx, ldw, ldz, 0, 0, 0, c.accumulate ? SH_EPI_ACCUMULATE : 0, 0,
                        "sh_gemm_xmcast", nullptr);
}

int sh_gemm_xmcast(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw,
                   uint32_t ldz, const sh_gemm_cfg *cfg) {
    return sh_gemm_xmcast_ex(x, w, z, M, N, K, ldx, ldw, ldz, cfg, SH_XM_AUTO);
}

int sh_cuda_gemm(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw,
                 uint32_t ldz, uint64_t bias, uint64_t residual, uint32_t ldr, uint32_t flags, uint32_t splits) {
    return sh::gemm_run(x, w, z, M, N, K, ldx, ldw, ldz, bias, residual, ldr, flags, splits, "sh_cuda_gemm",
                        nullptr);
}

int sh_cuda_gemm_plan(uint32_t M, uint32_t N, uint32_t K, uint32_t splits, uint32_t num_sms,
                      sh_cuda_gemm_plan_t *out) {
    if (!out) return -1;
    *out = sh_cuda_gemm_plan_t{};
    if (M == 0 || N == 0) return 0;
    const uint32_t sms = num_sms ? num_sms : (uint32_t)sh::state().num_sms;
    if (K == 0 || sms == 0) return 0;   // the CUDA-core kernel
    const Plan p = make_plan(M, N, K, splits, (int)sms);
    out->k_blocks = p.k_blocks;
    out->splits = p.splits;
    out->tiles_n = p.tiles_n;
    if (p.pair) {
        out->kernel = 2;
        out->bn = (uint32_t)p.pair_bn;
        out->tiles_m = (M + 255) / 256;
        const PairUnits pu = pair_units(out->tiles_m * p.tiles_n, out->bn, sms / 2);
        out->full_units = pu.full;
        out->units = pu.units;
        out->grid = 2 * std::min(pu.units, sms / 2);
    } else {
        out->kernel = 1;
        out->bn = (uint32_t)p.bn;
        out->tiles_m = p.tiles_m;
        out->units = out->full_units = p.tiles_m * p.tiles_n * p.splits;
        out->grid = std::min(out->units, sms);
    }
    return 0;
}

int sh_cuda_gemm_ln(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx,
                    uint32_t ldw, uint32_t ldz, uint64_t bias, uint64_t residual, uint32_t ldr, uint32_t flags,
                    uint64_t ln_stats, uint64_t ln_colsum, float ln_eps, uint64_t stats_out) {
    const sh::LnFold ln{ln_stats, ln_colsum, ln_eps, stats_out};
    return sh::gemm_run(x, w, z, M, N, K, ldx, ldw, ldz, bias, residual, ldr,
                        flags & ~(uint32_t)SH_GEMM_SIMT, 1, "sh_cuda_gemm_ln", &ln);
}

}  // extern "C"

// ================================================================================================================
// Split-K GEMM that allocates nothing: sh_cuda_gemm_splitk_noalloc.
//
// Some callers cannot let a library call cudaMalloc: hosts that hand every byte of device memory to their own pool
// (a serving runtime with a fixed memory budget, a framework allocator that owns the device), and loops that cannot
// afford cudaMalloc's implicit device-wide synchronisation. sh_cuda_gemm may grow its split-K workspace with
// cudaMalloc on first use of a shape; this entry point instead uses one fixed scratch array compiled into the
// library (kNoAllocScratchBytes = 8 MiB per device, which every GPU that loads the library holds until exit).
// Layout: [arrival counters, 4096 x u32][error word][fp32 partial tiles]. The partial tiles of a call need
// tiles x splits x 128 x BN x 4 bytes; a call that would need more than the array holds returns -2 and changes
// nothing. The first call on a device looks up the array's device address with cudaGetSymbolAddress (with that
// device current) and should therefore come before any stream capture on it. Every call shares the array and
// clears the counters it uses before its kernel, on the caller's stream: calls that overlap on the GPU (two
// streams, two threads) race on the array and must be serialised by the caller.
// It always runs the single-CTA kernel (the only one with a split-K path), so the planner's 2-CTA choice is
// replaced by 128 x BN tiles. Stream: the one bound with sh_cuda_set_stream once the runtime has started on the
// device, else the legacy default stream; a kernel's bounded-wait error then lands in the array's error word,
// which sh_cuda_device_error also reads and clears.
// ================================================================================================================
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr size_t kNoAllocCounters = 4096;
constexpr size_t kNoAllocErrOffset = kNoAllocCounters * sizeof(uint32_t);
constexpr size_t kNoAllocPartialOffset = 32768;
static __device__ __align__(256) unsigned char g_splitk_scratch[kNoAllocScratchBytes];

static void *g_scratch_addr[sh::kMaxDevices];
static std::mutex g_scratch_mu;

// Device address of g_splitk_scratch on `dev` (the current device); nullptr after printing the reason.
void *noalloc_scratch(int dev) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_splitk_scratch);
        if (e != cudaSuccess || !p) {
            sh::set_error((int)e, "[sh_cuda_gemm_splitk_noalloc] cudaGetSymbolAddress failed: %s",
                          cudaGetErrorString(e));
            return nullptr;
        }
        g_scratch_addr[dev] = p;
    }
    return g_scratch_addr[dev];
}

}  // namespace

namespace sh {

// Returns and clears the no-alloc array's error word on `dev` (the current device); 0 when no call has looked
// the array up there. Used by sh_cuda_device_error after its stream synchronisation.
int noalloc_take_error(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return 0;
    void *base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        base = g_scratch_addr[dev];
    }
    if (!base) return 0;
    int v = 0;
    int *word = reinterpret_cast<int *>(static_cast<unsigned char *>(base) + kNoAllocErrOffset);
    if (!cuda_ok(cudaMemcpy(&v, word, sizeof v, cudaMemcpyDeviceToHost), "sh_cuda_device_error")) return -1;
    if (v) cudaMemset(word, 0, sizeof(int));
    return v;
}

}  // namespace sh

extern "C" int sh_cuda_gemm_splitk_noalloc(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K,
                                           uint32_t ldx, uint32_t ldw, uint32_t ldz, uint64_t bias, uint64_t residual,
                                           uint32_t ldr, uint32_t flags, uint32_t splits) {
    const char *name = "sh_cuda_gemm_splitk_noalloc";
    constexpr uint32_t kFlags = SH_EPI_ACCUMULATE | SH_EPI_BIAS | SH_EPI_GELU | SH_EPI_RESIDUAL | SH_EPI_F32_OUT |
                                SH_EPI_ACC_F32_IN | SH_GEMM_SIMT;
    if (flags & ~kFlags) {
        sh::set_error(-1, "[%s] flags %#x: only accumulate / bias / gelu / residual / fp32 out / fp32 carry-in / "
                          "simt are supported", name, flags);
        return -1;
    }
    if (M == 0 || N == 0) return 0;
    if (!x || !w || !z || ldx < K || ldw < N || ldz < N || ((flags & SH_EPI_BIAS) && !bias) ||
        ((flags & (SH_EPI_RESIDUAL | SH_EPI_ACC_F32_IN)) && (!residual || ldr < N)) ||
        ((flags & SH_EPI_RESIDUAL) && (flags & SH_EPI_ACC_F32_IN))) {
        sh::set_error(-1, "[%s] bad operands: %ux%ux%u ld %u/%u/%u flags %#x", name, M, N, K, ldx, ldw, ldz, flags);
        return -1;
    }
    int dev = 0;
    if (!sh::cuda_ok(cudaGetDevice(&dev), name)) return -1;
    if (dev >= sh::kMaxDevices) {
        sh::set_error(-1, "[%s] device %d out of range", name, dev);
        return -1;
    }
    int num_sms = 0;
    if (!sh::cuda_ok(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev), name)) return -1;
    int *bound_err = nullptr;
    cudaStream_t st = sh::peek_stream(dev, &bound_err);
    unsigned char *scratch = static_cast<unsigned char *>(noalloc_scratch(dev));
    if (!scratch) return -1;

    GemmArgs a;
    memset(&a, 0, sizeof a);
    a.z = (__half *)z;
    a.bias = (const __half *)bias;
    a.resid = (const __half *)residual;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ldz = ldz;
    a.ldr = ldr;
    a.flags = flags & ~(uint32_t)SH_GEMM_SIMT;
    a.err = bound_err ? bound_err : reinterpret_cast<int *>(scratch + kNoAllocErrOffset);
    a.vec = sh::aligned16(z) && ldz % 8 == 0 && (!(flags & SH_EPI_BIAS) || sh::aligned16(bias)) &&
            (!(flags & (SH_EPI_RESIDUAL | SH_EPI_ACC_F32_IN)) || (sh::aligned16(residual) && ldr % 8 == 0));
    const bool tc = !(flags & SH_GEMM_SIMT) && K > 0 && sh::aligned16(x) && sh::aligned16(w) && ldx % 8 == 0 &&
                    ldw % 8 == 0 && sh::encode_tiled() != nullptr;
    if (!tc) {   // the CUDA-core kernel needs no scratch
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        if (grid.y > 65535u) {
            sh::set_error(-1, "[%s] M = %u too large for the fallback kernel", name, M);
            return -1;
        }
        k_gemm_simt<<<grid, 256, 0, st>>>((const __half *)x, (const __half *)w, ldx, ldw, a);
        return sh::cuda_ok(cudaGetLastError(), name) ? 0 : -1;
    }
    Plan p = make_plan(M, N, K, splits, num_sms);
    if (p.pair) {   // 256 x 512 pair tiles set tiles_n = N / 512; this entry point launches 128 x bn tiles
        p.pair = false;
        p.pair_bn = 256;
        p.tiles_n = (N + p.bn - 1) / p.bn;
    }
    a.tiles_n = p.tiles_n;
    a.group_m = gemm_group_m();
    a.num_tiles = p.tiles_m * p.tiles_n;
    a.k_blocks = p.k_blocks;
    a.splits = p.splits;
    a.kb_per_split = p.kb_per_split;
    if (p.splits > 1) {
        const size_t need = (size_t)a.num_tiles * p.splits * BM * p.bn * sizeof(float);
        if (a.num_tiles > kNoAllocCounters || need > kNoAllocScratchBytes - kNoAllocPartialOffset) {
            sh::set_error(-2, "[%s] %ux%ux%u in %u splits needs %zu B of partial tiles for %u tiles; the fixed scratch "
                          "holds %zu B and %zu tiles", name, M, N, K, p.splits, need, a.num_tiles,
                          kNoAllocScratchBytes - kNoAllocPartialOffset, kNoAllocCounters);
            return -2;
        }
        a.counters = reinterpret_cast<uint32_t *>(scratch);
        a.ws = reinterpret_cast<float *>(scratch + kNoAllocPartialOffset);
        // the arrival counters this call uses must start at zero (a call that gave up may have left them set)
        if (!sh::cuda_ok(cudaMemsetAsync(a.counters, 0, a.num_tiles * sizeof(uint32_t), st), name)) return -1;
    }
    CUtensorMap mx, mw;
    if (!sh::make_map_2d(&mx, (const void *)x, M, K, ldx, BM, BK, true) ||
        !sh::make_map_2d(&mw, (const void *)w, K, N, ldw, BK, 64, true)) {
        sh::set_error(-1, "[%s] cuTensorMapEncodeTiled failed for %ux%ux%u", name, M, N, K);
        return -1;
    }
    const uint32_t grid = min(a.num_tiles * p.splits, (uint32_t)num_sms);
    switch (p.bn) {
        case 256:
            if (!set_smem_attr<256>()) return -1;
            k_gemm_tc<256><<<grid, kThreads, TileCfg<256>::kSmem, st>>>(mx, mw, mx, a);
            break;
        case 128:
            if (!set_smem_attr<128>()) return -1;
            k_gemm_tc<128><<<grid, kThreads, TileCfg<128>::kSmem, st>>>(mx, mw, mx, a);
            break;
        default:
            if (!set_smem_attr<64>()) return -1;
            k_gemm_tc<64><<<grid, kThreads, TileCfg<64>::kSmem, st>>>(mx, mw, mx, a);
            break;
    }
    return sh::cuda_ok(cudaGetLastError(), name) ? 0 : -1;
}
