// Fused multi-head attention of the operator library: o = softmax(scale q k^T) v per head
// (reference: runtime/sh_attention.inc.c:41-243; declared at runtime/sh_ops.h:102-127).
//
// The reference keeps a whole sq x S score block in one cluster's TCDM (no online softmax), so S is bounded by
// L1. Here attention is flash-style with an online softmax, so S is unbounded:
//   - k_attn_tc (sm_100a tensor cores, dh = 64): one CTA per (sequence, head, 128 query rows); Q/K/V tiles come
//     in by TMA, S = Q K^T accumulates in tensor memory (tcgen05.mma), the softmax runs in registers from
//     tcgen05.ld, P (fp16) goes to shared memory and O += P V accumulates in tensor memory;
//   - k_attn_simt: CUDA-core fallback for other head widths and unaligned operands.
#include <math.h>
#include <string.h>

#include "sh_internal.cuh"

namespace sh {
int attention_tc_launch(const __half *q, const __half *k, const __half *v, __half *o, uint32_t S, uint32_t H,
                        uint32_t dh, uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t B,
                        bool *launched);
}

namespace {

constexpr int kSimtRows = 128;   // query rows per CTA (one per thread)
constexpr int kSimtKeys = 32;    // keys staged per step

template <int DH>
__global__ void __launch_bounds__(kSimtRows) k_attn_simt(const __half *q, const __half *k, const __half *v, __half *o,
                                                         uint32_t S, uint32_t dh, uint32_t ldq, uint32_t ldk,
                                                         uint32_t ldv, uint32_t ldo, float scale_log2) {
    __shared__ float ks[kSimtKeys][DH];
    __shared__ float vs[kSimtKeys][DH];
    const uint32_t b = blockIdx.z, h = blockIdx.y;
    const uint32_t row = blockIdx.x * kSimtRows + threadIdx.x;
    const size_t r0 = (size_t)b * S;
    const size_t col0 = (size_t)h * dh;
    float qr[DH], acc[DH];
    float m = -INFINITY, l = 0.f;
#pragma unroll
    for (int d = 0; d < DH; ++d) {
        qr[d] = (row < S && d < (int)dh) ? __half2float(q[(r0 + row) * ldq + col0 + d]) * scale_log2 : 0.f;
        acc[d] = 0.f;
    }
    for (uint32_t kt = 0; kt < S; kt += kSimtKeys) {
        for (uint32_t i = threadIdx.x; i < kSimtKeys * DH; i += kSimtRows) {
            const uint32_t j = i / DH, d = i % DH;
            const bool in = kt + j < S && d < dh;
            ks[j][d] = in ? __half2float(k[(r0 + kt + j) * ldk + col0 + d]) : 0.f;
            vs[j][d] = in ? __half2float(v[(r0 + kt + j) * ldv + col0 + d]) : 0.f;
        }
        __syncthreads();
        const uint32_t nk = min((uint32_t)kSimtKeys, S - kt);
        float s[kSimtKeys];
        float tmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < kSimtKeys; ++j) {
            float t = 0.f;
#pragma unroll
            for (int d = 0; d < DH; ++d) t += qr[d] * ks[j][d];
            s[j] = (j < (int)nk) ? t : -INFINITY;
            tmax = fmaxf(tmax, s[j]);
        }
        const float mn = fmaxf(m, tmax);
        const float corr = exp2f(m - mn);
        l *= corr;
#pragma unroll
        for (int d = 0; d < DH; ++d) acc[d] *= corr;
#pragma unroll
        for (int j = 0; j < kSimtKeys; ++j) {
            const float p = exp2f(s[j] - mn);
            l += p;
#pragma unroll
            for (int d = 0; d < DH; ++d) acc[d] += p * vs[j][d];
        }
        m = mn;
        __syncthreads();
    }
    if (row < S) {
        const float inv = 1.f / l;
        for (uint32_t d = 0; d < dh; ++d) o[(r0 + row) * ldo + col0 + d] = __float2half_rn(acc[d] * inv);
    }
}

// The reference's TCDM layout of one work item (sh_attention.inc.c:43-49, base 0x1000, 8 profile words).
uint32_t ref_l1_bytes(uint32_t S, uint32_t dh, uint32_t sq) {
    const uint32_t kb = S * dh * 2, qb = sq * dh * 2, sb = sq * S * 2;
    return 0x1000u + 2 * qb + 3 * kb + sb + sq * 4 + 8 * 4;
}

int check(uint32_t S, uint32_t dh, uint32_t sq) {   // sh_attention.inc.c:198-205 without the TCDM budget
    if ((S & 3) || (dh & 3) || dh == 0 || sq == 0 || (sq & 3) || S % sq) {
        sh::set_error(-1, "[sh_attention] S=%u dh=%u sq=%u: need S %% 4 == 0, dh %% 4 == 0, sq | S, sq %% 4 == 0", S,
                      dh, sq);
        return -1;
    }
    return 0;
}

int run(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t H, uint32_t dh, uint32_t ldq,
        uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t B) {
    if (S == 0 || H == 0 || B == 0) return 0;
    if (!q || !k || !v || !o) {
        sh::set_error(-1, "[sh_attention] null operand");
        return -1;
    }
    bool launched = false;
    const int rc = sh::attention_tc_launch((const __half *)q, (const __half *)k, (const __half *)v, (__half *)o, S, H,
                                           dh, ldq, ldk, ldv, ldo, scale, B, &launched);
    if (launched || rc) return rc;
    const float sl2 = scale * 1.4426950408889634f;
    dim3 grid((S + kSimtRows - 1) / kSimtRows, H, B);
    if (grid.y > 65535u || grid.z > 65535u) {
        sh::set_error(-1, "[sh_attention] H=%u B=%u too large", H, B);
        return -1;
    }
    cudaStream_t st = sh::stream();
#define SH_ATTN_SIMT(DHT)                                                                                        \
    k_attn_simt<DHT><<<grid, kSimtRows, 0, st>>>((const __half *)q, (const __half *)k, (const __half *)v,        \
                                                 (__half *)o, S, dh, ldq, ldk, ldv, ldo, sl2)
    if (dh <= 16)
        SH_ATTN_SIMT(16);
    else if (dh <= 32)
        SH_ATTN_SIMT(32);
    else if (dh <= 64)
        SH_ATTN_SIMT(64);
    else if (dh <= 128)
        SH_ATTN_SIMT(128);
    else {
        sh::set_error(-1, "[sh_attention] dh=%u > 128 is not supported", dh);
        return -1;
    }
#undef SH_ATTN_SIMT
    return sh::cuda_ok(cudaGetLastError(), "sh_attention") ? 0 : -1;
}

}  // namespace

extern "C" {

uint32_t sh_attention_l1_bytes_q(uint32_t S, uint32_t dh, uint32_t sq) {
    (void)S;
    (void)sq;
    // the tensor-core kernel (dh = 64): Q, K, V tiles of 128 x 64 + the 128 x 128 P tile + alignment + barriers;
    // the CUDA-core kernel: one staged block of 32 keys of K and V in fp32
    return dh == 64 ? 3 * 128 * 64 * 2 + 128 * 128 * 2 + 1024 + 128 : 2 * kSimtKeys * (dh <= 128 ? dh : 128) * 4;
}

uint32_t sh_attention_l1_bytes(uint32_t S, uint32_t dh) { return sh_attention_l1_bytes_q(S, dh, S); }

// sh_attention.inc.c:55-65, evaluated against the reference's 1 MB TCDM so that the compiler's mirror of this rule
// (frontend/siglip.py:67-71 -> dse/tiling.py:80-90) and the library agree.
uint32_t sh_attention_q_block(uint32_t S, uint32_t dh, uint32_t H, uint32_t P) {
    const uint32_t cand[4] = {S, 256, 128, 64};
    uint32_t best = 0, best_rows = 0;
    if (P == 0) P = 1;
    for (int i = 0; i < 4; ++i) {
        const uint32_t sq = cand[i];
        if (sq == 0 || sq > S || S % sq || sq % 4 || ref_l1_bytes(S, dh, sq) > 0x100000u) continue;
        const uint32_t items = H * (S / sq), rows = ((items + P - 1) / P) * sq;
        if (!best || rows < best_rows) {
            best = sq;
            best_rows = rows;
        }
    }
    return best;
}

uint32_t sh_attention_profile(uint32_t, uint32_t, uint32_t) { return 0; }

int sh_attention_head(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t dh, uint32_t ldq,
                      uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t) {
    if (check(S, dh, 4)) return -1;
    return run(q, k, v, o, S, 1, dh, ldq, ldk, ldv, ldo, scale, 1);
}

int sh_attention_q(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t D, uint32_t H, uint32_t ldq,
                   uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t cluster, uint32_t sq) {
    const uint32_t dh = H ? D / H : 0;
    if (H == 0 || dh * H != D) {
        sh::set_error(-1, "[sh_attention] D=%u not divisible by H=%u", D, H);
        return -1;
    }
    if (!sq) sq = sh_attention_q_block(S, dh, H, cluster == SH_ALL ? 16u : 1u);
    if (!sq) sq = 4;   // the reference's rule found no TCDM fit; this kernel has no such bound
    if (check(S, dh, sq)) return -1;
    return run(q, k, v, o, S, H, dh, ldq, ldk, ldv, ldo, scale, 1);
}

int sh_attention(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t D, uint32_t H, uint32_t ldq,
                 uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t cluster) {
    return sh_attention_q(q, k, v, o, S, D, H, ldq, ldk, ldv, ldo, scale, cluster, 0);
}

int sh_cuda_attention_batched(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t D, uint32_t H,
                              uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t B) {
    const uint32_t dh = H ? D / H : 0;
    if (H == 0 || dh * H != D) {
        sh::set_error(-1, "[sh_attention] D=%u not divisible by H=%u", D, H);
        return -1;
    }
    if (check(S, dh, 4)) return -1;
    return run(q, k, v, o, S, H, dh, ldq, ldk, ldv, ldo, scale, B);
}

}  // extern "C"

// ================================================================================================================
// Tensor-core path (dh = 64). One CTA per (sequence, head, block of 128 query rows), 160 threads:
//   warp 0, lane 0 : TMA loads (Q once, K/V block by block) and the tcgen05.mma issue;
//   warps 1..4     : softmax + output, one query row per thread (warp w owns TMEM lanes 32 (w % 4) ..).
// Per key block of 128:  S = Q K^T (M=128, N=128, K=64; both K-major) -> TMEM columns [0, 128);
//   softmax warps read S twice (row max, then exp2 + fp16 P into shared memory in the 128-byte-swizzled K-major
//   layout the next MMA reads), Opart = P V (M=128, N=64, K=128; V is MN-major as stored) -> TMEM [128, 192);
//   the running output o = o * exp2(m_old - m_new) + Opart, running max m and sum l stay in registers.
// Q/K/V are read through 3-D tensor maps [sequence, row, column], so rows past the end of a sequence are zeros;
// keys past the end are masked to -inf before the softmax. Shared memory: Q 16 KB + K 16 KB + V 16 KB + P 32 KB,
// tensor memory 256 columns: two CTAs fit on an SM and overlap each other's softmax with their MMAs.
// ================================================================================================================
namespace {

constexpr int kTcRows = 128, kTcKeys = 128, kTcDh = 64;
constexpr uint32_t kTileBytes = kTcRows * kTcDh * 2;          // 16 KB: Q, K or V tile
constexpr uint32_t kPBytes = kTcRows * kTcKeys * 2;           // 32 KB: P, two 64-key halves of 16 KB
constexpr uint32_t kAttnSmem = 3 * kTileBytes + kPBytes + 1024 + 128;
constexpr uint32_t kAttnTmemCols = 256;

struct AttnArgs {
    __half *o;
    uint32_t S, ldo, nkb;
    float sl2;   // scale * log2(e)
    int *err;
};

__global__ void __launch_bounds__(160, 2)
    k_attn_tc(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
              const __grid_constant__ CUtensorMap mv, AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t *sm = smem_raw + pad;
    uint8_t *sq = sm, *sk = sm + kTileBytes, *sv = sm + 2 * kTileBytes, *sp = sm + 3 * kTileBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + 3 * kTileBytes + kPBytes);
    uint64_t *bq = bars, *bkv = bars + 1, *bs = bars + 2, *bp = bars + 3, *bo = bars + 4, *bdone = bars + 5;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 6);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    if (threadIdx.x == 0) {
        mbar_init(bq, 1);
        mbar_init(bkv, 1);
        mbar_init(bs, 1);
        mbar_init(bp, 4);
        mbar_init(bo, 1);
        mbar_init(bdone, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kAttnTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int32_t col = (int32_t)(h * kTcDh);

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&mq);
            prefetch_tmap(&mk);
            prefetch_tmap(&mv);
            constexpr uint32_t idesc_s = umma_idesc_f16(kTcRows, kTcKeys, 0, 0);
            constexpr uint32_t idesc_o = umma_idesc_f16(kTcRows, kTcDh, 0, 1);
            mbar_arrive_expect_tx(bq, kTileBytes);
            tma_load_3d(sq, &mq, bq, col, (int32_t)(qb * kTcRows), (int32_t)b);
            bool q_landed = false, kv_armed = false, ok = true;
            uint32_t kv_phase = 0;
            for (uint32_t j = 0; ok && j < a.nkb; ++j) {
                const uint32_t ph = j & 1u;
                if (j > 0 && !mbar_wait(bo, ph ^ 1u, abort, a.err)) break;   // P V of block j-1 done with V, P
                mbar_arrive_expect_tx(bkv, 2 * kTileBytes);
                kv_armed = true;
                kv_phase = ph;
                tma_load_3d(sk, &mk, bkv, col, (int32_t)(j * kTcKeys), (int32_t)b);
                tma_load_3d(sv, &mv, bkv, col, (int32_t)(j * kTcKeys), (int32_t)b);
                if (!q_landed) {
                    if (!mbar_wait(bq, 0, abort, a.err)) break;
                    q_landed = true;
                }
                if (!mbar_wait(bkv, ph, abort, a.err)) break;
                tc_fence_after();
                const uint32_t aq = smem_u32(sq), ak = smem_u32(sk), av = smem_u32(sv), ap = smem_u32(sp);
#pragma unroll
                for (int k = 0; k < kTcDh / 16; ++k)
                    umma_f16_ss(tmem, sw128_desc(aq + k * 32, 16, 1024), sw128_desc(ak + k * 32, 16, 1024), idesc_s,
                                k > 0 ? 1u : 0u);
                umma_commit(bs);
                if (!mbar_wait(bp, ph, abort, a.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < kTcKeys / 16; ++k)
                    umma_f16_ss(tmem + kTcKeys,
                                sw128_desc(ap + (k >> 2) * (kTcRows * 128) + (k & 3) * 32, 16, 1024),
                                sw128_desc(av + k * 2048, 16384, 1024), idesc_o, k > 0 ? 1u : 0u);
                umma_commit(bo);
            }
            // exit: every issued MMA complete, every issued TMA landed
            umma_commit(bdone);
            const long long t0 = clock64();
            while (!mbar_try_wait(bdone, 0) && (unsigned long long)(clock64() - t0) < SH_SPIN_CYCLES) {
            }
            if (kv_armed)
                while (!mbar_try_wait(bkv, kv_phase) && (unsigned long long)(clock64() - t0) < 2 * SH_SPIN_CYCLES) {
                }
            if (!q_landed)
                while (!mbar_try_wait(bq, 0) && (unsigned long long)(clock64() - t0) < 3 * SH_SPIN_CYCLES) {
                }
        }
    } else {
        // ---------------- softmax + output (warps 1..4) ----------------
        const uint32_t quarter = warp & 3u;
        const uint32_t r = quarter * 32 + lane;                 // query row within the tile
        const uint32_t lane_addr = tmem + ((quarter * 32u) << 16);
        float o[kTcDh];
#pragma unroll
        for (int d = 0; d < kTcDh; ++d) o[d] = 0.f;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (uint32_t j = 0; j < a.nkb; ++j) {
            const uint32_t ph = j & 1u;
            if (!mbar_wait(bs, ph, abort, a.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int32_t valid = (int32_t)a.S - (int32_t)(j * kTcKeys);   // keys of this block inside the sequence
            // pass 1: row max of the scaled scores
            float mb = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < kTcKeys / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(lane_addr + c * 32, v);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (c * 32 + i < valid) mb = fmaxf(mb, __uint_as_float(v[i]) * a.sl2);
            }
            const float mn = fmaxf(m, mb);
            const float alpha = fast_exp2(m - mn);
            // pass 2: p = 2^(s sl2 - mn) -> fp16 into the swizzled P tile; l accumulates the rounded values
            float ls = 0.f;
            uint8_t *prow = sp + r * 128;
#pragma unroll 1
            for (int c = 0; c < kTcKeys / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(lane_addr + c * 32, v);
                tmem_ld_wait();
                uint32_t packed[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int k0 = c * 32 + 2 * i;
                    const float p0 = (k0 < valid) ? fast_exp2(__uint_as_float(v[2 * i]) * a.sl2 - mn) : 0.f;
                    const float p1 = (k0 + 1 < valid) ? fast_exp2(__uint_as_float(v[2 * i + 1]) * a.sl2 - mn) : 0.f;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    const float2 back = __half22float2(hp);
                    ls += back.x + back.y;
                    packed[i] = *reinterpret_cast<const uint32_t *>(&hp);
                }
                // 32 keys = 4 units of 16 B; key unit u (0..15 over the row) lives in half (u >> 3) at unit
                // (u & 7) ^ (r & 7) of row r
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t u = c * 4 + q;
                    uint8_t *dst = prow + (u >> 3) * (kTcRows * 128) + (((u & 7u) ^ (r & 7u)) * 16);
                    *reinterpret_cast<uint4 *>(dst) =
                        make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
                }
            }
            l = l * alpha + ls;
            m = mn;
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bp);
            if (!mbar_wait(bo, ph, abort, a.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < kTcDh / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(lane_addr + kTcKeys + c * 32, v);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha + __uint_as_float(v[i]);
            }
            tc_fence_before();
        }
        const uint32_t row = qb * kTcRows + r;
        if (ok && row < a.S) {
            const float inv = 1.f / l;
            __half *dst = a.o + ((size_t)b * a.S + row) * a.ldo + (size_t)h * kTcDh;
#pragma unroll
            for (int q = 0; q < kTcDh / 8; ++q) {
                uint4 out;
                __half2 *hh = reinterpret_cast<__half2 *>(&out);
#pragma unroll
                for (int i = 0; i < 4; ++i) hh[i] = __floats2half2_rn(o[8 * q + 2 * i] * inv, o[8 * q + 2 * i + 1] * inv);
                *reinterpret_cast<uint4 *>(dst + 8 * q) = out;
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kAttnTmemCols);
    }
}

}  // namespace

namespace sh {
int attention_tc_launch(const __half *q, const __half *k, const __half *v, __half *o, uint32_t S, uint32_t H,
                        uint32_t dh, uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t B,
                        bool *launched) {
    *launched = false;
    if (dh != kTcDh || !aligned16((uint64_t)q) || !aligned16((uint64_t)k) || !aligned16((uint64_t)v) ||
        !aligned16((uint64_t)o) || ldq % 8 || ldk % 8 || ldv % 8 || ldo % 8 || !encode_tiled())
        return 0;   // the CUDA-core kernel handles it
    const uint64_t cols_q = (uint64_t)H * dh;
    CUtensorMap mq, mk, mv;
    if (!make_map_3d(&mq, q, B, S, cols_q, ldq, (uint64_t)S * ldq, kTcRows, kTcDh) ||
        !make_map_3d(&mk, k, B, S, cols_q, ldk, (uint64_t)S * ldk, kTcKeys, kTcDh) ||
        !make_map_3d(&mv, v, B, S, cols_q, ldv, (uint64_t)S * ldv, kTcKeys, kTcDh))
        return 0;
    static bool attr_done[kMaxDevices] = {};
    const int dev = current_device() % kMaxDevices;
    if (!attr_done[dev]) {
        if (!cuda_ok(cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnSmem),
                     "cudaFuncSetAttribute(attention)"))
            return -1;
        attr_done[dev] = true;
    }
    AttnArgs a;
    a.o = o;
    a.S = S;
    a.ldo = ldo;
    a.nkb = (S + kTcKeys - 1) / kTcKeys;
    a.sl2 = scale * 1.4426950408889634f;
    a.err = state().dev_err;
    dim3 grid((S + kTcRows - 1) / kTcRows, H, B);
    if (grid.y > 65535u || grid.z > 65535u) return 0;
    k_attn_tc<<<grid, 160, kAttnSmem, stream()>>>(mq, mk, mv, a);
    *launched = true;
    return cuda_ok(cudaGetLastError(), "sh_attention") ? 0 : -1;
}
}  // namespace sh
