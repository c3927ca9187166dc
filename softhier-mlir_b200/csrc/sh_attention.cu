// Fused multi-head attention of the operator library: o = softmax(scale q k^T) v per head
// (reference: runtime/sh_attention.inc.c:41-243; declared at runtime/sh_ops.h:102-127).
//
// The reference keeps a whole sq x S score block in one cluster's TCDM (no online softmax), so S is bounded by
// L1. Here attention is flash-style with an online softmax, so S is unbounded:
//   - k_attn_tc (sm_100a tensor cores, dh = 64): persistent, one CTA per SM over (sequence, head, 256 query rows)
//     items; Q/K/V tiles come in by TMA, S = Q K^T accumulates in tensor memory (tcgen05.mma), the softmax runs in
//     registers from tcgen05.ld, P (fp16) goes to shared memory and O += P V accumulates in tensor memory;
//   - k_attn_simt: CUDA-core fallback for other head widths and unaligned operands.
#include <math.h>
#include <string.h>

#include <algorithm>

#include "sh_internal.cuh"

namespace sh {
int attention_tc_launch(const __half *q, const __half *k, const __half *v, __half *o, uint32_t S, uint32_t H,
                        uint32_t dh, uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t B,
                        uint32_t kv_group, bool *launched);
}

namespace {

constexpr int kSimtRows = 128;   // query rows per CTA (one per thread)
constexpr int kSimtKeys = 32;    // keys staged per step

// kv_group query heads share one key/value head (grouped-query attention; 1 = multi-head). tok (nullable): one
// uint16 class per position, query i attends key j iff tok[j] <= tok[i], a PAD (0xFFFF) query row averages every
// value row (sh_ops.h:277-300).
template <int DH>
__global__ void __launch_bounds__(kSimtRows) k_attn_simt(const __half *q, const __half *k, const __half *v, __half *o,
                                                         uint32_t S, uint32_t dh, uint32_t ldq, uint32_t ldk,
                                                         uint32_t ldv, uint32_t ldo, float scale_log2,
                                                         uint32_t kv_group, const uint16_t *tok) {
    __shared__ float ks[kSimtKeys][DH];
    __shared__ float vs[kSimtKeys][DH];
    __shared__ uint16_t ts[kSimtKeys];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t b = blockIdx.z, h = blockIdx.y;
    const uint32_t row = blockIdx.x * kSimtRows + threadIdx.x;
    const size_t r0 = (size_t)b * S;
    const size_t col0 = (size_t)h * dh, kcol0 = (size_t)(h / kv_group) * dh;
    const uint32_t tq = (tok && row < S) ? tok[r0 + row] : 0u;
    const bool pad_row = tok && tq == 0xFFFFu;
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
            ks[j][d] = in ? __half2float(k[(r0 + kt + j) * ldk + kcol0 + d]) : 0.f;
            vs[j][d] = in ? __half2float(v[(r0 + kt + j) * ldv + kcol0 + d]) : 0.f;
        }
        if (tok && threadIdx.x < kSimtKeys) ts[threadIdx.x] = (kt + threadIdx.x < S) ? tok[r0 + kt + threadIdx.x] : 0;
        __syncthreads();
        const uint32_t nk = min((uint32_t)kSimtKeys, S - kt);
        float s[kSimtKeys];
        float tmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < kSimtKeys; ++j) {
            float t = 0.f;
#pragma unroll
            for (int d = 0; d < DH; ++d) t += qr[d] * ks[j][d];
            if (pad_row) t = 0.f;                                   // uniform over every key
            else if (tok && ts[j] > tq) t = -INFINITY;              // key class above the query's
            s[j] = (j < (int)nk) ? t : -INFINITY;
            tmax = fmaxf(tmax, s[j]);
        }
        const float mn = fmaxf(m, tmax);
        const float mref = (mn == -INFINITY) ? 0.f : mn;   // no attendable key yet (masked block): p = 0
        const float corr = exp2f(m - mref);
        l *= corr;
#pragma unroll
        for (int d = 0; d < DH; ++d) acc[d] *= corr;
#pragma unroll
        for (int j = 0; j < kSimtKeys; ++j) {
            const float p = exp2f(s[j] - mref);
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
        uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t B, uint32_t kv_group = 1,
        uint64_t tok = 0, const char *name = "sh_attention") {
    if (S == 0 || H == 0 || B == 0) return 0;
    if (!q || !k || !v || !o) {
        sh::set_error(-1, "[%s] null operand", name);
        return -1;
    }
    if (!tok) {   // the tensor-core kernel has no token mask
        bool launched = false;
        const int rc = sh::attention_tc_launch((const __half *)q, (const __half *)k, (const __half *)v, (__half *)o,
                                               S, H, dh, ldq, ldk, ldv, ldo, scale, B, kv_group, &launched);
        if (launched || rc) return rc;
    }
    const float sl2 = scale * 1.4426950408889634f;
    dim3 grid((S + kSimtRows - 1) / kSimtRows, H, B);
    if (grid.y > 65535u || grid.z > 65535u) {
        sh::set_error(-1, "[%s] H=%u B=%u too large", name, H, B);
        return -1;
    }
    cudaStream_t st = sh::stream();
#define SH_ATTN_SIMT(DHT)                                                                                        \
    sh::launch_pdl(k_attn_simt<DHT>, grid, dim3(kSimtRows), 0, st, (const __half *)q, (const __half *)k,      \
                   (const __half *)v, (__half *)o, S, dh, ldq, ldk, ldv, ldo, sl2, kv_group, (const uint16_t *)tok)
    if (dh <= 16)
        SH_ATTN_SIMT(16);
    else if (dh <= 32)
        SH_ATTN_SIMT(32);
    else if (dh <= 64)
        SH_ATTN_SIMT(64);
    else if (dh <= 128)
        SH_ATTN_SIMT(128);
    else {
        sh::set_error(-1, "[%s] dh=%u > 128 is not supported", name, dh);
        return -1;
    }
#undef SH_ATTN_SIMT
    return sh::cuda_ok(cudaGetLastError(), name) ? 0 : -1;
}

}  // namespace

extern "C" {

uint32_t sh_attention_l1_bytes_q(uint32_t S, uint32_t dh, uint32_t sq) {
    (void)S;
    (void)sq;
    // the tensor-core kernel (dh = 64): two Q slots of two 128 x 64 tiles, four K/V stages of 128 keys, two
    // 128 x 64 O staging tiles, barriers and alignment; the CUDA-core kernel: one staged block of 32 keys of K and V
    // in fp32
    return dh == 64 ? 4 * 128 * 64 * 2 + 4 * 2 * 128 * 64 * 2 + 2 * 128 * 64 * 2 + 256 + 1024
                    : 2 * kSimtKeys * (dh <= 128 ? dh : 128) * 4;
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

// One head with the decoder token mask (sh_ops.h:294-295, sh_llm.inc.c:258): the reference keeps the head in TCDM
// (S <= 256); here any S.
int sh_attention_head_masked(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t dh, uint32_t ldq,
                             uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint64_t tok, uint32_t) {
    if (check(S, dh, 4)) return -1;
    return run(q, k, v, o, S, 1, dh, ldq, ldk, ldv, ldo, scale, 1, 1, tok, "sh_attention_head_masked");
}

// Grouped-query attention (sh_ops.h:296-300, sh_llm.inc.c:325-340): query head h reads key / value head
// h / (H / Hkv); without a token mask and with dh = 64 it runs on the tensor-core kernel.
int sh_attention_gqa(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t D, uint32_t H, uint32_t Hkv,
                     uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint64_t tok, uint32_t) {
    const uint32_t dh = H ? D / H : 0;
    if (H == 0 || Hkv == 0 || dh * H != D || H % Hkv) {
        sh::set_error(-1, "[sh_attention_gqa] bad D=%u H=%u Hkv=%u", D, H, Hkv);
        return -1;
    }
    if (check(S, dh, 4)) return -1;
    return run(q, k, v, o, S, H, dh, ldq, ldk, ldv, ldo, scale, 1, H / Hkv, tok, "sh_attention_gqa");
}

}  // extern "C"

// ================================================================================================================
// Tensor-core path (dh = 64): a persistent, warp-specialised flash-attention kernel.
// Work item = (sequence b, head h, pair of 128-row query tiles); a CTA per SM walks the items. 320 threads:
//   warp 0 (one thread)  : TMA loads: the item's two Q tiles into one of two Q slots, K / V blocks of 128 keys into
//                          a 4-stage ring (separate `full` barriers for K and V, one `empty` barrier per stage);
//   warp 1 (lane 0)      : tcgen05.mma issue (the whole warp walks the loop, lane 0 issues). Per key block g:
//                          S_t = Q_t K^T (M=128, N=128, K=64) for both tiles t into tensor memory as soon as each
//                          softmax holds its previous scores, then (one block
//                          behind, so the next scores are ready when a softmax finishes) O_t (+)= P_t V (M=128, N=64,
//                          K=128; P from tensor memory, V MN-major from shared memory). (One issuer thread per tile measured
//                          6 % slower at B = 512, S = 256.)
//   warps 2..5 / 6..9    : softmax of tile 0 / 1, one query row per thread (warp w reads TMEM lanes 32 (w % 4) ..).
//                          The 128 scores of a block are loaded into registers at once (S is free for the next block
//                          right after), the running max m is only raised when a block's max exceeds it by more than
//                          8 (log2 units; P <= 2^8 then, exact in fp16), in which case O (in tensor memory) is
//                          rescaled before the next P V accumulates. P = 2^(s sl2 - m) goes to tensor memory as fp16
//                          pairs (tcgen05.st; no shared-memory traffic for P); l sums P in fp32. At the end of an item
//                          O / l is staged (128-byte swizzle) in shared memory and leaves by a TMA store.
// Q/K/V/O are addressed through 3-D tensor maps [sequence, row, column]: rows past the end of a sequence read as zero
// and are not written; keys past the end are masked to -inf. Tensor memory (512 columns): S_0, S_1 (128 each), P_0, P_1
// (64 each), O_0, O_1 (64 each). Shared memory: Q 2 x 32 KB, K/V 4 x 32 KB, O staging 2 x 16 KB.
// ================================================================================================================
namespace {

constexpr int kTcRows = 128, kTcKeys = 128, kTcDh = 64;
constexpr int kKvStages = 4;
constexpr uint32_t kTileBytes = kTcRows * kTcDh * 2;          // 16 KB: one Q, K or V tile, or one O staging tile
constexpr uint32_t kQOff = 0, kKvOff = 4 * kTileBytes, kStgOff = kKvOff + kKvStages * 2 * kTileBytes;
constexpr uint32_t kBarOff = kStgOff + 2 * kTileBytes;
constexpr uint32_t kAttnSmem = kBarOff + 256 + 1024;
// tensor memory columns: S_t (fp32 scores), P_t (fp16 pairs), O_t (fp32 output) of query tile t
constexpr uint32_t kTmS = 0, kTmP = 2 * kTcKeys, kTmO = kTmP + kTcKeys;
constexpr uint32_t kAttnTmemCols = 512;
constexpr uint32_t kAttnThreads = 320;
constexpr float kRescaleLog2 = 8.f;

struct AttnArgs {
    uint32_t S, H, kv_group, nkb, nqp, items;
    float sl2;   // scale * log2(e)
    int *err;
};

__global__ void __launch_bounds__(kAttnThreads, 1)
    k_attn_tc(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
              const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mo, AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    uint8_t *sm = smem_raw + pad;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kBarOff);
    uint64_t *q_full = bars, *q_empty = bars + 2;
    uint64_t *k_full = bars + 4, *v_full = k_full + kKvStages, *kv_empty = v_full + kKvStages;
    uint64_t *s_full = kv_empty + kKvStages, *s_free = s_full + 2, *p_full = s_free + 2, *o_full = p_full + 2;
    uint64_t *mdone = o_full + 2;   // [2], one per issuer
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mdone + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);    // both issuers' commits
            mbar_init(&mdone[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
            mbar_init(&p_full[i], 4);
            mbar_init(&o_full[i], 1);
        }
        for (int i = 0; i < kKvStages; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&kv_empty[i], 1);   // both issuers' commits
        }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kAttnTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // set-up above overlaps the previous kernel (programmatic dependent launch); Q/K/V only after it is done
    pdl_launch_dependents();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            prefetch_tmap(&mq);
            prefetch_tmap(&mk);
            prefetch_tmap(&mv);
            uint32_t qs = 0, qph = 0, st = 0, kph = 0;
            uint32_t q_armed[2] = {2, 2}, kv_armed[kKvStages];
            for (int i = 0; i < kKvStages; ++i) kv_armed[i] = 2;
            bool ok = true;
            for (uint32_t it = blockIdx.x; ok && it < a.items; it += gridDim.x) {
                const uint32_t qp = it % a.nqp, bh = it / a.nqp;
                const int32_t col = (int32_t)((bh % a.H) * kTcDh), b = (int32_t)(bh / a.H);
                const int32_t kcol = (int32_t)(((bh % a.H) / a.kv_group) * kTcDh);   // grouped-query K / V head
                if (!mbar_wait(&q_empty[qs], qph ^ 1u, abort, a.err)) break;
                mbar_arrive_expect_tx(&q_full[qs], 2 * kTileBytes);
                q_armed[qs] = qph;
                uint8_t *q0 = sm + kQOff + qs * 2 * kTileBytes;
                tma_load_3d(q0, &mq, &q_full[qs], col, (int32_t)(qp * 2 * kTcRows), b);
                tma_load_3d(q0 + kTileBytes, &mq, &q_full[qs], col, (int32_t)(qp * 2 * kTcRows + kTcRows), b);
                if (++qs == 2) {
                    qs = 0;
                    qph ^= 1u;
                }
                for (uint32_t j = 0; j < a.nkb; ++j) {
                    if (!mbar_wait(&kv_empty[st], kph ^ 1u, abort, a.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *kt = sm + kKvOff + st * 2 * kTileBytes;
                    mbar_arrive_expect_tx(&k_full[st], kTileBytes);
                    tma_load_3d(kt, &mk, &k_full[st], kcol, (int32_t)(j * kTcKeys), b);
                    mbar_arrive_expect_tx(&v_full[st], kTileBytes);
                    tma_load_3d(kt + kTileBytes, &mv, &v_full[st], kcol, (int32_t)(j * kTcKeys), b);
                    kv_armed[st] = kph;
                    if (++st == kKvStages) {
                        st = 0;
                        kph ^= 1u;
                    }
                }
            }
            // drain: every armed load must have landed before the CTA may exit
            for (int i = 0; i < 2; ++i)
                if (q_armed[i] != 2) drain_wait(&q_full[i], q_armed[i]);
            for (int i = 0; i < kKvStages; ++i)
                if (kv_armed[i] != 2) {
                    drain_wait(&k_full[i], kv_armed[i]);
                    drain_wait(&v_full[i], kv_armed[i]);
                }
        }
    } else if (warp == 1) {
        {
            // ---------------- MMA issuer: the whole warp walks the loop, lane 0 issues (is0) ----------------
            const uint32_t is0 = lane == 0 ? 1u : 0u;
            constexpr uint32_t idesc_s = umma_idesc_f16(kTcRows, kTcKeys, 0, 0);
            constexpr uint32_t idesc_o = umma_idesc_f16(kTcRows, kTcDh, 0, 1);
            uint32_t qs = 0, qph = 0, st = 0, kph = 0, g = 0;
            // the P V of the previous block: its stage, block counter and whether it opens an item
            bool have_prev = false, prev_first = false;
            uint32_t prev_st = 0, prev_ph = 0, prev_g = 0;
            bool ok = true;
            // descriptors built once; a stage / slot / k-step adds its byte offset / 16 to the 14-bit address field
            // (shared-memory offsets stay below 256 KB, so the sum never carries out of the field)
            const uint64_t kv_desc0 = sw128_desc(smem_u32(sm + kKvOff), 16, 1024);                 // K, stage 0
            const uint64_t v_desc0 = sw128_desc(smem_u32(sm + kKvOff + kTileBytes), 16384, 1024);  // V, stage 0
            const uint64_t q_desc0 = sw128_desc(smem_u32(sm + kQOff), 16, 1024);                   // Q, slot 0
            auto issue_pv = [&](uint32_t pst, uint32_t pph, uint32_t pg, bool first) -> bool {
                if (!mbar_wait(&v_full[pst], pph, abort, a.err)) return false;
                const uint64_t vd = v_desc0 + ((pst * 2 * kTileBytes) >> 4);
#pragma unroll 1
                for (uint32_t t = 0; t < 2; ++t) {
                    if (!mbar_wait(&p_full[t], pg & 1u, abort, a.err)) return false;
                    tc_fence_after();
                    // P_t (128 x 128 keys) from tensor memory: 16 keys = 8 columns per MMA
#pragma unroll
                    for (int k = 0; k < kTcKeys / 16; ++k)
                        umma_f16_ts_if(is0, tmem + kTmO + t * kTcDh, tmem + kTmP + t * (kTcKeys / 2) + k * 8,
                                       vd + (uint64_t)(k * (2048 >> 4)), idesc_o, (first && k == 0) ? 0u : 1u);
                    umma_commit_if(is0, &o_full[t]);
                }
                umma_commit_if(is0, &kv_empty[pst]);
                return true;
            };
            for (uint32_t it = blockIdx.x; ok && it < a.items; it += gridDim.x) {
                const uint64_t qd = q_desc0 + ((qs * 2 * kTileBytes) >> 4);
                for (uint32_t j = 0; j < a.nkb; ++j) {
                    // at an item boundary the previous item's last P V goes first: its softmax waits on it to finish
                    // the item, while the new item's scores are not needed before that
                    if (j == 0 && have_prev) {
                        if (!issue_pv(prev_st, prev_ph, prev_g, prev_first)) {
                            ok = false;
                            break;
                        }
                        have_prev = false;
                    }
                    if ((j == 0 && !mbar_wait(&q_full[qs], qph, abort, a.err)) ||
                        !mbar_wait(&k_full[st], kph, abort, a.err)) {
                        ok = false;
                        break;
                    }
                    const uint64_t kd = kv_desc0 + ((st * 2 * kTileBytes) >> 4);
#pragma unroll 1
                    for (uint32_t t = 0; t < 2 && ok; ++t) {
                        // the softmax of tile t has its previous scores in registers
                        if (!mbar_wait(&s_free[t], (g & 1u) ^ 1u, abort, a.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
#pragma unroll
                        for (int k = 0; k < kTcDh / 16; ++k)
                            umma_f16_ss_if(is0, tmem + kTmS + t * kTcKeys,
                                           qd + (uint64_t)((t * kTileBytes + k * 32) >> 4), kd + (uint64_t)(k * 2),
                                           idesc_s, k > 0 ? 1u : 0u);
                        umma_commit_if(is0, &s_full[t]);
                    }
                    if (!ok) break;
                    if (j + 1 == a.nkb) umma_commit_if(is0, &q_empty[qs]);   // Q slot free once these MMAs complete
                    if (have_prev && !issue_pv(prev_st, prev_ph, prev_g, prev_first)) {
                        ok = false;
                        break;
                    }
                    have_prev = true;
                    prev_first = j == 0;
                    prev_st = st;
                    prev_ph = kph;
                    prev_g = g;
                    ++g;
                    if (++st == kKvStages) {
                        st = 0;
                        kph ^= 1u;
                    }
                }
                if (++qs == 2) {
                    qs = 0;
                    qph ^= 1u;
                }
            }
            if (ok && have_prev) issue_pv(prev_st, prev_ph, prev_g, prev_first);
            // exit path: tensor memory may only be freed once every issued MMA has completed
            umma_commit_if(is0, &mdone[0]);
            if (is0) drain_wait(&mdone[0], 0);
        }
    } else {
        // ---------------- softmax + output (warps 2..5: tile 0, warps 6..9: tile 1) ----------------
        const uint32_t t = (warp - 2u) >> 2;
        const uint32_t quarter = warp & 3u;
        const uint32_t r = quarter * 32 + lane;                  // query row within the tile
        const uint32_t lane_base = tmem + ((quarter * 32u) << 16);
        const uint32_t s_addr = lane_base + kTmS + t * kTcKeys, p_addr = lane_base + kTmP + t * (kTcKeys / 2);
        const uint32_t o_addr = lane_base + kTmO + t * kTcDh;
        uint8_t *stg = sm + kStgOff + t * kTileBytes;     // O staging of tile t: 128 rows x 128 B, 128-byte swizzle
        uint8_t *srow = stg + r * 128;
        uint32_t g = 0;
        bool store_pending = false, ok = true;
        for (uint32_t it = blockIdx.x; ok && it < a.items; it += gridDim.x) {
            float m = -INFINITY, l = 0.f;
            for (uint32_t j = 0; j < a.nkb; ++j, ++g) {
                if (!mbar_wait(&s_full[t], g & 1u, abort, a.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float sc[kTcKeys];
                {
                    uint32_t v0[32], v1[32], v2[32], v3[32];   // four loads in flight, one wait
                    tmem_ld_32x32b_x32(s_addr, v0);
                    tmem_ld_32x32b_x32(s_addr + 32, v1);
                    tmem_ld_32x32b_x32(s_addr + 64, v2);
                    tmem_ld_32x32b_x32(s_addr + 96, v3);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        sc[i] = __uint_as_float(v0[i]);
                        sc[32 + i] = __uint_as_float(v1[i]);
                        sc[64 + i] = __uint_as_float(v2[i]);
                        sc[96 + i] = __uint_as_float(v3[i]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[t]);
                const int32_t valid = (int32_t)a.S - (int32_t)(j * kTcKeys);
                if (valid < kTcKeys) {   // masked keys: s * sl2 = -inf whatever the sign of the scale
                    const float ninf = a.sl2 >= 0.f ? -INFINITY : INFINITY;
#pragma unroll
                    for (int i = 0; i < kTcKeys; ++i)
                        if (i >= valid) sc[i] = ninf;
                }
                // row max of s * sl2: eight independent chains, then a tree (a single chain would serialise 127
                // dependent ops); with a negative scale the largest s * sl2 comes from the smallest s
                float mx[8];
                float mb;
                if (a.sl2 >= 0.f) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) mx[i] = sc[i];
#pragma unroll
                    for (int i = 8; i < kTcKeys; ++i) mx[i & 7] = fmaxf(mx[i & 7], sc[i]);
                    mb = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) mx[i] = sc[i];
#pragma unroll
                    for (int i = 8; i < kTcKeys; ++i) mx[i & 7] = fminf(mx[i & 7], sc[i]);
                    mb = fminf(fminf(fminf(mx[0], mx[1]), fminf(mx[2], mx[3])),
                               fminf(fminf(mx[4], mx[5]), fminf(mx[6], mx[7])));
                }
                mb *= a.sl2;
                // P V of the previous block is done: P's buffer and O may be touched
                if (j > 0 && !mbar_wait(&o_full[t], (g - 1u) & 1u, abort, a.err)) {
                    ok = false;
                    break;
                }
                float alpha = 1.f;
                bool raise = false;
                if (j == 0) {
                    m = mb;
                } else if (mb > m + kRescaleLog2) {
                    raise = true;
                    alpha = fast_exp2(m - mb);
                    l *= alpha;
                    m = mb;
                }
                // P = 2^(s sl2 - m) as fp16 pairs into tensor memory (64 columns per row), in four parts of 32 keys
                float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    uint32_t packed[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int k0 = 32 * h + 2 * i;
                        const float x0 = fmaf(sc[k0], a.sl2, -m);
                        const float x1 = fmaf(sc[k0 + 1], a.sl2, -m);
                        const float p0 = fast_exp2(x0);
                        const float p1 = fast_exp2(x1);
                        ls8[(2 * i) & 7] += p0;
                        ls8[(2 * i + 1) & 7] += p1;
                        const __half2 hp = __floats2half2_rn(p0, p1);
                        packed[i] = *reinterpret_cast<const uint32_t *>(&hp);
                    }
                    tmem_st_32x32b_x16(p_addr + 16 * h, packed);
                }
                l += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
                if (__any_sync(0xffffffffu, raise)) {   // O *= alpha before the next P V accumulates into it
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < kTcDh / 32; ++c) {
                        uint32_t v[32];
                        tmem_ld_32x32b_x32(o_addr + c * 32, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                        tmem_st_32x32b_x32(o_addr + c * 32, v);
                    }
                }
                tmem_st_wait();   // P (and a rescaled O) in tensor memory before the MMA may read it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[t]);
            }
            if (!ok) break;
            // ---- item epilogue: O / l -> fp16, staged in this warp's 32 rows of the staging tile, one TMA store ----
            if (!mbar_wait(&o_full[t], (g - 1u) & 1u, abort, a.err)) break;
            tc_fence_after();
            if (store_pending) {   // the previous item's O is still being read out of the staging rows
                if (lane == 0) bulk_wait_read0();
                __syncwarp();
            }
            const float inv = 1.f / l;
#pragma unroll
            for (int c = 0; c < kTcDh / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(o_addr + c * 32, v);
                tmem_ld_wait();
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint4 out;
                    __half2 *hh = reinterpret_cast<__half2 *>(&out);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        hh[i] = __floats2half2_rn(__uint_as_float(v[8 * q + 2 * i]) * inv,
                                                  __uint_as_float(v[8 * q + 2 * i + 1]) * inv);
                    const uint32_t u = c * 4 + q;
                    *reinterpret_cast<uint4 *>(srow + ((u ^ (r & 7u)) * 16)) = out;
                }
            }
            tc_fence_before();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                const uint32_t qp = it % a.nqp, bh = it / a.nqp;
                tma_store_3d(&mo, stg + quarter * 32 * 128, (int32_t)((bh % a.H) * kTcDh),
                             (int32_t)(qp * 2 * kTcRows + t * kTcRows + quarter * 32), (int32_t)(bh / a.H));
                bulk_commit();
            }
            store_pending = true;
        }
        if (lane == 0) bulk_wait_all();
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kAttnTmemCols);
    }
}

}  // namespace

namespace sh {
int attention_tc_launch(const __half *q, const __half *k, const __half *v, __half *o, uint32_t S, uint32_t H,
                        uint32_t dh, uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t B,
                        uint32_t kv_group, bool *launched) {
    *launched = false;
    if (dh != kTcDh || !aligned16((uint64_t)q) || !aligned16((uint64_t)k) || !aligned16((uint64_t)v) ||
        !aligned16((uint64_t)o) || ldq % 8 || ldk % 8 || ldv % 8 || ldo % 8 || !encode_tiled())
        return 0;   // the CUDA-core kernel handles it
    const uint64_t cols_q = (uint64_t)H * dh, cols_kv = (uint64_t)(H / kv_group) * dh;
    CUtensorMap mq, mk, mv, mo;
    if (!make_map_3d(&mq, q, B, S, cols_q, ldq, (uint64_t)S * ldq, kTcRows, kTcDh) ||
        !make_map_3d(&mk, k, B, S, cols_kv, ldk, (uint64_t)S * ldk, kTcKeys, kTcDh) ||
        !make_map_3d(&mv, v, B, S, cols_kv, ldv, (uint64_t)S * ldv, kTcKeys, kTcDh) ||
        !make_map_3d(&mo, o, B, S, cols_q, ldo, (uint64_t)S * ldo, 32, kTcDh))
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
    a.S = S;
    a.H = H;
    a.kv_group = kv_group;
    a.nkb = (S + kTcKeys - 1) / kTcKeys;
    a.nqp = (S + 2 * kTcRows - 1) / (2 * kTcRows);
    const uint64_t items = (uint64_t)B * H * a.nqp;
    if (items > 0xffffffffull) return 0;
    a.items = (uint32_t)items;
    a.sl2 = scale * 1.4426950408889634f;
    a.err = state().dev_err;
    const uint32_t grid = (uint32_t)std::min<uint64_t>(items, (uint64_t)state().num_sms);
    *launched = true;
    return cuda_ok(launch_pdl(k_attn_tc, dim3(grid), dim3(kAttnThreads), kAttnSmem, stream(), mq, mk, mv, mo, a),
                   "sh_attention")
               ? 0
               : -1;
}
}  // namespace sh
