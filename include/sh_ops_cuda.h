/* sh_ops_cuda.h -- extensions of libsh_ops_cuda.so beyond the reference header (runtime/sh_ops.h).
 *
 * They have no counterpart in the reference: they expose what a GPU backend needs and a RISC-V cluster did not
 * (caller-owned device memory, streams, asynchronous error state) and the fused / batched forms of the hot-path
 * ops that the encoder driver uses (GEMM epilogues, residual + LayerNorm, attention over a batch of sequences).
 * All pointers are device pointers passed as uint64_t, sizes and leading dimensions are in elements, like the
 * reference ABI.
 */
#ifndef SH_OPS_CUDA_H
#define SH_OPS_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- runtime ------------------------------------------------------------------------------------------------
 * Bind caller-owned device memory (e.g. a torch tensor's data_ptr) as the HBM arena of the current device;
 * the library never frees it. Returns 0, or -1 when base is NULL / not 256-byte aligned. */
int      sh_cuda_set_arena(void *base, size_t bytes);
void    *sh_cuda_arena_base(void);
size_t   sh_cuda_arena_bytes(void);
/* All ops of the calling thread's current device are enqueued on this stream (a cudaStream_t; NULL = the
 * legacy default stream). */
int      sh_cuda_set_stream(void *stream);
void    *sh_cuda_get_stream(void);
int      sh_cuda_synchronize(void);                 /* stream sync; returns the cudaError_t code */
int      sh_cuda_last_error(void);                  /* first error recorded since the previous call, then cleared */
const char *sh_cuda_last_error_string(void);        /* text of that error ("" when none) */
int      sh_cuda_device_error(void);                /* syncs, returns and clears the kernels' error word (1 = a
                                                       bounded wait gave up) */
int      sh_cuda_num_sms(void);
float    sh_cuda_timer_last_ms(void);               /* the period the last sh_timer_end printed */
uint32_t sh_cuda_abi_version(void);                 /* 1 */

/* ---- GEMM with fused epilogue ---------------------------------------------------------------------------------
 * Z[M,N] = epi(X[M,K] . W[K,N]) with fp32 accumulation, fp16 out. `flags`:
 *   SH_EPI_ACCUMULATE  t = acc + Z_old           (sh_gemm_cfg.accumulate)
 *   SH_EPI_BIAS        t = t + bias[col]         (bias: 1 x N fp16)
 *   SH_EPI_GELU        t = gelu_tanh(t)          (after the bias)
 *   SH_EPI_RESIDUAL    t = t + R[row, col]       (R: M x N fp16, leading dim ldr)
 *   SH_EPI_F32_OUT     Z is fp32 (ldz in fp32 elements; SH_EPI_ACCUMULATE then reads fp32 Z)
 *   SH_EPI_ACC_F32_IN  t = t + R32[row, col] with R32 an fp32 matrix passed as `residual` (leading dim ldr);
 *                      not combined with SH_EPI_RESIDUAL. Together with SH_EPI_F32_OUT this carries a K-split
 *                      product in fp32 across calls (the SUMMA panels) and rounds it to fp16 once.
 *   SH_GEMM_SIMT       use the CUDA-core fallback kernel (tests)
 * splits: 0 = library choice of split-K, 1 = none, n = K split n ways (partials reduced in a fixed order).
 * Returns 0 or -1 (reason printed). */
#define SH_EPI_ACCUMULATE 0x1u
#define SH_EPI_BIAS       0x2u
#define SH_EPI_GELU       0x4u
#define SH_EPI_RESIDUAL   0x8u
#define SH_EPI_F32_OUT    0x10u
#define SH_EPI_ACC_F32_IN 0x20u
#define SH_GEMM_SIMT      0x100u
int sh_cuda_gemm(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx, uint32_t ldw,
                 uint32_t ldz, uint64_t bias, uint64_t residual, uint32_t ldr, uint32_t flags, uint32_t splits);

/* ---- the GEMM planner as a query ---------------------------------------------------------------------------------
 * No counterpart in the reference. The kernel and tiling sh_cuda_gemm picks for 16-byte-aligned operands of an
 * M x N x K product with `splits` as in sh_cuda_gemm, on a GPU with `num_sms` SMs (0: the current device's; any
 * other value makes no CUDA call, so the query runs without a GPU):
 *   kernel      0 CUDA-core fallback (K == 0), 1 single-CTA tcgen05 (128 x bn tiles), 2 two-CTA tcgen05 (256 x bn)
 *   k_blocks    64-deep K blocks; splits: K pieces per tile (split-K, single-CTA kernel only)
 *   units       work units of the launch: tiles x splits, or for kernel 2 whole tiles below full_units and
 *               256-column slices of the remaining tiles past it (a short last wave of 256 x 512 tiles)
 *   grid        CTAs launched
 * Returns 0, or -1 when out is NULL. */
typedef struct sh_cuda_gemm_plan_t {
    uint32_t kernel, bn, tiles_m, tiles_n, k_blocks, splits, full_units, units, grid;
} sh_cuda_gemm_plan_t;
int sh_cuda_gemm_plan(uint32_t M, uint32_t N, uint32_t K, uint32_t splits, uint32_t num_sms,
                      sh_cuda_gemm_plan_t *out);

/* ---- GEMM with LayerNorm folded in, and row statistics out ----------------------------------------------------------
 * No counterpart in the reference: the library form of "layernorm -> gemm" (frontend/siglip.py:136-162) without
 * materialising the normalised rows. With W' = diag(gamma) W, colsum = 1^T W' (fp32, 1 x N) and
 * d = beta W + bias (fp16, 1 x N, passed as `bias` with SH_EPI_BIAS),
 *     layernorm(X) W + bias = rstd_r (X W' - mean_r colsum) + d,
 * so the GEMM reads raw X. Flags (in addition to sh_cuda_gemm's):
 *   SH_EPI_LN_IN     t = rstd_r (acc - mean_r colsum[col]) first; mean_r / rstd_r (eps `ln_eps`) come from
 *                    `ln_stats`: K / 64 (sum, sum of squares) fp32 pairs per row, K % 64 == 0
 *   SH_EPI_STATS_OUT write N / 64 (sum, sum of squares) fp32 pairs per row of the final outputs (before fp16
 *                    rounding) to `stats_out`, N % 64 == 0: the next GEMM's ln_stats
 * No split-K; 16-byte aligned operands. Returns 0 or -1 (reason printed). */
#define SH_EPI_LN_IN      0x40u
#define SH_EPI_STATS_OUT  0x80u
int sh_cuda_gemm_ln(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx,
                    uint32_t ldw, uint32_t ldz, uint64_t bias, uint64_t residual, uint32_t ldr, uint32_t flags,
                    uint64_t ln_stats, uint64_t ln_colsum, float ln_eps, uint64_t stats_out);
/* (sum, sum of squares) of every 64 columns of each row of X (cols % 64 == 0): the row statistics of a matrix no
 * GEMM produced (the encoder's input). Returns 0 or -1. */
int sh_cuda_row_stats(uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, uint64_t stats_out);
/* dst[r, c] = src[r, c] * gamma[r] in fp16 (W' = diag(gamma) W for sh_cuda_gemm_ln). Returns 0 or -1. */
int sh_cuda_scale_rows(uint64_t dst, uint64_t src, uint32_t rows, uint32_t cols, uint32_t ld_src, uint32_t ld_dst,
                       uint64_t gamma);

/* ---- split-K GEMM without allocation -------------------------------------------------------------------------
 * No counterpart in the reference. The same computation, arguments and return codes as sh_cuda_gemm, for callers
 * that cannot let the library call cudaMalloc (a host whose own pool owns all device memory, or a loop that cannot
 * take cudaMalloc's implicit device synchronisation). Split-K partial tiles and arrival counters live in one fixed
 * 8 MiB array compiled into the library (held on every GPU that loads it until exit) instead of a growable
 * workspace; a call needing more (tiles x splits x 128 x BN x 4 bytes of partials, or more than 4096 tiles) returns
 * -2. The first call on a device looks the array up with cudaGetSymbolAddress and should come before any stream
 * capture. Calls share the array: calls that overlap on the GPU race and must be serialised by the caller. */
int sh_cuda_gemm_splitk_noalloc(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K, uint32_t ldx,
                                uint32_t ldw, uint32_t ldz, uint64_t bias, uint64_t residual, uint32_t ldr,
                                uint32_t flags, uint32_t splits);

/* ---- fused residual add + LayerNorm ---------------------------------------------------------------------------
 * h = a + b (stored, fp16), y = layernorm(h) * gamma + beta, both rows x cols with leading dim ld. */
void sh_cuda_add_layernorm(uint64_t h, uint64_t y, uint64_t a, uint64_t b, uint64_t gamma, uint64_t beta,
                           uint32_t rows, uint32_t cols, uint32_t ld, float eps);

/* ---- attention over a batch of sequences ------------------------------------------------------------------------
 * B sequences of S rows stacked along the rows of q/k/v/o (sequence b = rows [b S, (b+1) S)); otherwise
 * sh_attention. Returns 0 or -1. */
int sh_cuda_attention_batched(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t D, uint32_t H,
                              uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t B);

/* ---- synthetic inputs -------------------------------------------------------------------------------------------
 * N(mean, std) fp16 from the LCG of sh_test_fill_fp16: per element two draws d0, d1, u = (d + 0.5) / 2^24 and
 * Box-Muller z = sqrt(-2 ln u0) cos(2 pi u1), with ln and cos evaluated as fixed series of correctly rounded fp32
 * operations (no library math, no FMA contraction), so every implementation of the definition gives the same bits.
 * sh_cuda_fill_normal_fp16 fills device memory on the library stream; sh_cuda_host_fill_normal_fp16 fills host
 * memory (fp16 codes) on the calling CPU thread and needs no GPU. */
void sh_cuda_fill_normal_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, float mean,
                              float stdev);
void sh_cuda_host_fill_normal_fp16(uint16_t *dst, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed,
                                   float mean, float stdev);

/* ---- LCG sub-block fill (2-D block-distributed inputs) -----------------------------------------------------------
 * Fill rows x cols (leading dim ld) with elements [row0 .., col0 ..] of the global gcols-wide matrix that
 * sh_test_fill_fp16(.., seed, lo, hi, scale) would produce: every rank generates exactly its own block. */
void sh_cuda_fill_lcg_block(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, int lo, int hi,
                            float scale, uint64_t row0, uint64_t col0, uint64_t gcols);

/* ---- HBM preload images -------------------------------------------------------------------------------------------
 * No counterpart in the reference's C runtime (its simulator loads the image at reset): the ELF32 images of
 * softhier_mlir/sim/preload.py (one PT_LOAD segment per array, physical address hbm_base + HBM offset, hbm_base
 * 0xC0000000 there) copied into the arena at sh_hbm_addr(offset) with synchronous copies; bytes between a
 * segment's file size and memory size are zeroed. Returns the number of segments, -1 (bad file) or -2 (a segment
 * outside the arena). sh_preload_elf_segments only lists the segments (offsets, memory sizes; no GPU needed) and
 * returns their count. */
int sh_cuda_preload_elf(const char *path, uint64_t hbm_base);
int sh_preload_elf_segments(const char *path, uint64_t hbm_base, uint64_t *offsets, uint64_t *sizes,
                            uint32_t max_segments);

/* ---- peer memory for the multi-GPU SUMMA --------------------------------------------------------------------------
 * Device buffers that other processes of the node can map (CUDA IPC), and asynchronous 2-D copies between any two
 * device addresses of the node (copy engines over NVLink when source and destination are on different GPUs). */
void *sh_cuda_ipc_alloc(size_t bytes);                     /* cudaMalloc'd, exportable; NULL on failure */
int   sh_cuda_ipc_free(void *p);
int   sh_cuda_ipc_handle(void *p, void *handle64);          /* 64-byte handle of a sh_cuda_ipc_alloc buffer */
void *sh_cuda_ipc_open(const void *handle64);               /* map a peer's buffer into this process */
int   sh_cuda_ipc_close(void *p);
int   sh_cuda_copy2d(uint64_t dst, size_t dpitch, uint64_t src, size_t spitch, size_t width_bytes, size_t rows,
                     void *stream);

#ifdef __cplusplus
}
#endif
#endif /* SH_OPS_CUDA_H */
