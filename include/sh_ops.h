/* sh_ops.h -- C ABI of libsh_ops_cuda.so, the B200 (sm_100a) build of the softhier-ops operator library.
 *
 * Drop-in for the hot-path part of the reference header runtime/sh_ops.h (runwangdl/softhier-mlir): every
 * declaration below keeps the reference's name, argument order, types and return convention, and cites the
 * line it replaces. Generated programs (softhier_cuda.emit_cuda, the reference's emit_c.py template) and the C
 * tests include this header unchanged and link against libsh_ops_cuda.so.
 *
 * Execution model on the GPU (replaces sh_ops.h:3-12):
 *  - one host thread per GPU calls each op ONCE (not SPMD on every core); `cluster` arguments are accepted and
 *    every value runs on the whole GPU;
 *  - tensors are fp16 row-major in device memory, addressed by 64-bit byte addresses (device pointers);
 *    sh_hbm_addr(off) = base of the HBM arena + off (the arena is caller-owned memory bound with
 *    sh_cuda_set_arena, or allocated by sh_init when none was bound);
 *  - ops are asynchronous on the library's stream (sh_cuda_set_stream); sh_barrier_global() synchronises it;
 *  - constraint violations return <0 and print one "[sh_...] reason" line, exactly as the reference does;
 *    asynchronous CUDA failures are reported by sh_cuda_last_error() (sh_ops_cuda.h). Nothing aborts the
 *    process or traps the device.
 * Reference symbols outside the hot path (sh_l1_*, sh_redmule, sh_dma_*, sh_x_*, sh_t_*, sh_f_*, sh_wm_*)
 * are not exported by this library. The sh_llm decoder ops (sh_ops.h:277-303) are, and are declared below.
 */
#ifndef SH_OPS_H
#define SH_OPS_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- runtime wrappers (sh_ops.h:20-37) ------------------------------------------------------------------ */
void     sh_init(void);                 /* sh_ops.h:20  bind/allocate the arena, create the context */
void     sh_barrier_global(void);       /* sh_ops.h:21  synchronise the library stream */
void     sh_barrier_cluster(void);      /* sh_ops.h:22  same as sh_barrier_global */
uint32_t sh_cluster_id(void);           /* sh_ops.h:23  always 0 */
uint32_t sh_core_id(void);              /* sh_ops.h:24  always 0 */
int      sh_is_first_core(void);        /* sh_ops.h:25  always 1: the one host thread */
int      sh_is_dm_core(void);           /* sh_ops.h:26  always 1 */
uint32_t sh_num_clusters(void);         /* sh_ops.h:27  always 1 (the whole GPU is one "cluster") */
void     sh_timer_start(void);          /* sh_ops.h:28  CUDA event on the library stream */
void     sh_timer_end(void);            /* sh_ops.h:29  prints "[Performance Counter]: Execution period is N ns" */
void     sh_eoc(uint32_t val);          /* sh_ops.h:30  synchronises; nothing else to signal */
uint32_t sh_cycles(void);               /* sh_ops.h:31  ns since sh_init after a stream sync (1 GHz convention) */
void     sh_printf(const char *fmt, ...);          /* sh_ops.h:32 */
uint64_t sh_hbm_addr(uint64_t byte_offset);        /* sh_ops.h:33 */
uint64_t sh_hbm_malloc(uint32_t bytes);            /* sh_ops.h:34  carved from the arena's end, 256 B aligned */
uint32_t sh_l1_size(void);                         /* sh_ops.h:35  opt-in shared memory per CTA */
void     sh_preload_wait(uint64_t sentinel);       /* sh_ops.h:36  host preloads are synchronous: a stream sync */

#define SH_ALL 0xFFFFFFFFu                          /* sh_ops.h:39 */
#define SH_CORE_STACK_BYTES 40960u                  /* sh_ops.h:47 */
void sh_call_on_core_stack(void (*fn)(void), uint32_t bytes_per_core);   /* sh_ops.h:48  calls fn() */
#define SH_SELF (sh_cluster_id())                   /* sh_ops.h:308 */

/* ---- formats + GEMM (sh_ops.h:50-88) ------------------------------------------------------------------- */
enum sh_fmt { SH_FP16 = 0, SH_FP8 = 1, SH_INT16 = 2, SH_INT8 = 3 };   /* sh_ops.h:51; only SH_FP16 runs here */

typedef struct {                /* sh_ops.h:54-60; tm/tn/tk are checked like the reference, then used as hints */
    uint32_t tm, tn, tk;
    uint32_t pipeline;
    uint32_t accumulate;        /* 1: Z += X.W */
    uint32_t fmt;
    uint32_t l1_base;
} sh_gemm_cfg;

/* Z[M,N] (+)= X[M,K] . W[K,N], fp32 accumulation on tcgen05 (sh_ops.h:62-67). 0, -1 shape, -2 budget, -3 fmt. */
int sh_gemm(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K,
            uint32_t ldx, uint32_t ldw, uint32_t ldz, const sh_gemm_cfg *cfg, uint32_t cluster);
/* The mesh SUMMA schedule of sh_ops.h:69-73 called from one process: same result as sh_gemm on this GPU
 * (tm == tn required). The multi-GPU block-distributed SUMMA is sh_cuda_summa_* in sh_ops_cuda.h. */
int sh_gemm_mesh(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K,
                 uint32_t ldx, uint32_t ldw, uint32_t ldz, const sh_gemm_cfg *cfg);
enum { SH_XM_AUTO = 0, SH_XM_PANEL = 1, SH_XM_WHOLE = 2 };           /* sh_ops.h:80 */
/* Small-M GEMM (sh_ops.h:75-85): the split-K tcgen05 path; cfg->tm = rows per block must divide M. */
int sh_gemm_xmcast(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K,
                   uint32_t ldx, uint32_t ldw, uint32_t ldz, const sh_gemm_cfg *cfg);
int sh_gemm_xmcast_ex(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K,
                      uint32_t ldx, uint32_t ldw, uint32_t ldz, const sh_gemm_cfg *cfg, uint32_t mode);
uint32_t sh_gemm_xmcast_l1_bytes(uint32_t M, uint32_t N, uint32_t K, const sh_gemm_cfg *cfg, uint32_t mode);
/* sh_ops.h:88: shared memory bytes per CTA of the tile configuration this library picks for the shape. */
uint32_t sh_gemm_l1_bytes(uint32_t M, uint32_t N, uint32_t K, const sh_gemm_cfg *cfg);

/* ---- row-wise / elementwise ops (sh_ops.h:90-100) --------------------------------------------------------
 * One warp per row, fp32 math, fp16 RNE stores, 16-byte vector I/O when addresses and ld allow (else an
 * element-wise path). Outputs may alias inputs. Parameter rows (gamma, beta, bias) are 1 x cols. */
void sh_layernorm(uint64_t y, uint64_t x, uint64_t gamma, uint64_t beta, uint32_t rows, uint32_t cols, uint32_t ld, float eps, uint32_t cluster);
void sh_softmax_rows(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, float scale, uint32_t cluster);
void sh_gelu(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t cluster);
void sh_add(uint64_t y, uint64_t a, uint64_t b, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t cluster);
void sh_add_bias(uint64_t y, uint64_t x, uint64_t bias_row, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t cluster);
void sh_scale(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, float s, uint32_t cluster);
void sh_transpose(uint64_t dst, uint64_t src, uint32_t rows, uint32_t cols, uint32_t ld_src, uint32_t ld_dst, uint32_t cluster);

/* ---- fused attention (sh_ops.h:102-127) ------------------------------------------------------------------
 * o = softmax(scale q k^T) v per head (head h = columns [h dh, (h+1) dh)), flash-style with an online softmax
 * (no bound on S); dh = 64 runs on tcgen05, other dh <= 128 on CUDA cores. The reference's divisibility rules
 * (S % 4, dh % 4, sq | S, sq % 4) are kept; `sq` is otherwise a hint. Returns 0 or -1 (reason printed). */
int sh_attention_head(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t dh,
                      uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t cluster);
int sh_attention_q(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t D, uint32_t H,
                   uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t cluster, uint32_t sq);
int sh_attention(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t D, uint32_t H,
                 uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint32_t cluster);
uint32_t sh_attention_l1_bytes_q(uint32_t S, uint32_t dh, uint32_t sq);   /* shared memory per CTA of this library */
uint32_t sh_attention_l1_bytes(uint32_t S, uint32_t dh);
uint32_t sh_attention_q_block(uint32_t S, uint32_t dh, uint32_t H, uint32_t P);   /* the reference's rule, 1 MB TCDM */
uint32_t sh_attention_profile(uint32_t S, uint32_t dh, uint32_t phase);   /* no per-phase stamps here: 0 */

/* ---- Llama-style decoder ops (sh_ops.h:277-304; runtime/sh_llm.inc.c) --------------------------------------
 * Token masks: one uint16 class per position; query i attends key j iff tok[j] <= tok[i] (unsigned), SH_LLM_PAD
 * marks padding, a PAD query row gets uniform probabilities. fp16 tensors, cols % 4 == 0 as in the reference. */
#define SH_LLM_PAD 0xFFFFu                                                                  /* sh_ops.h:283 */
void sh_rmsnorm(uint64_t y, uint64_t x, uint64_t gamma, uint32_t rows, uint32_t cols, uint32_t ld, float eps,
                uint32_t cluster);                                                          /* sh_ops.h:284 */
void sh_rope(uint64_t y, uint64_t x, uint64_t cos_sin, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t ld_table,
             uint32_t dh, uint32_t cluster);                                                /* sh_ops.h:288 */
void sh_silu_mul(uint64_t y, uint64_t a, uint64_t b, uint32_t rows, uint32_t cols, uint32_t ld,
                 uint32_t cluster);                                                         /* sh_ops.h:289 */
void sh_softmax_masked(uint64_t y, uint64_t x, uint32_t rows, uint32_t cols, uint32_t ld, float scale,
                       uint64_t tok_q, uint64_t tok_k, uint32_t cluster);                   /* sh_ops.h:292 */
int sh_attention_head_masked(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t dh, uint32_t ldq,
                             uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint64_t tok,
                             uint32_t cluster);                                             /* sh_ops.h:294-295 */
int sh_attention_gqa(uint64_t q, uint64_t k, uint64_t v, uint64_t o, uint32_t S, uint32_t D, uint32_t H, uint32_t Hkv,
                     uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo, float scale, uint64_t tok,
                     uint32_t cluster);                                                     /* sh_ops.h:299-300 */
void sh_pixel_shuffle(uint64_t dst, uint64_t src, uint32_t grid, uint32_t D, uint32_t s,
                      uint32_t cluster);                                                    /* sh_ops.h:303 */

/* ---- test helpers (sh_ops.h:220-240) ---------------------------------------------------------------------- */
void sh_test_fill_int_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, int lo, int hi);
void sh_test_fill_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, int lo, int hi, float scale);
void sh_test_dump_samples(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, uint32_t nsamples, const char *tag);
void sh_test_dump_samples_idx(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t seed, uint32_t nsamples, const char *tag, uint32_t idx);
uint32_t sh_test_check_gemm(uint64_t x, uint64_t w, uint64_t z, uint32_t M, uint32_t N, uint32_t K,
                            uint32_t ldx, uint32_t ldw, uint32_t ldz, uint32_t nsamples, float tol,
                            float z0, const char *tag);
void     sh_test_fill_const_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t bits);
void     sh_test_fill_colparity_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t even, uint32_t odd);
uint32_t sh_test_check_const_fp16(uint64_t a, uint32_t rows, uint32_t cols, uint32_t ld, uint32_t bits, uint32_t tol, const char *tag);
float    sh_fp16_to_f32(uint16_t h);                 /* sh_ops.h:239, host */
uint16_t sh_f32_to_fp16(float f);                    /* sh_ops.h:240, host, RNE */

#ifdef __cplusplus
}
#endif
#endif /* SH_OPS_H */
