// Runtime of libsh_ops_cuda.so: the reference's runtime wrappers (runtime/sh_rt.inc.c:2-98, declared at
// runtime/sh_ops.h:20-48) mapped onto one CUDA device per host thread, plus the arena / stream / error
// extensions of sh_ops_cuda.h.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <mutex>
#include <vector>

#include "sh_internal.cuh"

namespace sh {

static DeviceState g_state[kMaxDevices];
static std::mutex g_mu;
static thread_local int t_err_code = 0;
static thread_local char t_err_msg[512] = {0};
static float g_last_timer_ms = 0.f;
static long long g_t_init_ns = 0;

static long long now_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (long long)ts.tv_sec * 1000000000ll + ts.tv_nsec;
}

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return d;
}

void set_error(int code, const char *fmt, ...) {
    char buf[480];
    va_list va;
    va_start(va, fmt);
    vsnprintf(buf, sizeof buf, fmt, va);
    va_end(va);
    if (t_err_code == 0) {
        t_err_code = code;
        snprintf(t_err_msg, sizeof t_err_msg, "%s", buf);
    }
    fputs(buf, stdout);
    size_t n = strlen(buf);
    if (n == 0 || buf[n - 1] != '\n') fputc('\n', stdout);
    fflush(stdout);
}

bool cuda_ok(cudaError_t e, const char *where) {
    if (e == cudaSuccess) return true;
    set_error((int)e, "[sh_cuda] %s: %s", where, cudaGetErrorString(e));
    return false;
}

DeviceState &state() {
    const int d = current_device();
    DeviceState &s = g_state[d < kMaxDevices ? d : 0];
    if (!s.ready) {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!s.ready) {
            s.device = d;
            cudaDeviceProp prop;
            if (cuda_ok(cudaGetDeviceProperties(&prop, d), "cudaGetDeviceProperties")) {
                s.num_sms = prop.multiProcessorCount;
                s.smem_optin = prop.sharedMemPerBlockOptin;
            }
            cuda_ok(cudaMalloc(&s.dev_err, sizeof(int)), "cudaMalloc(error word)");
            if (s.dev_err) cuda_ok(cudaMemset(s.dev_err, 0, sizeof(int)), "cudaMemset(error word)");
            cuda_ok(cudaEventCreate(&s.t0), "cudaEventCreate");
            cuda_ok(cudaEventCreate(&s.t1), "cudaEventCreate");
            if (g_t_init_ns == 0) g_t_init_ns = now_ns();
            s.ready = true;
        }
    }
    return s;
}

static bool capturing(cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return cs != cudaStreamCaptureStatusNone;
}

float *workspace(size_t bytes) {
    DeviceState &s = state();
    if (bytes <= s.ws_bytes) return s.ws;
    if (capturing(s.stream)) {
        set_error(-1, "[sh_gemm] split-K workspace of %zu B must be allocated before stream capture", bytes);
        return nullptr;
    }
    cudaStreamSynchronize(s.stream);
    if (s.ws) cudaFree(s.ws);
    s.ws = nullptr;
    s.ws_bytes = 0;
    size_t want = bytes < (size_t)(8u << 20) ? (size_t)(8u << 20) : bytes;
    if (!cuda_ok(cudaMalloc(&s.ws, want), "cudaMalloc(split-K workspace)")) return nullptr;
    s.ws_bytes = want;
    return s.ws;
}

uint32_t *tile_counters(size_t n) {
    DeviceState &s = state();
    if (n <= s.counters_len) return s.counters;
    if (capturing(s.stream)) {
        set_error(-1, "[sh_gemm] split-K counters must be allocated before stream capture");
        return nullptr;
    }
    cudaStreamSynchronize(s.stream);
    if (s.counters) cudaFree(s.counters);
    s.counters = nullptr;
    s.counters_len = 0;
    size_t want = n < 65536 ? 65536 : n;
    if (!cuda_ok(cudaMalloc(&s.counters, want * sizeof(uint32_t)), "cudaMalloc(split-K counters)")) return nullptr;
    if (!cuda_ok(cudaMemset(s.counters, 0, want * sizeof(uint32_t)), "cudaMemset(split-K counters)")) return nullptr;
    s.counters_len = want;
    return s.counters;
}

cudaStream_t peek_stream(int device, int **dev_err) {
    if (device < 0 || device >= kMaxDevices || !g_state[device].ready) {
        *dev_err = nullptr;
        return nullptr;
    }
    *dev_err = g_state[device].dev_err;
    return g_state[device].stream;
}

PFN_encodeTiled encode_tiled() {
    static PFN_encodeTiled fn = nullptr;
    static bool tried = false;
    if (!tried) {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!tried) {
            void *p = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
                q == cudaDriverEntryPointSuccess)
                fn = reinterpret_cast<PFN_encodeTiled>(p);
            else
                cudaGetLastError();
            tried = true;
        }
    }
    return fn;
}

bool make_map_2d(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                 uint32_t box_cols, bool swizzle128) {
    PFN_encodeTiled enc = encode_tiled();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_map_2d_sw(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                    uint32_t box_cols, CUtensorMapSwizzle sw) {
    PFN_encodeTiled enc = encode_tiled();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_3d(CUtensorMap *m, const void *base, uint64_t batches, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint64_t batch_ld, uint32_t box_rows, uint32_t box_cols) {
    PFN_encodeTiled enc = encode_tiled();
    if (!enc) return false;
    cuuint64_t dims[3] = {cols, rows, batches};
    cuuint64_t strides[2] = {ld * 2, batch_ld * 2};
    cuuint32_t box[3] = {box_cols, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace sh

using namespace sh;

extern "C" {

// ---- sh_ops.h runtime wrappers --------------------------------------------------------------------------------
void sh_init(void) {
    DeviceState &s = state();
    if (!s.arena) {
        size_t bytes = 256u << 20;
        if (const char *e = getenv("SH_CUDA_ARENA_BYTES")) bytes = (size_t)strtoull(e, nullptr, 0);
        void *p = nullptr;
        if (cuda_ok(cudaMalloc(&p, bytes), "cudaMalloc(arena)")) {
            cudaMemset(p, 0, bytes);
            s.arena = (char *)p;
            s.arena_bytes = bytes;
            s.arena_owned = true;
            s.malloc_top = bytes;
        }
    }
    cuda_ok(cudaDeviceSynchronize(), "sh_init");
}

void sh_barrier_global(void) { cuda_ok(cudaStreamSynchronize(state().stream), "sh_barrier_global"); }
void sh_barrier_cluster(void) { sh_barrier_global(); }
uint32_t sh_cluster_id(void) { return 0; }
uint32_t sh_core_id(void) { return 0; }
int sh_is_first_core(void) { return 1; }
int sh_is_dm_core(void) { return 1; }
uint32_t sh_num_clusters(void) { return 1; }

void sh_timer_start(void) {
    DeviceState &s = state();
    cuda_ok(cudaEventRecord(s.t0, s.stream), "sh_timer_start");
    s.timer_running = true;
}

void sh_timer_end(void) {
    DeviceState &s = state();
    if (!s.timer_running) return;
    cuda_ok(cudaEventRecord(s.t1, s.stream), "sh_timer_end");
    float ms = 0.f;
    if (cuda_ok(cudaEventSynchronize(s.t1), "sh_timer_end") && cuda_ok(cudaEventElapsedTime(&ms, s.t0, s.t1), "sh_timer_end")) {
        g_last_timer_ms = ms;
        printf("[Performance Counter]: Execution period is %llu ns\n", (unsigned long long)(ms * 1e6 + 0.5));
        fflush(stdout);
    }
    // like the reference's timer: every end restarts the period (rowops/main.c times op after op)
    cuda_ok(cudaEventRecord(s.t0, s.stream), "sh_timer_end");
}

void sh_eoc(uint32_t) { sh_barrier_global(); fflush(stdout); }

uint32_t sh_cycles(void) {
    sh_barrier_global();
    return (uint32_t)(now_ns() - g_t_init_ns);
}

void sh_printf(const char *fmt, ...) {
    va_list va;
    va_start(va, fmt);
    vprintf(fmt, va);
    va_end(va);
    fflush(stdout);
}

uint64_t sh_hbm_addr(uint64_t off) { return (uint64_t)(uintptr_t)state().arena + off; }

uint64_t sh_hbm_malloc(uint32_t bytes) {
    DeviceState &s = state();
    size_t need = ((size_t)bytes + 255) & ~(size_t)255;
    if (!s.arena || need > s.malloc_top) {
        set_error(-1, "[sh_hbm_malloc] %u B do not fit the arena", bytes);
        return 0;
    }
    s.malloc_top -= need;
    return (uint64_t)(uintptr_t)(s.arena + s.malloc_top);
}

uint32_t sh_l1_size(void) { return (uint32_t)state().smem_optin; }
void sh_preload_wait(uint64_t) { sh_barrier_global(); }
void sh_call_on_core_stack(void (*fn)(void), uint32_t) {
    if (fn) fn();
}

// ---- HBM preload images ---------------------------------------------------------------------------------------
// The reference's preload image (softhier_mlir/sim/preload.py: make_preload_elf) is an ELF32 little-endian file
// whose PT_LOAD segments carry raw array bytes at physical address hbm_base + HBM byte offset; GVSoC's loader writes
// them into HBM at reset. Here the same image is copied into the arena (sh_hbm_addr(offset)) with synchronous host
// copies, so the sentinel it ends with is visible as soon as sh_cuda_preload_elf returns.

}  // extern "C"

namespace {

struct Segment {
    uint64_t offset, file_off, filesz, memsz;
};

uint32_t rd32(const unsigned char *p) { return p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24); }
uint16_t rd16(const unsigned char *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// Reads the file and lists its PT_LOAD segments; false (reason recorded) on anything that is not such an image.
bool parse_preload(const char *path, uint64_t hbm_base, const char *who, std::vector<unsigned char> &data,
                   std::vector<Segment> &segs) {
    FILE *f = path ? fopen(path, "rb") : nullptr;
    if (!f) {
        sh::set_error(-1, "[%s] cannot open %s", who, path ? path : "(null)");
        return false;
    }
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    data.resize(n > 0 ? (size_t)n : 0);
    const size_t got = n > 0 ? fread(data.data(), 1, (size_t)n, f) : 0;
    fclose(f);
    const unsigned char *d = data.data();
    if (got != data.size() || data.size() < 52 || memcmp(d, "\x7f" "ELF", 4) != 0 || d[4] != 1 || d[5] != 1) {
        sh::set_error(-1, "[%s] %s is not a little-endian ELF32 image", who, path);
        return false;
    }
    const uint32_t phoff = rd32(d + 28);
    const uint16_t phentsize = rd16(d + 42), phnum = rd16(d + 44);
    if (phentsize < 32 || (uint64_t)phoff + (uint64_t)phnum * phentsize > data.size()) {
        sh::set_error(-1, "[%s] %s: program headers out of the file", who, path);
        return false;
    }
    segs.clear();
    for (uint32_t i = 0; i < phnum; ++i) {
        const unsigned char *ph = d + phoff + (size_t)i * phentsize;
        if (rd32(ph) != 1) continue;   // PT_LOAD only
        const uint64_t fo = rd32(ph + 4), paddr = rd32(ph + 12), fsz = rd32(ph + 16), msz = rd32(ph + 20);
        if (paddr < hbm_base || fo + fsz > data.size() || msz < fsz) {
            sh::set_error(-1, "[%s] %s: segment %u (paddr %#llx, %llu B at file offset %llu) is malformed", who, path,
                          i, (unsigned long long)paddr, (unsigned long long)fsz, (unsigned long long)fo);
            return false;
        }
        segs.push_back(Segment{paddr - hbm_base, fo, fsz, msz});
    }
    return true;
}

}  // namespace

extern "C" {

int sh_preload_elf_segments(const char *path, uint64_t hbm_base, uint64_t *offsets, uint64_t *sizes,
                            uint32_t max_segments) {
    std::vector<unsigned char> data;
    std::vector<Segment> segs;
    if (!parse_preload(path, hbm_base, "sh_preload_elf_segments", data, segs)) return -1;
    for (size_t i = 0; i < segs.size() && i < max_segments; ++i) {
        if (offsets) offsets[i] = segs[i].offset;
        if (sizes) sizes[i] = segs[i].memsz;
    }
    return (int)segs.size();
}

int sh_cuda_preload_elf(const char *path, uint64_t hbm_base) {
    std::vector<unsigned char> data;
    std::vector<Segment> segs;
    if (!parse_preload(path, hbm_base, "sh_cuda_preload_elf", data, segs)) return -1;
    DeviceState &s = state();
    if (!s.arena) {
        set_error(-1, "[sh_cuda_preload_elf] no arena bound (sh_init or sh_cuda_set_arena first)");
        return -1;
    }
    for (const Segment &g : segs)
        if (g.offset + g.memsz > s.arena_bytes) {
            set_error(-2, "[sh_cuda_preload_elf] segment at %#llx (%llu B) is outside the %zu B arena",
                      (unsigned long long)g.offset, (unsigned long long)g.memsz, s.arena_bytes);
            return -2;
        }
    for (const Segment &g : segs) {
        if (g.filesz && !cuda_ok(cudaMemcpy(s.arena + g.offset, data.data() + g.file_off, g.filesz,
                                            cudaMemcpyHostToDevice), "sh_cuda_preload_elf"))
            return -1;
        if (g.memsz > g.filesz &&
            !cuda_ok(cudaMemset(s.arena + g.offset + g.filesz, 0, g.memsz - g.filesz), "sh_cuda_preload_elf"))
            return -1;
    }
    return (int)segs.size();
}

// ---- sh_ops_cuda.h ------------------------------------------------------------------------------------------
int sh_cuda_set_arena(void *base, size_t bytes) {
    if (!base || ((uintptr_t)base & 255u)) {
        set_error(-1, "[sh_cuda_set_arena] base %p must be non-null and 256-byte aligned", base);
        return -1;
    }
    DeviceState &s = state();
    if (s.arena_owned && s.arena) cudaFree(s.arena);
    s.arena = (char *)base;
    s.arena_bytes = bytes;
    s.arena_owned = false;
    s.malloc_top = bytes;
    return 0;
}
void *sh_cuda_arena_base(void) { return state().arena; }
size_t sh_cuda_arena_bytes(void) { return state().arena_bytes; }

int sh_cuda_set_stream(void *st) {
    DeviceState &s = state();
    s.stream = (cudaStream_t)st;
    s.stream_set = true;
    return 0;
}
void *sh_cuda_get_stream(void) { return (void *)state().stream; }

int sh_cuda_synchronize(void) {
    cudaError_t e = cudaStreamSynchronize(state().stream);
    cuda_ok(e, "sh_cuda_synchronize");
    return (int)e;
}

int sh_cuda_last_error(void) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && t_err_code == 0) {
        t_err_code = (int)e;
        snprintf(t_err_msg, sizeof t_err_msg, "[sh_cuda] %s", cudaGetErrorString(e));
    }
    int c = t_err_code;
    t_err_code = 0;
    return c;
}
const char *sh_cuda_last_error_string(void) { return t_err_msg; }

int sh_cuda_device_error(void) {
    DeviceState &s = state();
    int v = 0;
    if (!cuda_ok(cudaStreamSynchronize(s.stream), "sh_cuda_device_error")) return -1;
    if (s.dev_err) {
        if (!cuda_ok(cudaMemcpy(&v, s.dev_err, sizeof v, cudaMemcpyDeviceToHost), "sh_cuda_device_error")) return -1;
        if (v) cudaMemset(s.dev_err, 0, sizeof(int));
    }
    // kernels of sh_cuda_gemm_splitk_noalloc launched before the runtime started report into its fixed array
    const int nv = noalloc_take_error(s.device);
    return v ? v : nv;
}

int sh_cuda_num_sms(void) { return state().num_sms; }

void *sh_cuda_ipc_alloc(size_t bytes) {
    void *p = nullptr;
    if (!cuda_ok(cudaMalloc(&p, bytes), "sh_cuda_ipc_alloc")) return nullptr;
    cudaMemset(p, 0, bytes);
    return p;
}
int sh_cuda_ipc_free(void *p) { return cuda_ok(cudaFree(p), "sh_cuda_ipc_free") ? 0 : -1; }
int sh_cuda_ipc_handle(void *p, void *handle64) {
    cudaIpcMemHandle_t h;
    if (!cuda_ok(cudaIpcGetMemHandle(&h, p), "sh_cuda_ipc_handle")) return -1;
    memcpy(handle64, &h, sizeof h < 64 ? sizeof h : 64);
    return 0;
}
void *sh_cuda_ipc_open(const void *handle64) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof h < 64 ? sizeof h : 64);
    void *p = nullptr;
    if (!cuda_ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "sh_cuda_ipc_open")) return nullptr;
    return p;
}
int sh_cuda_ipc_close(void *p) { return cuda_ok(cudaIpcCloseMemHandle(p), "sh_cuda_ipc_close") ? 0 : -1; }
int sh_cuda_copy2d(uint64_t dst, size_t dpitch, uint64_t src, size_t spitch, size_t width_bytes, size_t rows,
                   void *st) {
    return cuda_ok(cudaMemcpy2DAsync((void *)dst, dpitch, (const void *)src, spitch, width_bytes, rows,
                                     cudaMemcpyDefault, (cudaStream_t)st),
                   "sh_cuda_copy2d")
               ? 0
               : -1;
}
float sh_cuda_timer_last_ms(void) { return g_last_timer_ms; }
uint32_t sh_cuda_abi_version(void) { return 1; }

}  // extern "C"
