"""ctypes binding of libsh_ops_cuda.so (the C ABI declared in include/sh_ops.h and include/sh_ops_cuda.h).

`load()` returns the library with every entry point's argtypes / restype set. It raises if the shared object is
missing: there is no fallback implementation behind this module.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]
LIB_PATH = Path(os.environ.get("SH_OPS_CUDA_LIB", PKG / "lib" / "libsh_ops_cuda.so"))

u32, u64, i32, f32, vp, sz, cp = C.c_uint32, C.c_uint64, C.c_int, C.c_float, C.c_void_p, C.c_size_t, C.c_char_p
u16 = C.c_uint16


class GemmCfg(C.Structure):
    """sh_gemm_cfg (runtime/sh_ops.h:54-60)."""
    _fields_ = [("tm", u32), ("tn", u32), ("tk", u32), ("pipeline", u32), ("accumulate", u32), ("fmt", u32),
                ("l1_base", u32)]


CFG_P = C.POINTER(GemmCfg)


class GemmPlan(C.Structure):
    """sh_cuda_gemm_plan_t (include/sh_ops_cuda.h): the planner's choice for one GEMM shape."""
    _fields_ = [(n, u32) for n in ("kernel", "bn", "tiles_m", "tiles_n", "k_blocks", "splits", "full_units",
                                   "units", "grid")]
FN_VOID = C.CFUNCTYPE(None)

# name: (restype, [argtypes]) -- one entry per declaration in include/*.h
SIGNATURES: dict[str, tuple] = {
    # runtime (sh_ops.h:20-48)
    "sh_init": (None, []), "sh_barrier_global": (None, []), "sh_barrier_cluster": (None, []),
    "sh_cluster_id": (u32, []), "sh_core_id": (u32, []), "sh_is_first_core": (i32, []), "sh_is_dm_core": (i32, []),
    "sh_num_clusters": (u32, []), "sh_timer_start": (None, []), "sh_timer_end": (None, []), "sh_eoc": (None, [u32]),
    "sh_cycles": (u32, []), "sh_printf": (None, [cp]), "sh_hbm_addr": (u64, [u64]), "sh_hbm_malloc": (u64, [u32]),
    "sh_l1_size": (u32, []), "sh_preload_wait": (None, [u64]), "sh_call_on_core_stack": (None, [FN_VOID, u32]),
    # GEMM (sh_ops.h:54-88)
    "sh_gemm": (i32, [u64, u64, u64, u32, u32, u32, u32, u32, u32, CFG_P, u32]),
    "sh_gemm_mesh": (i32, [u64, u64, u64, u32, u32, u32, u32, u32, u32, CFG_P]),
    "sh_gemm_xmcast": (i32, [u64, u64, u64, u32, u32, u32, u32, u32, u32, CFG_P]),
    "sh_gemm_xmcast_ex": (i32, [u64, u64, u64, u32, u32, u32, u32, u32, u32, CFG_P, u32]),
    "sh_gemm_xmcast_l1_bytes": (u32, [u32, u32, u32, CFG_P, u32]),
    "sh_gemm_l1_bytes": (u32, [u32, u32, u32, CFG_P]),
    # row ops (sh_ops.h:94-100)
    "sh_layernorm": (None, [u64, u64, u64, u64, u32, u32, u32, f32, u32]),
    "sh_softmax_rows": (None, [u64, u64, u32, u32, u32, f32, u32]),
    "sh_gelu": (None, [u64, u64, u32, u32, u32, u32]),
    "sh_add": (None, [u64, u64, u64, u32, u32, u32, u32]),
    "sh_add_bias": (None, [u64, u64, u64, u32, u32, u32, u32]),
    "sh_scale": (None, [u64, u64, u32, u32, u32, f32, u32]),
    "sh_transpose": (None, [u64, u64, u32, u32, u32, u32, u32]),
    # attention (sh_ops.h:109-127)
    "sh_attention_head": (i32, [u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, u32]),
    "sh_attention_q": (i32, [u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, u32, f32, u32, u32]),
    "sh_attention": (i32, [u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, u32, f32, u32]),
    "sh_attention_l1_bytes_q": (u32, [u32, u32, u32]),
    "sh_attention_l1_bytes": (u32, [u32, u32]),
    "sh_attention_q_block": (u32, [u32, u32, u32, u32]),
    "sh_attention_profile": (u32, [u32, u32, u32]),
    # test helpers (sh_ops.h:223-240)
    "sh_test_fill_int_fp16": (None, [u64, u32, u32, u32, u32, i32, i32]),
    "sh_test_fill_fp16": (None, [u64, u32, u32, u32, u32, i32, i32, f32]),
    "sh_test_dump_samples": (None, [u64, u32, u32, u32, u32, u32, cp]),
    "sh_test_dump_samples_idx": (None, [u64, u32, u32, u32, u32, u32, cp, u32]),
    "sh_test_check_gemm": (u32, [u64, u64, u64, u32, u32, u32, u32, u32, u32, u32, f32, f32, cp]),
    "sh_test_fill_const_fp16": (None, [u64, u32, u32, u32, u32]),
    "sh_test_fill_colparity_fp16": (None, [u64, u32, u32, u32, u32, u32]),
    "sh_test_check_const_fp16": (u32, [u64, u32, u32, u32, u32, u32, cp]),
    "sh_fp16_to_f32": (f32, [u16]),
    "sh_f32_to_fp16": (u16, [f32]),
    # extensions (sh_ops_cuda.h)
    "sh_cuda_set_arena": (i32, [vp, sz]), "sh_cuda_arena_base": (vp, []), "sh_cuda_arena_bytes": (sz, []),
    "sh_cuda_set_stream": (i32, [vp]), "sh_cuda_get_stream": (vp, []), "sh_cuda_synchronize": (i32, []),
    "sh_cuda_last_error": (i32, []), "sh_cuda_last_error_string": (cp, []), "sh_cuda_device_error": (i32, []),
    "sh_cuda_num_sms": (i32, []), "sh_cuda_timer_last_ms": (f32, []), "sh_cuda_abi_version": (u32, []),
    "sh_cuda_gemm": (i32, [u64, u64, u64, u32, u32, u32, u32, u32, u32, u64, u64, u32, u32, u32]),
    "sh_cuda_gemm_plan": (i32, [u32, u32, u32, u32, u32, C.POINTER(GemmPlan)]),
    "sh_cuda_gemm_ln": (i32, [u64, u64, u64, u32, u32, u32, u32, u32, u32, u64, u64, u32, u32, u64, u64, f32, u64]),
    "sh_rmsnorm": (None, [u64, u64, u64, u32, u32, u32, f32, u32]),
    "sh_rope": (None, [u64, u64, u64, u32, u32, u32, u32, u32, u32]),
    "sh_silu_mul": (None, [u64, u64, u64, u32, u32, u32, u32]),
    "sh_softmax_masked": (None, [u64, u64, u32, u32, u32, f32, u64, u64, u32]),
    "sh_attention_head_masked": (i32, [u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, u64, u32]),
    "sh_attention_gqa": (i32, [u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, u32, u32, f32, u64, u32]),
    "sh_pixel_shuffle": (None, [u64, u64, u32, u32, u32, u32]),
    "sh_cuda_preload_elf": (i32, [cp, u64]),
    "sh_preload_elf_segments": (i32, [cp, u64, C.c_void_p, C.c_void_p, u32]),
    "sh_cuda_row_stats": (i32, [u64, u32, u32, u32, u64]),
    "sh_cuda_scale_rows": (i32, [u64, u64, u32, u32, u32, u32, u64]),
    "sh_cuda_add_layernorm": (None, [u64, u64, u64, u64, u64, u64, u32, u32, u32, f32]),
    "sh_cuda_attention_batched": (i32, [u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, u32, f32, u32]),
    "sh_cuda_fill_normal_fp16": (None, [u64, u32, u32, u32, u32, f32, f32]),
    "sh_cuda_host_fill_normal_fp16": (None, [vp, u32, u32, u32, u32, f32, f32]),
    "sh_cuda_gemm_splitk_noalloc": (i32, [u64, u64, u64, u32, u32, u32, u32, u32, u32, u64, u64, u32, u32, u32]),
    "sh_cuda_fill_lcg_block": (None, [u64, u32, u32, u32, u32, i32, i32, f32, u64, u64, u64]),
    "sh_cuda_ipc_alloc": (vp, [sz]), "sh_cuda_ipc_free": (i32, [vp]), "sh_cuda_ipc_handle": (i32, [vp, vp]),
    "sh_cuda_ipc_open": (vp, [vp]), "sh_cuda_ipc_close": (i32, [vp]),
    "sh_cuda_copy2d": (i32, [u64, sz, u64, sz, sz, sz, vp]),
}

# sh_ops_cuda.h constants
EPI_ACCUMULATE, EPI_BIAS, EPI_GELU, EPI_RESIDUAL, GEMM_SIMT = 0x1, 0x2, 0x4, 0x8, 0x100
EPI_F32_OUT, EPI_ACC_F32_IN = 0x10, 0x20
EPI_LN_IN, EPI_STATS_OUT = 0x40, 0x80
SH_LLM_PAD = 0xFFFF
SH_ALL = 0xFFFFFFFF
SH_FP16, SH_FP8, SH_INT16, SH_INT8 = 0, 1, 2, 3
SH_XM_AUTO, SH_XM_PANEL, SH_XM_WHOLE = 0, 1, 2

_lib = None


def load(path: Path | str | None = None) -> C.CDLL:
    """Load the CUDA operator library (once) and attach the C signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: build it with `python softhier-mlir_b200/build.py`")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def cfg(tm=0, tn=0, tk=0, pipeline=1, accumulate=0, fmt=0, l1_base=0) -> GemmCfg:
    return GemmCfg(tm, tn, tk, pipeline, accumulate, fmt, l1_base)
