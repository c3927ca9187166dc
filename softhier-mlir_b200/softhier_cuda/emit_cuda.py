"""Lower a `softhier` dialect module to one libsh_ops_cuda.so call per op (the GPU backend beside the reference's
backend/emit_c.py).

Two outputs from the same walk:
  * `emit_c(text)`      a C program (`#include "sh_ops.h"`, phases <k>_inputs / <k> / <k>_checks, a main that
                        times the kernel phase) to compile against include/ and link with libsh_ops_cuda.so;
  * `Program(text, rt)` the same calls made in-process through ctypes on a Runtime's arena, phase by phase.

Lowering rules follow the reference backend's semantics (backend/emit_c.py:175-260 buffers / views / leading
dimensions / element offsets, 263-270 the gemm cfg, 280-605 op -> call, 608-669 the three phases):
  - a top-level hbm_buffer is `sh_hbm_addr(offset)`, named hb1, hb2, ... in program order; an indexed one
    (`%w = softhier.hbm_buffer %i {offset, stride}`) is `offset + i * stride` declared where it appears;
  - a view addresses its source's base; its strided layout gives (ld, element offset), an index operand adds
    index * stride elements;
  - `cluster` = -1 -> SH_ALL, -2 -> SH_SELF, absent -> 0;
  - prologue = test fills and the preload wait, epilogue = whole-buffer checks and the sample dumps of buffers no
    later op touches, kernel = the rest.
The module-level passes linalg-to-softhier / distribute-summa / pipeline-gemm are applied when requested, and
`fuse-epilogues` (this backend's own) folds add_bias / gelu / residual add into the producing GEMM.
"""
from __future__ import annotations

import ctypes
import re
import sys
from dataclasses import dataclass

from . import dialect as D
from . import lib as L

PROLOGUE = ("softhier.hbm_fill", "softhier.hbm_fill_col_parity", "softhier.hbm_fill_lcg", "softhier.preload_wait")
EPILOGUE = ("softhier.hbm_check_const",)
STRUCTURAL = ("softhier.hbm_buffer", "softhier.l1_buffer", "softhier.view", "softhier.cluster_id", "arith.constant",
              "arith.addi", "arith.subi", "arith.muli", "func.return")
_FMT = {"fp16": "SH_FP16", "fp8": "SH_FP8", "int16": "SH_INT16", "int8": "SH_INT8"}
_FMT_NUM = {"SH_FP16": 0, "SH_FP8": 1, "SH_INT16": 2, "SH_INT8": 3}
_XM = {"auto": "SH_XM_AUTO", "panel": "SH_XM_PANEL", "whole": "SH_XM_WHOLE"}
_ARITH = {"arith.addi": "+", "arith.subi": "-", "arith.muli": "*", "arith.divui": "/", "arith.remui": "%"}


def _f(v: float) -> str:
    return f"{float(v)!r}f"


def _cluster_c(attrs: dict) -> str:
    c = attrs.get("cluster", 0)
    return "SH_SELF" if c == -2 else "SH_ALL" if c < 0 else str(c)


def _cluster_v(attrs: dict) -> int:
    c = attrs.get("cluster", 0)
    return 0 if c == -2 else L.SH_ALL if c < 0 else int(c)


def apply_passes(fn: D.Func, passes: list[str] | tuple[str, ...] = ()) -> D.Func:
    for p in passes:
        if p == "linalg-to-softhier":
            fn = D.lower_linalg(fn)
        elif p == "distribute-summa":
            fn = D.mark_gemms(fn, "summa")
        elif p == "pipeline-gemm":
            fn = D.mark_gemms(fn, "pipeline")
        elif p == "fuse-epilogues":
            fn = fuse_epilogues(fn)
        else:
            raise ValueError(f"unknown pass {p}")
    return fn


# ---- epilogue fusion (this backend only) ------------------------------------------------------------------------------
FUSED = "softhier.gemm_fused"     # internal op: operands [x, w, bias(, residual)], into [z]; attrs["epi"] flags


def _tiles_ok(op: D.Op, m: int, n: int, k: int) -> bool:
    """sh_gemm's own shape checks (sh_gemm.inc.c:60-68) pass, so fusing cannot hide a -1 / -3 the module would see."""
    a = op.attrs
    tm, tn, tk = (int(a.get(t, 0)) or 256 for t in ("tile_m", "tile_n", "tile_k"))
    return a.get("fmt", "fp16") == "fp16" and m % tm == 0 and n % tn == 0 and k % tk == 0


def _read_before_overwrite(z: str, later: list[D.Op], defs: dict[str, D.Op]) -> bool:
    """Whether a later op may read buffer z (or a view of its buffer) before a plain GEMM overwrites all of z."""
    zbase = _base(z, defs)
    for lo in later:
        mentioned = [v for v in _all_operands(lo) if _base(v, defs) == zbase]
        if not mentioned:
            continue
        return not (lo.name == "softhier.gemm" and not lo.body and "accumulate" not in lo.attrs
                    and lo.into == [z] and defs[z].name == "softhier.hbm_buffer"
                    and all(_base(v, defs) != zbase for v in lo.operands))
    return False


def _fuse_list(ops: list[D.Op], defs: dict[str, D.Op]) -> list[D.Op]:
    out: list[D.Op] = []
    i = 0
    while i < len(ops):
        op = ops[i]
        if op.body:
            op = D.Op(name=op.name, results=op.results, operands=op.operands, into=op.into, outs=op.outs,
                      attrs=op.attrs, types=op.types, result_type=op.result_type, body=_fuse_list(op.body, defs),
                      text=op.text)
        nxt = ops[i + 1] if i + 1 < len(ops) else None
        if (op.name == "softhier.gemm" and not any(t in op.attrs for t in ("summa", "xmcast", "accumulate"))
                and nxt is not None and nxt.name == "softhier.add_bias" and nxt.operands[0] == op.into[0]
                and nxt.outs == op.into):
            x, w, z = op.operands[0], op.operands[1], op.into[0]
            mx, mw, mz = (defs[v].result_type for v in (x, w, z))
            m, k = mx.geom()[:2]
            n = mw.geom()[1]
            if _tiles_ok(op, m, n, k) and mz.geom()[:2] == (m, n):
                bias = nxt.operands[1]
                flags, dst, resid, used = L.EPI_BIAS, z, None, 2
                third = ops[i + 2] if i + 2 < len(ops) else None
                z_read_later = _read_before_overwrite(z, ops[i + 3:], defs)
                if third is not None and not z_read_later:
                    if (third.name == "softhier.gelu" and third.operands[0] == z
                            and defs[third.outs[0]].result_type.geom()[:2] == (m, n)):
                        flags, dst, used = flags | L.EPI_GELU, third.outs[0], 3
                    elif (third.name == "softhier.add" and "train" not in third.attrs and z in third.operands[:2]
                          and third.operands[0] != third.operands[1]
                          and defs[third.outs[0]].result_type.geom()[:2] == (m, n)):
                        r = third.operands[1] if third.operands[0] == z else third.operands[0]
                        if defs[r].result_type.geom()[:2] == (m, n):
                            flags, dst, resid, used = flags | L.EPI_RESIDUAL, third.outs[0], r, 3
                fused = D.Op(name=FUSED, operands=[x, w, bias] + ([resid] if resid else []), into=[dst],
                             attrs={"epi": flags, "tile_m": op.attrs.get("tile_m", 0),
                                    "tile_n": op.attrs.get("tile_n", 0), "tile_k": op.attrs.get("tile_k", 0)},
                             types=op.types, text=f"{FUSED} (from: {op.text.strip()[:60]} ...)")
                out.append(fused)
                i += used
                continue
        out.append(op)
        i += 1
    return out


def fuse_epilogues(fn: D.Func) -> D.Func:
    """`fuse-epilogues`: a plain fp16 softhier.gemm X, W into Z followed by `add_bias Z, b -> Z` becomes one GEMM
    with the bias in its epilogue; when the next op is `gelu Z -> G` or `add Z, R -> H` (either operand order) and
    nothing later reads Z, that op joins too (bias + tanh-GELU into G, or bias + residual R into H). The frontend's
    SigLIP layer (frontend/siglip.py:136-166) goes from 16 calls to 9. Results differ from the unfused program only by
    rounding: the fused epilogue rounds once to fp16 instead of after every op."""
    defs = _defs(fn.ops)
    return D.Func(name=fn.name, ops=_fuse_list(fn.ops, defs))


# ---- values: buffers and index expressions --------------------------------------------------------------------------
@dataclass
class Buf:
    space: str
    off: int
    mt: D.MemRef
    name: str                 # C name or address expression of the base


class Scope:
    """SSA values of one emitted phase: buffers (C names) and index expressions (C text)."""

    def __init__(self):
        self.bufs: dict[str, Buf] = {}
        self.idx: dict[str, str] = {}
        self.n_hb = 0
        self.n_iv = 0

    def hb_name(self) -> str:
        self.n_hb += 1
        return f"hb{self.n_hb}"

    def expr(self, v: str, defs: dict[str, D.Op]) -> str:
        if v in self.idx:
            return self.idx[v]
        op = defs.get(v)
        if op is None:
            raise D.ParseError(f"undefined index value {v}")
        if op.name == "arith.constant":
            return re.match(r"arith\.constant\s+(-?\d+)", op.text).group(1)
        if op.name == "softhier.cluster_id":
            return "sh_cluster_id()"
        if op.name in _ARITH:
            a, b = op.operands[:2]
            return f"({self.expr(a, defs)} {_ARITH[op.name]} {self.expr(b, defs)})"
        raise D.ParseError(f"index expression from {op.name}")

    def haddr(self, v: str) -> str:
        b = self.bufs[v]
        _, _, _, eoff = b.mt.geom()
        return b.name if eoff == 0 else f"({b.name} + {eoff * b.mt.elem_bytes})"


def _defs(ops: list[D.Op], out: dict | None = None) -> dict[str, D.Op]:
    out = {} if out is None else out
    for op in ops:
        for r in op.results:
            out[r] = op
        _defs(op.body, out)
    return out


def _base(v: str, defs: dict[str, D.Op]) -> str:
    while v in defs and defs[v].name == "softhier.view":
        v = defs[v].operands[0]
    return v


def _all_operands(op: D.Op) -> list[str]:
    out = list(op.operands) + list(op.into) + list(op.outs)
    for o in op.body:
        out += _all_operands(o)
    return out


def phase_of(op: D.Op, later: list[D.Op], defs: dict[str, D.Op]) -> str:
    """backend/emit_c.py:614-631."""
    if op.name in PROLOGUE:
        return "prologue"
    if op.name in EPILOGUE:
        return "epilogue"
    if op.name == "softhier.dump_samples":
        base = _base(op.operands[0], defs)
        for lo in later:
            if lo.name in ("softhier.dump_samples", "softhier.hbm_check_const"):
                continue
            if any(_base(o, defs) == base for o in _all_operands(lo)):
                return "kernel"
        return "epilogue"
    return "kernel"


# ---- C emission -----------------------------------------------------------------------------------------------------
def _gemm_cfg_c(op: D.Op) -> str:
    a = op.attrs
    fmt = _FMT.get(a.get("fmt", "fp16"), "SH_FP16")
    return (f"{{ .tm = {a.get('tile_m', 0)}, .tn = {a.get('tile_n', 0)}, .tk = {a.get('tile_k', 0)}, "
            f".pipeline = {1 if 'pipeline' in a else 0}, .accumulate = {1 if 'accumulate' in a else 0}, "
            f".fmt = {fmt}, .l1_base = 0 }}")


def _register_top(fn: D.Func, sc: Scope, decls: list[str]) -> None:
    for op in fn.ops:
        if op.name == "softhier.hbm_buffer" and not op.operands:
            mt = op.result_type
            name = sc.hb_name()
            sc.bufs[op.results[0]] = Buf("hbm", int(op.attrs["offset"]), mt, name)
            shape = "x".join(str(d) for d in mt.shape)
            decls.append(f"    const uint64_t {name} = sh_hbm_addr({int(op.attrs['offset'])});  "
                         f"// {shape}x{mt.elem} HBM, {mt.nbytes} B")


def _emit_ops(ops: list[D.Op], sc: Scope, defs: dict, out: list[str], tag: str, ind: str) -> None:
    for op in ops:
        n = op.name
        a = op.attrs
        if n in ("softhier.l1_buffer", "softhier.cluster_id", "arith.constant", "arith.addi", "arith.subi",
                 "arith.muli", "arith.divui", "arith.remui", "func.return", "scf.yield"):
            continue
        if n == "softhier.hbm_buffer":
            if op.results[0] in sc.bufs:
                continue
            mt = op.result_type
            name = sc.hb_name()
            sc.bufs[op.results[0]] = Buf("hbm", int(a["offset"]), mt, name)
            shape = "x".join(str(d) for d in mt.shape)
            out.append(f"{ind}const uint64_t {name} = sh_hbm_addr((uint64_t){int(a['offset'])} + "
                       f"(uint64_t)({sc.expr(op.operands[0], defs)}) * {int(a.get('stride', 0))}u);"
                       f"  // {shape}x{mt.elem} HBM, {mt.nbytes} B, indexed")
        elif n == "softhier.view":
            src = sc.bufs[op.operands[0]]
            mt = op.result_type
            name = src.name
            if len(op.operands) > 1:
                name = (f"({src.name} + (uint64_t)({sc.expr(op.operands[1], defs)}) * "
                        f"{int(a.get('stride', 0)) * mt.elem_bytes}u)")
            sc.bufs[op.results[0]] = Buf(src.space, src.off, mt, name)
        elif n == "scf.for":
            iv = op.results[0]
            sc.n_iv += 1
            sc.idx[iv] = f"i{sc.n_iv}"
            lb, ub, st = (sc.expr(v, defs) for v in op.operands)
            out.append(f"{ind}for (uint32_t {sc.idx[iv]} = {lb}; {sc.idx[iv]} < {ub}; {sc.idx[iv]} += {st}) {{")
            _emit_ops(op.body, sc, defs, out, tag, ind + "    ")
            out.append(f"{ind}}}")
        elif n == "softhier.gemm":
            x, w = op.operands[:2]
            z = op.into[0]
            m, k, ldx, _ = sc.bufs[x].mt.geom()
            _, nn, ldw, _ = sc.bufs[w].mt.geom()
            ldz = sc.bufs[z].mt.geom()[2]
            args = f"{sc.haddr(x)}, {sc.haddr(w)}, {sc.haddr(z)}, {m}, {nn}, {k}, {ldx}, {ldw}, {ldz}, &cfg"
            if "summa" in a:
                out.append(f"{ind}{{ sh_gemm_cfg cfg = {_gemm_cfg_c(op)};  // mesh-wide SUMMA")
                out.append(f"{ind}  sh_gemm_mesh({args}); }}")
            elif "xmcast" in a:
                mode = _XM[a["xmcast"] if isinstance(a["xmcast"], str) else "auto"]
                out.append(f"{ind}{{ sh_gemm_cfg cfg = {_gemm_cfg_c(op)};  // X-panel multicast, column slice per cluster")
                out.append(f"{ind}  sh_gemm_xmcast_ex({args}, {mode}); }}")
            else:
                out.append(f"{ind}{{ sh_gemm_cfg cfg = {_gemm_cfg_c(op)};")
                out.append(f"{ind}  sh_gemm({args}, {_cluster_c(a)}); }}")
        elif n == FUSED:
            x, w, b = op.operands[:3]
            z = op.into[0]
            m, k, ldx, _ = sc.bufs[x].mt.geom()
            _, nn, ldw, _ = sc.bufs[w].mt.geom()
            ldz = sc.bufs[z].mt.geom()[2]
            if len(op.operands) > 3:
                r = op.operands[3]
                res, ldr = sc.haddr(r), sc.bufs[r].mt.geom()[2]
            else:
                res, ldr = "0", ldz
            epi = [f for f, bit in (("SH_EPI_BIAS", L.EPI_BIAS), ("SH_EPI_GELU", L.EPI_GELU),
                                    ("SH_EPI_RESIDUAL", L.EPI_RESIDUAL)) if op.attrs["epi"] & bit]
            out.append(f"{ind}sh_cuda_gemm({sc.haddr(x)}, {sc.haddr(w)}, {sc.haddr(z)}, {m}, {nn}, {k}, {ldx}, {ldw}, "
                       f"{ldz}, {sc.haddr(b)}, {res}, {ldr}, {' | '.join(epi)}, 0);  // fused epilogue")
        elif n == "softhier.hbm_fill":
            rows, cols = op.types[0].shape[:2] if len(op.types[0].shape) > 1 else (1, op.types[0].shape[0])
            out.append(f"{ind}sh_test_fill_const_fp16({sc.bufs[op.operands[0]].name}, {rows}, {cols}, {cols}, "
                       f"{int(a['value_bits']) & 0xFFFF}u);")
        elif n == "softhier.hbm_fill_col_parity":
            rows, cols = op.types[0].shape[:2]
            out.append(f"{ind}sh_test_fill_colparity_fp16({sc.bufs[op.operands[0]].name}, {rows}, {cols}, {cols}, "
                       f"{int(a['even_bits']) & 0xFFFF}u, {int(a['odd_bits']) & 0xFFFF}u);")
        elif n == "softhier.hbm_check_const":
            rows, cols = op.types[0].shape[:2]
            out.append(f"{ind}sh_test_check_const_fp16({sc.bufs[op.operands[0]].name}, {rows}, {cols}, {cols}, "
                       f"{int(a['value_bits']) & 0xFFFF}u, {int(a['tol'])}, \"{tag}\");")
        elif n == "softhier.layernorm":
            x, g, b = op.operands[:3]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_layernorm({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {sc.haddr(g)}, {sc.haddr(b)}, "
                       f"{rows}, {cols}, {ld}, {_f(a['eps'])}, {_cluster_c(a)});")
        elif n == "softhier.softmax" and len(op.operands) == 1:
            x = op.operands[0]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_softmax_rows({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {rows}, {cols}, {ld}, "
                       f"{_f(a['scale'])}, {_cluster_c(a)});")
        elif n == "softhier.softmax":            # token-masked (emit_c.py:363-367): the same array for rows / columns
            x, m = op.operands[:2]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_softmax_masked({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {rows}, {cols}, {ld}, "
                       f"{_f(a['scale'])}, {sc.haddr(m)}, {sc.haddr(m)}, {_cluster_c(a)});")
        elif n == "softhier.rmsnorm":
            x, g = op.operands[:2]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_rmsnorm({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {sc.haddr(g)}, {rows}, {cols}, {ld}, "
                       f"{_f(a['eps'])}, {_cluster_c(a)});")
        elif n == "softhier.rope":
            x, t = op.operands[:2]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            ldt = sc.bufs[t].mt.geom()[2]
            out.append(f"{ind}sh_rope({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {sc.haddr(t)}, {rows}, {cols}, {ld}, {ldt}, "
                       f"{int(a['head_dim'])}, {_cluster_c(a)});")
        elif n == "softhier.silu_mul" and len(op.operands) == 2 and \
                sc.bufs[op.operands[0]].mt.geom()[2] == sc.bufs[op.operands[1]].mt.geom()[2] == \
                sc.bufs[op.outs[0]].mt.geom()[2]:   # one leading dimension (emit_c.py:381-385)
            x, y = op.operands
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_silu_mul({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {sc.haddr(y)}, {rows}, {cols}, {ld}, "
                       f"{_cluster_c(a)});")
        elif n == "softhier.pixel_shuffle":
            src = op.operands[0]
            rows, cols, _, _ = sc.bufs[src].mt.geom()
            grid = int(round(rows ** 0.5))
            out.append(f"{ind}sh_pixel_shuffle({sc.haddr(op.outs[0])}, {sc.haddr(src)}, {grid}, {cols}, "
                       f"{int(a['scale'])}, {_cluster_c(a)});")
        elif n == "softhier.attention" and (len(op.operands) == 4 or "kv_heads" in a):
            q, k, v = op.operands[:3]
            o = op.outs[0]
            S, Dm, ldq, _ = sc.bufs[q].mt.geom()
            ldk, ldv, ldo = (sc.bufs[t].mt.geom()[2] for t in (k, v, o))
            H = int(a["heads"])
            hkv = int(a.get("kv_heads", H))
            m = sc.haddr(op.operands[3]) if len(op.operands) == 4 else "0"
            out.append(f"{ind}sh_attention_gqa({sc.haddr(q)}, {sc.haddr(k)}, {sc.haddr(v)}, {sc.haddr(o)}, {S}, {Dm}, "
                       f"{H}, {hkv}, {ldq}, {ldk}, {ldv}, {ldo}, {_f(a['scale'])}, {m}, {_cluster_c(a)});")
        elif n == "softhier.scale":
            x = op.operands[0]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_scale({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {rows}, {cols}, {ld}, "
                       f"{_f(a['scale'])}, {_cluster_c(a)});")
        elif n == "softhier.gelu":
            x = op.operands[0]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_gelu({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {rows}, {cols}, {ld}, {_cluster_c(a)});")
        elif n == "softhier.add" and "train" not in a:
            x, y = op.operands[:2]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_add({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {sc.haddr(y)}, {rows}, {cols}, {ld}, "
                       f"{_cluster_c(a)});")
        elif n == "softhier.add_bias":
            x, b = op.operands[:2]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}sh_add_bias({sc.haddr(op.outs[0])}, {sc.haddr(x)}, {sc.haddr(b)}, {rows}, {cols}, "
                       f"{ld}, {_cluster_c(a)});")
        elif n == "softhier.attention" and len(op.operands) == 3 and "kv_heads" not in a:
            q, k, v = op.operands
            o = op.outs[0]
            S, Dm, ldq, _ = sc.bufs[q].mt.geom()
            ldk, ldv, ldo = (sc.bufs[t].mt.geom()[2] for t in (k, v, o))
            qb = int(a.get("q_block", 0))
            tail = f", {qb}" if qb else ""
            out.append(f"{ind}sh_attention{'_q' if qb else ''}({sc.haddr(q)}, {sc.haddr(k)}, {sc.haddr(v)}, "
                       f"{sc.haddr(o)}, {S}, {Dm}, {int(a['heads'])}, {ldq}, {ldk}, {ldv}, {ldo}, {_f(a['scale'])}, "
                       f"{_cluster_c(a)}{tail});")
        elif n == "softhier.transpose" and sc.bufs[op.operands[0]].mt.space != "tcdm":
            src, dst = op.operands[0], op.outs[0]
            rows, cols, lds, _ = sc.bufs[src].mt.geom()
            ldd = sc.bufs[dst].mt.geom()[2]
            out.append(f"{ind}sh_transpose({sc.haddr(dst)}, {sc.haddr(src)}, {rows}, {cols}, {lds}, {ldd}, "
                       f"{_cluster_c(a)});")
        elif n == "softhier.hbm_fill_lcg":
            x = op.operands[0]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            out.append(f"{ind}if (sh_cluster_id() == 0 && sh_is_first_core()) sh_test_fill_fp16({sc.haddr(x)}, "
                       f"{rows}, {cols}, {ld}, {int(a['seed'])}, {int(a['lo'])}, {int(a['hi'])}, {_f(a['scale'])});")
        elif n == "softhier.dump_samples":
            x = op.operands[0]
            rows, cols, ld, _ = sc.bufs[x].mt.geom()
            head = f"{ind}if (sh_cluster_id() == 0 && sh_is_first_core()) "
            if len(op.operands) > 1:
                out.append(head + f"sh_test_dump_samples_idx({sc.haddr(x)}, {rows}, {cols}, {ld}, {int(a['seed'])}, "
                                  f"{int(a['n'])}, \"{a['tag']}\", (uint32_t)({sc.expr(op.operands[1], defs)}));")
            else:
                out.append(head + f"sh_test_dump_samples({sc.haddr(x)}, {rows}, {cols}, {ld}, {int(a['seed'])}, "
                                  f"{int(a['n'])}, \"{a['tag']}\");")
        elif n == "softhier.group_barrier":
            out.append(f"{ind}sh_barrier_global();")
        elif n == "softhier.preload_wait":
            out.append(f"{ind}sh_preload_wait({sc.haddr(op.operands[0])});")
        elif n == "softhier.mark":
            head = f"{ind}if (sh_cluster_id() == 0 && sh_is_first_core()) "
            if op.operands:
                out.append(head + f"sh_printf(\"[mark] %s%u %u\\n\", \"{a['tag']}\", "
                                  f"(uint32_t)({sc.expr(op.operands[0], defs)}), sh_cycles());")
            else:
                out.append(head + f"sh_printf(\"[mark] %s %u\\n\", \"{a['tag']}\", sh_cycles());")
        else:
            out.append(f"{ind}// (unsupported on this backend: {n})")


def emit_kernel(fn: D.Func, phase: str | None = None) -> str:
    defs = _defs(fn.ops)
    sc = Scope()
    decls: list[str] = []
    _register_top(fn, sc, decls)
    top = fn.ops
    ops = [op for i, op in enumerate(top)
           if phase is None or op.name in STRUCTURAL or phase_of(op, top[i + 1:], defs) == phase]
    body: list[str] = []
    _emit_ops(ops, sc, defs, body, fn.name.upper(), "    ")
    return "\n".join(decls + body)


_MAIN = """\
// Generated by softhier_cuda.emit_cuda (softhier dialect -> libsh_ops_cuda.so calls). Do not edit by hand.
#include "sh_ops.h"
#include "sh_ops_cuda.h"

static void {k}_inputs(void) {{   // preload wait + test inputs (not timed)
{pro}
}}

static void {k}(void) {{
{ker}
}}

static void {k}_checks(void) {{   // test outputs (not timed)
{epi}
}}

int main(void) {{
    sh_init();
    {k}_inputs();
    sh_barrier_global();
    sh_timer_start();
    {k}();
    sh_barrier_global();
    sh_timer_end();
    {k}_checks();
    sh_barrier_global();
    sh_eoc(0);
    return 0;
}}
"""


def emit_c(text: str, passes: tuple[str, ...] = ()) -> str:
    fn = apply_passes(D.parse_module(text), passes)
    return _MAIN.format(k=fn.name, pro=emit_kernel(fn, "prologue"), ker=emit_kernel(fn, "kernel"),
                        epi=emit_kernel(fn, "epilogue"))


# ---- in-process program ------------------------------------------------------------------------------------------
class Program:
    """The module's calls made directly through the C ABI on a Runtime (arena offsets = the module's offsets).

    run() executes prologue, kernel (between sh_timer_start / sh_timer_end, which prints the reference's
    `[Performance Counter]` line) and epilogue; buffers can be read back with `tensor(name)`."""

    def __init__(self, text: str, rt, passes: tuple[str, ...] = ()):
        self.fn = apply_passes(D.parse_module(text), passes)
        self.rt = rt
        self.lib = rt.lib
        self.defs = _defs(self.fn.ops)
        need = 0
        for op in self.fn.ops:
            if op.name == "softhier.hbm_buffer" and not op.operands:
                need = max(need, int(op.attrs["offset"]) + op.result_type.nbytes)
        if need > rt.arena_bytes:
            raise ValueError(f"module needs {need} B of arena, the runtime has {rt.arena_bytes}")
        self.unsupported: list[str] = []

    # address of an SSA buffer value under an index environment
    def _addr(self, v: str, env: dict) -> tuple[int, D.MemRef]:
        op = self.defs[v]
        if op.name == "softhier.hbm_buffer":
            off = int(op.attrs["offset"])
            if op.operands:
                off += self._ival(op.operands[0], env) * int(op.attrs.get("stride", 0))
            return self.lib.sh_hbm_addr(off), op.result_type
        if op.name == "softhier.view":
            base, _ = self._addr(op.operands[0], env)
            mt = op.result_type
            if len(op.operands) > 1:
                base += self._ival(op.operands[1], env) * int(op.attrs.get("stride", 0)) * mt.elem_bytes
            return base + mt.geom()[3] * mt.elem_bytes, mt
        raise D.ParseError(f"{v} is not a buffer")

    def _ival(self, v: str, env: dict) -> int:
        if v in env:
            return env[v]
        op = self.defs[v]
        if op.name == "arith.constant":
            return int(re.match(r"arith\.constant\s+(-?\d+)", op.text).group(1))
        if op.name == "softhier.cluster_id":
            return 0
        a, b = (self._ival(x, env) for x in op.operands[:2])
        return {"arith.addi": a + b, "arith.subi": a - b, "arith.muli": a * b, "arith.divui": a // max(b, 1),
                "arith.remui": a % max(b, 1)}[op.name]

    def _call(self, op: D.Op, env: dict) -> int:
        lib, n, a = self.lib, op.name, op.attrs
        A = lambda v: self._addr(v, env)  # noqa: E731
        if n in ("softhier.hbm_buffer", "softhier.view", "arith.constant", "arith.addi", "arith.subi", "arith.muli",
                 "arith.divui", "arith.remui", "softhier.cluster_id", "softhier.l1_buffer"):
            return 0
        if n == "scf.for":
            lb, ub, st = (self._ival(v, env) for v in op.operands)
            for i in range(lb, ub, st):
                env2 = dict(env)
                env2[op.results[0]] = i
                for o in op.body:
                    rc = self._call(o, env2)
                    if rc:
                        return rc
            return 0
        if n == "softhier.gemm":
            (x, mx), (w, mw), (z, mz) = A(op.operands[0]), A(op.operands[1]), A(op.into[0])
            m, k, ldx, _ = mx.geom()
            _, nn, ldw, _ = mw.geom()
            cfg = L.cfg(a.get("tile_m", 0), a.get("tile_n", 0), a.get("tile_k", 0), 1 if "pipeline" in a else 0,
                        1 if "accumulate" in a else 0, _FMT_NUM[_FMT.get(a.get("fmt", "fp16"), "SH_FP16")], 0)
            args = (x, w, z, m, nn, k, ldx, ldw, mz.geom()[2], ctypes.byref(cfg))
            if "summa" in a:
                return lib.sh_gemm_mesh(*args)
            if "xmcast" in a:
                mode = {"auto": 0, "panel": 1, "whole": 2}[a["xmcast"] if isinstance(a["xmcast"], str) else "auto"]
                return lib.sh_gemm_xmcast_ex(*args, mode)
            return lib.sh_gemm(*args, _cluster_v(a))
        if n == FUSED:
            (x, mx), (w, mw), (b, _), (z, mz) = A(op.operands[0]), A(op.operands[1]), A(op.operands[2]), A(op.into[0])
            m, k, ldx, _ = mx.geom()
            _, nn, ldw, _ = mw.geom()
            r, ldr = (A(op.operands[3])[0], A(op.operands[3])[1].geom()[2]) if len(op.operands) > 3 else (0, mz.geom()[2])
            return lib.sh_cuda_gemm(x, w, z, m, nn, k, ldx, ldw, mz.geom()[2], b, r, ldr, op.attrs["epi"], 0)
        if n == "softhier.layernorm":
            (x, mx), (g, _), (b, _), (y, _) = A(op.operands[0]), A(op.operands[1]), A(op.operands[2]), A(op.outs[0])
            rows, cols, ld, _ = mx.geom()
            lib.sh_layernorm(y, x, g, b, rows, cols, ld, a["eps"], _cluster_v(a))
            return 0
        if n == "softhier.softmax" and len(op.operands) == 1:
            (x, mx), (y, _) = A(op.operands[0]), A(op.outs[0])
            rows, cols, ld, _ = mx.geom()
            lib.sh_softmax_rows(y, x, rows, cols, ld, a["scale"], _cluster_v(a))
            return 0
        if n == "softhier.softmax":
            (x, mx), (m, _), (y, _) = A(op.operands[0]), A(op.operands[1]), A(op.outs[0])
            rows, cols, ld, _ = mx.geom()
            lib.sh_softmax_masked(y, x, rows, cols, ld, a["scale"], m, m, _cluster_v(a))
            return 0
        if n == "softhier.rmsnorm":
            (x, mx), (g, _), (y, _) = A(op.operands[0]), A(op.operands[1]), A(op.outs[0])
            rows, cols, ld, _ = mx.geom()
            lib.sh_rmsnorm(y, x, g, rows, cols, ld, a["eps"], _cluster_v(a))
            return 0
        if n == "softhier.rope":
            (x, mx), (t, mt), (y, _) = A(op.operands[0]), A(op.operands[1]), A(op.outs[0])
            rows, cols, ld, _ = mx.geom()
            lib.sh_rope(y, x, t, rows, cols, ld, mt.geom()[2], int(a["head_dim"]), _cluster_v(a))
            return 0
        if n == "softhier.silu_mul" and len(op.operands) == 2:
            (x, mx), (b, mb), (y, my) = A(op.operands[0]), A(op.operands[1]), A(op.outs[0])
            rows, cols, ld, _ = mx.geom()
            if mb.geom()[2] == ld == my.geom()[2]:
                lib.sh_silu_mul(y, x, b, rows, cols, ld, _cluster_v(a))
                return 0
        if n == "softhier.pixel_shuffle":
            (x, mx), (y, _) = A(op.operands[0]), A(op.outs[0])
            rows, cols, _, _ = mx.geom()
            lib.sh_pixel_shuffle(y, x, int(round(rows ** 0.5)), cols, int(a["scale"]), _cluster_v(a))
            return 0
        if n == "softhier.attention" and (len(op.operands) == 4 or "kv_heads" in a):
            (q, mq), (k, mk), (v, mv), (o, mo) = (A(t) for t in (*op.operands[:3], op.outs[0]))
            S, Dm, ldq, _ = mq.geom()
            H = int(a["heads"])
            m = A(op.operands[3])[0] if len(op.operands) == 4 else 0
            return lib.sh_attention_gqa(q, k, v, o, S, Dm, H, int(a.get("kv_heads", H)), ldq, mk.geom()[2],
                                        mv.geom()[2], mo.geom()[2], a["scale"], m, _cluster_v(a))
        if n in ("softhier.gelu", "softhier.scale"):
            (x, mx), (y, _) = A(op.operands[0]), A(op.outs[0])
            rows, cols, ld, _ = mx.geom()
            if n == "softhier.gelu":
                lib.sh_gelu(y, x, rows, cols, ld, _cluster_v(a))
            else:
                lib.sh_scale(y, x, rows, cols, ld, a["scale"], _cluster_v(a))
            return 0
        if n in ("softhier.add", "softhier.add_bias"):
            (x, mx), (b, _), (y, _) = A(op.operands[0]), A(op.operands[1]), A(op.outs[0])
            rows, cols, ld, _ = mx.geom()
            (lib.sh_add if n == "softhier.add" else lib.sh_add_bias)(y, x, b, rows, cols, ld, _cluster_v(a))
            return 0
        if n == "softhier.transpose":
            (s, ms), (d, md) = A(op.operands[0]), A(op.outs[0])
            rows, cols, lds, _ = ms.geom()
            lib.sh_transpose(d, s, rows, cols, lds, md.geom()[2], _cluster_v(a))
            return 0
        if n == "softhier.attention" and len(op.operands) == 3:
            (q, mq), (k, mk), (v, mv), (o, mo) = (A(t) for t in (*op.operands, op.outs[0]))
            S, Dm, ldq, _ = mq.geom()
            qb = int(a.get("q_block", 0))
            argv = (q, k, v, o, S, Dm, int(a["heads"]), ldq, mk.geom()[2], mv.geom()[2], mo.geom()[2], a["scale"],
                    _cluster_v(a))
            return lib.sh_attention_q(*argv, qb) if qb else lib.sh_attention(*argv)
        if n == "softhier.hbm_fill_lcg":
            x, mx = A(op.operands[0])
            rows, cols, ld, _ = mx.geom()
            lib.sh_test_fill_fp16(x, rows, cols, ld, int(a["seed"]), int(a["lo"]), int(a["hi"]), a["scale"])
            return 0
        if n in ("softhier.hbm_fill", "softhier.hbm_fill_col_parity", "softhier.hbm_check_const"):
            x, mx = A(op.operands[0])
            rows, cols = mx.shape[:2] if len(mx.shape) > 1 else (1, mx.shape[0])
            if n == "softhier.hbm_fill":
                lib.sh_test_fill_const_fp16(x, rows, cols, cols, int(a["value_bits"]) & 0xFFFF)
            elif n == "softhier.hbm_fill_col_parity":
                lib.sh_test_fill_colparity_fp16(x, rows, cols, cols, int(a["even_bits"]) & 0xFFFF,
                                                int(a["odd_bits"]) & 0xFFFF)
            else:
                lib.sh_test_check_const_fp16(x, rows, cols, cols, int(a["value_bits"]) & 0xFFFF, int(a["tol"]),
                                             self.fn.name.upper().encode())
            return 0
        if n == "softhier.dump_samples":
            x, mx = A(op.operands[0])
            rows, cols, ld, _ = mx.geom()
            if len(op.operands) > 1:
                lib.sh_test_dump_samples_idx(x, rows, cols, ld, int(a["seed"]), int(a["n"]), a["tag"].encode(),
                                             self._ival(op.operands[1], env))
            else:
                lib.sh_test_dump_samples(x, rows, cols, ld, int(a["seed"]), int(a["n"]), a["tag"].encode())
            return 0
        if n == "softhier.group_barrier":
            lib.sh_barrier_global()
            return 0
        if n == "softhier.preload_wait":
            lib.sh_preload_wait(A(op.operands[0])[0])
            return 0
        if n == "softhier.mark":
            t = lib.sh_cycles()
            idx = f"{self._ival(op.operands[0], env)}" if op.operands else ""
            sys.stdout.write(f"[mark] {a['tag']}{idx} {t}\n")
            sys.stdout.flush()
            return 0
        self.unsupported.append(n)
        raise NotImplementedError(f"{n} is outside this library's operator set")

    def run_phase(self, phase: str) -> int:
        top = self.fn.ops
        for i, op in enumerate(top):
            if op.name in STRUCTURAL or phase_of(op, top[i + 1:], self.defs) != phase:
                continue
            rc = self._call(op, {})
            if rc:
                return rc
        return 0

    def run(self, timed: bool = True) -> int:
        lib = self.lib
        rc = self.run_phase("prologue")
        lib.sh_barrier_global()
        if timed:
            lib.sh_timer_start()
        rc = rc or self.run_phase("kernel")
        lib.sh_barrier_global()
        if timed:
            lib.sh_timer_end()
        rc = rc or self.run_phase("epilogue")
        lib.sh_barrier_global()
        return rc

    def address(self, name: str) -> tuple[int, D.MemRef]:
        """Device address and type of a top-level SSA buffer (e.g. "%q")."""
        return self._addr(name if name.startswith("%") else "%" + name, {})

    def tensor(self, name: str):
        addr, mt = self.address(name)
        rows, cols, ld, _ = mt.geom()
        return self.rt.get(addr, rows, cols, ld)
