"""Parser for the textual `softhier` dialect modules that the reference's frontends and examples produce.

The reference parses these modules with xDSL (softhier_mlir/dialects/softhier.py, tools/softhier_translate.py).
xDSL is not available to this package, so this module reads the generic MLIR text form of the subset on the
operator-library path directly: a `builtin.module` holding one `func.func` whose body is a list of ops --

    softhier.hbm_buffer / view                      buffers and strided views (memref types with strided layouts)
    softhier.gemm / layernorm / softmax / gelu / add / add_bias / scale / transpose / attention
    softhier.hbm_fill / hbm_fill_col_parity / hbm_fill_lcg / hbm_check_const / dump_samples
    softhier.mark / group_barrier / preload_wait
    linalg.matmul ins(..) outs(..)                  (lowered like the linalg-to-softhier pass, HBM operands)
    scf.for + arith.constant / addi / subi / muli / divui / remui on `index` values

Ops outside the subset are kept as `Op` records with their name so a caller can report them.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field

import numpy as np

_ELEM_BYTES = {"f16": 2, "bf16": 2, "f32": 4, "f64": 8, "i8": 1, "i16": 2, "i32": 4}


@dataclass
class MemRef:
    shape: tuple[int, ...]
    elem: str
    space: str
    strides: tuple[int, ...] | None = None
    offset: int = 0

    @property
    def elem_bytes(self) -> int:
        return _ELEM_BYTES.get(self.elem, 2)

    @property
    def nbytes(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n * self.elem_bytes

    def geom(self) -> tuple[int, int, int, int]:
        """(rows, cols, leading dim, element offset) of the 2-D (or 1-D as 1 x n) view (emit_c.py:226-235)."""
        if len(self.shape) == 1:
            rows, cols = 1, self.shape[0]
        else:
            rows, cols = self.shape[0], self.shape[1]
        if self.strides is not None:
            ld = self.strides[0] if len(self.shape) > 1 else cols
            return rows, cols, ld, self.offset
        return rows, cols, cols, 0


@dataclass
class Op:
    name: str
    results: list[str] = field(default_factory=list)
    operands: list[str] = field(default_factory=list)      # before `into` / `->`
    into: list[str] = field(default_factory=list)          # after `into`
    outs: list[str] = field(default_factory=list)          # after `->`
    attrs: dict = field(default_factory=dict)
    types: list[MemRef] = field(default_factory=list)      # every memref type written on the op
    result_type: MemRef | None = None
    body: list["Op"] = field(default_factory=list)         # scf.for region
    text: str = ""


@dataclass
class Func:
    name: str
    ops: list[Op]


class ParseError(ValueError):
    pass


# ---- lexical helpers ---------------------------------------------------------------------------------------------
_MEMREF = re.compile(r"memref<")


def _split_top(s: str, sep: str = ",") -> list[str]:
    """Split on `sep` outside <>, [], (), {} and quotes."""
    out, depth, cur, q = [], 0, [], False
    for ch in s:
        if ch == '"':
            q = not q
        elif not q and ch in "<[({":
            depth += 1
        elif not q and ch in ">])}":
            depth -= 1
        if ch == sep and depth == 0 and not q:
            out.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        out.append("".join(cur))
    return [p.strip() for p in out]


def _match_bracket(s: str, i: int, open_ch: str, close_ch: str) -> int:
    """Index of the bracket closing the one at s[i]."""
    depth, q = 0, False
    for j in range(i, len(s)):
        ch = s[j]
        if ch == '"':
            q = not q
        elif not q and ch == open_ch:
            depth += 1
        elif not q and ch == close_ch:
            depth -= 1
            if depth == 0:
                return j
    raise ParseError(f"unbalanced {open_ch}{close_ch} in: {s}")


def parse_memref(t: str) -> MemRef:
    t = t.strip()
    if not t.startswith("memref<") or not t.endswith(">"):
        raise ParseError(f"not a memref type: {t}")
    parts = _split_top(t[len("memref<"):-1])
    dims = parts[0].split("x")
    elem = dims[-1]
    shape = tuple(int(d) for d in dims[:-1])
    strides, offset, space = None, 0, "hbm"
    for p in parts[1:]:
        if p.startswith("strided<"):
            m = re.match(r"strided<\[([^\]]*)\](?:,\s*offset:\s*(-?\d+))?>", p)
            if not m:
                raise ParseError(f"bad layout {p}")
            strides = tuple(int(v) for v in m.group(1).split(","))
            offset = int(m.group(2) or 0)
        elif p.startswith('"'):
            space = p.strip('"')
    return MemRef(shape, elem, space, strides, offset)


def _memrefs_in(s: str) -> list[MemRef]:
    out = []
    for m in _MEMREF.finditer(s):
        j = _match_bracket(s, m.start() + len("memref"), "<", ">")
        out.append(parse_memref(s[m.start():j + 1]))
    return out


def _parse_value(v: str):
    v = v.strip()
    if v.startswith('"'):
        return v[1:-1]
    m = re.match(r"^(-?[0-9.eE+\-]+)\s*:\s*(\w+)$", v)
    if m:
        num, ty = m.group(1), m.group(2)
        if ty.startswith("f"):
            x = float(num)
            return float(np.float32(x)) if ty == "f32" else x
        return int(num)
    if re.match(r"^-?\d+$", v):
        return int(v)
    try:
        return float(v)
    except ValueError:
        return v


def parse_attrs(s: str) -> dict:
    attrs = {}
    for item in _split_top(s):
        if not item:
            continue
        if "=" in item:
            k, v = item.split("=", 1)
            attrs[k.strip()] = _parse_value(v)
        else:
            attrs[item.strip()] = True     # unit attribute
    return attrs


def _strip_comment(line: str) -> str:
    """Drop a `//` comment that is not inside a string literal."""
    q = False
    for i, ch in enumerate(line):
        if ch == '"':
            q = not q
        elif not q and line.startswith("//", i):
            return line[:i]
    return line


# ---- statements --------------------------------------------------------------------------------------------------
def _statements(body: str) -> list[str]:
    """Join the function body into one string per op: a new op starts at a line that begins with `%name =`,
    an op name, or a closing brace; other lines continue the previous op."""
    stmts: list[str] = []
    start = re.compile(r"^(%[\w.]+(\s*,\s*%[\w.]+)*\s*=|[a-z_]+\.[a-z_0-9.]+|\})")
    for raw in body.splitlines():
        line = _strip_comment(raw).rstrip()
        if not line.strip():
            continue
        s = line.strip()
        if start.match(s) or not stmts:
            stmts.append(s)
        else:
            stmts[-1] += " " + s
    return stmts


def _parse_op(s: str) -> Op:
    results: list[str] = []
    m = re.match(r"^((?:%[\w.]+\s*,\s*)*%[\w.]+)\s*=\s*(.*)$", s)
    if m:
        results = [r.strip() for r in m.group(1).split(",")]
        s = m.group(2)
    m = re.match(r"^([a-z_]+\.[a-z_0-9.]+)\s*(.*)$", s)
    if not m:
        raise ParseError(f"cannot parse op: {s}")
    name, rest = m.group(1), m.group(2)
    op = Op(name=name, results=results, text=s)
    if name == "linalg.matmul":
        ins = re.search(r"ins\(([^:]*):", rest)
        outs = re.search(r"outs\(([^:]*):", rest)
        if not ins or not outs:
            raise ParseError(f"bad linalg.matmul: {s}")
        op.operands = [v.strip() for v in ins.group(1).split(",")]
        op.into = [v.strip() for v in outs.group(1).split(",")]
        op.types = _memrefs_in(rest)
        return op
    # attribute dict (first top-level `{`)
    attr_txt = ""
    i = rest.find("{")
    head, tail = rest, ""
    if i >= 0:
        j = _match_bracket(rest, i, "{", "}")
        attr_txt = rest[i + 1:j]
        head, tail = rest[:i], rest[j + 1:]
    else:
        k = rest.find(":")
        if k >= 0:
            head, tail = rest[:k], rest[k:]
    op.attrs = parse_attrs(attr_txt)
    # operands: %a, %b [into %c] [-> %d]
    before, _, after_arrow = head.partition("->")
    before, _, after_into = before.partition("into")
    op.operands = [v.strip() for v in before.split(",") if v.strip().startswith("%")]
    op.into = [v.strip() for v in after_into.split(",") if v.strip().startswith("%")]
    op.outs = [v.strip() for v in after_arrow.split(",") if v.strip().startswith("%")]
    op.types = _memrefs_in(tail)
    if results and op.types:
        op.result_type = op.types[-1]
    return op


def _parse_block(stmts: list[str], i: int) -> tuple[list[Op], int]:
    ops: list[Op] = []
    while i < len(stmts):
        s = stmts[i]
        if s.startswith("}"):
            return ops, i + 1
        if s.startswith("scf.for"):
            m = re.match(r"^scf\.for\s+(%[\w.]+)\s*=\s*(%[\w.]+)\s+to\s+(%[\w.]+)\s+step\s+(%[\w.]+)\s*\{", s)
            if not m:
                raise ParseError(f"bad scf.for: {s}")
            op = Op(name="scf.for", operands=[m.group(2), m.group(3), m.group(4)], results=[m.group(1)], text=s)
            op.body, i = _parse_block(stmts, i + 1)
            ops.append(op)
            continue
        if s.startswith("func.return") or s.startswith("scf.yield"):
            i += 1
            continue
        ops.append(_parse_op(s))
        i += 1
    return ops, i


def parse_module(text: str) -> Func:
    """The (single) function of a `builtin.module`."""
    text = "\n".join(_strip_comment(ln) for ln in text.splitlines())
    m = re.search(r"func\.func\s+@([\w.]+)\s*\(\s*\)\s*(?:attributes\s*\{[^}]*\}\s*)?\{", text)
    if not m:
        raise ParseError("no func.func @name() { ... } in the module")
    start = m.end() - 1
    end = _match_bracket(text, start, "{", "}")
    stmts = _statements(text[start + 1:end])
    ops, _ = _parse_block(stmts, 0)
    return Func(m.group(1), ops)


# ---- the module-level passes of the reference, restated on this representation --------------------------------------
def lower_linalg(fn: Func) -> Func:
    """linalg-to-softhier (transforms/linalg_to_softhier.py:40-60) for HBM outputs: linalg.matmul -> softhier.gemm
    with fmt = "fp16" and no tile attributes. TCDM outputs (RedMulE tiles) are outside this library."""
    def walk(ops):
        out = []
        for op in ops:
            if op.name == "linalg.matmul":
                out.append(Op(name="softhier.gemm", operands=op.operands[:2], into=op.into[:1],
                              attrs={"fmt": "fp16"}, types=op.types, text=op.text))
            else:
                if op.body:
                    op.body = walk(op.body)
                out.append(op)
        return out
    return Func(fn.name, walk(fn.ops))


def mark_gemms(fn: Func, attr: str) -> Func:
    """distribute-summa (`summa`, transforms/distribute_summa.py:27-30) / pipeline-gemm (`pipeline`,
    transforms/pipeline_gemm.py:26-32): add a unit attribute to every softhier.gemm."""
    def walk(ops):
        for op in ops:
            if op.name == "softhier.gemm":
                op.attrs = {attr: True, **op.attrs}
            walk(op.body)
    walk(fn.ops)
    return fn


# ---- printing (generic form of the ops the passes rewrite) ---------------------------------------------------------
def _attr_str(k: str, v) -> str:
    if v is True:
        return k
    if isinstance(v, str):
        return f'{k} = "{v}"'
    if isinstance(v, float):
        return f"{k} = {v!r} : f32"
    return f"{k} = {v} : i32"


def print_op(op: Op, ind: str = "    ") -> str:
    head = f"{', '.join(op.results)} = " if op.results else ""
    parts = [op.name]
    if op.operands:
        parts.append(", ".join(op.operands))
    if op.into:
        parts.append("into " + ", ".join(op.into))
    if op.outs:
        parts.append("-> " + ", ".join(op.outs))
    if op.attrs:
        parts.append("{" + ", ".join(_attr_str(k, v) for k, v in op.attrs.items()) + "}")
    return ind + head + " ".join(parts)


def print_func(fn: Func) -> str:
    lines = [f"func.func @{fn.name}() {{"]

    def walk(ops, ind):
        for op in ops:
            if op.name == "scf.for":
                lines.append(f"{ind}scf.for {op.results[0]} = {op.operands[0]} to {op.operands[1]} step "
                             f"{op.operands[2]} {{")
                walk(op.body, ind + "  ")
                lines.append(ind + "}")
            else:
                lines.append(print_op(op, ind) if op.name.startswith("softhier.") else ind + op.text)
    walk(fn.ops, "  ")
    lines.append("}")
    return "\n".join(lines)
