"""A small work-alike of LLVM FileCheck for the reference's `// CHECK` lines (CHECK, CHECK-NEXT, CHECK-NOT,
CHECK-LABEL; `{{regex}}` blocks; horizontal whitespace compared as single spaces)."""
from __future__ import annotations

import re

_DIRECTIVE = re.compile(r"//\s*(CHECK(?:-NEXT|-NOT|-LABEL)?):\s?(.*)$")


def directives(text: str) -> list[tuple[str, str]]:
    out = []
    for line in text.splitlines():
        m = _DIRECTIVE.search(line)
        if m:
            out.append((m.group(1), m.group(2).rstrip()))
    return out


def _pattern(p: str) -> re.Pattern:
    parts, i = [], 0
    while i < len(p):
        j = p.find("{{", i)
        if j < 0:
            parts.append(re.escape(" ".join(p[i:].split(" "))))
            break
        parts.append(re.escape(p[i:j]))
        k = p.find("}}", j)
        parts.append(p[j + 2:k])
        i = k + 2
    rx = "".join(parts)
    rx = re.sub(r"(\\ )+", r"\\s+", rx)
    return re.compile(rx)


def check(output: str, text: str) -> None:
    """Raise AssertionError with the failing directive if `output` does not satisfy the CHECK lines of `text`."""
    lines = [re.sub(r"[ \t]+", " ", ln) for ln in output.splitlines()]
    pos = 0          # first line the next positive match may use
    last = -1        # line of the previous match
    pending_not: list[str] = []
    for kind, pat in directives(text):
        rx = _pattern(re.sub(r"[ \t]+", " ", pat.strip()))
        if kind == "CHECK-NOT":
            pending_not.append(pat)
            continue
        if kind == "CHECK-NEXT":
            if last + 1 >= len(lines) or not rx.search(lines[last + 1]):
                raise AssertionError(f"CHECK-NEXT: {pat!r} not on the line after {lines[last] if last >= 0 else ''!r}")
            hit = last + 1
        else:
            hit = next((i for i in range(pos, len(lines)) if rx.search(lines[i])), None)
            if hit is None:
                raise AssertionError(f"{kind}: {pat!r} not found after line {pos}")
        for npat in pending_not:
            nrx = _pattern(re.sub(r"[ \t]+", " ", npat.strip()))
            for i in range(last + 1, hit):
                if nrx.search(lines[i]):
                    raise AssertionError(f"CHECK-NOT: {npat!r} found on line {i}: {lines[i]!r}")
        pending_not = []
        last, pos = hit, hit + 1
    for npat in pending_not:
        nrx = _pattern(re.sub(r"[ \t]+", " ", npat.strip()))
        for i in range(last + 1, len(lines)):
            if nrx.search(lines[i]):
                raise AssertionError(f"CHECK-NOT: {npat!r} found on line {i}: {lines[i]!r}")
