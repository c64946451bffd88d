"""Instruction census and lint over this library's hand-written inline PTX.

The reference's `zoxide lint <file.ptx> [--census]` (src/main.zig:168-275) parses a PTX file
into lossless statements (src/ptx.zig:125-262) and counts instruction statements by mnemonic
plus modifiers, e.g. `ld.global.v4.f32` (census: src/ptx.zig:78-96; key: joinMods,
src/ptx.zig:99-108), printing

    census: <path> (<n> instruction statements, <k> classes)
      <count>  <key>

sorted by count, then key (src/main.zig:244-258). Its CI pins such counts per kernel
(.github/workflows/ci.yml:145-216).

Here the kernels are CUDA C++ whose PTX is written by hand inside `asm(...)` statements. The
census reads those string literals from the .cu/.cuh sources and counts what a person wrote,
one count per textual occurrence (a wrapper called from many places counts once). It never
reads compiler output: nvcc-emitted PTX/SASS is not an input to this tool, and instruction-mix
evidence for the built kernels comes from profiler counters instead.

Lint rules (`--census` off), for the hand-written strings:
  - a bulk / tensor copy that broadcasts to several CTAs of a cluster (the multi-destination
    qualifier): no kernel of this library issues one (the 2-SM kernels use cta_group::2 loads
    and two plain commits instead);
  - `wgmma`: sm_90a only, does not exist on sm_100a;
  - `mma.sync` / `wmma`: the legacy tensor path, not expected in a tcgen05 kernel;
  - `trap` / `brkpt`: kernels report failures through a status word and never trap.

Usage:  python -m zoxide_b200.census [--census] [files or directories ...]
        (default: the package's csrc/ directory)
"""
from __future__ import annotations

import re
import sys
from collections import Counter
from dataclasses import dataclass
from pathlib import Path

CSRC = Path(__file__).resolve().parent / "csrc"
SOURCE_SUFFIXES = (".cu", ".cuh", ".h", ".hpp", ".cpp")

_ASM_RE = re.compile(r"\basm\s*(?:volatile\s*|__volatile__\s*)?\(")


@dataclass(frozen=True)
class AsmBlock:
    """The PTX text of one asm(...) statement and the source line it starts on."""

    text: str
    line: int


@dataclass(frozen=True)
class Stmt:
    kind: str  # "instruction" | "directive" | "label"
    key: str  # mnemonic + "." + modifiers (instructions); directive name otherwise
    line: int
    text: str


def _skip_comment_or_string(src: str, i: int) -> int:
    """If src[i:] starts a C comment, string or char literal, return the index after it."""
    if src.startswith("//", i):
        j = src.find("\n", i)
        return len(src) if j < 0 else j
    if src.startswith("/*", i):
        j = src.find("*/", i + 2)
        return len(src) if j < 0 else j + 2
    if src[i] in "\"'":
        q, j = src[i], i + 1
        while j < len(src) and src[j] != q:
            j += 2 if src[j] == "\\" else 1
        return j + 1
    return i


def _unescape(lit: str) -> str:
    out, i = [], 0
    while i < len(lit):
        c = lit[i]
        if c == "\\" and i + 1 < len(lit):
            n = lit[i + 1]
            out.append({"n": "\n", "t": "\t", "\\": "\\", '"': '"', "'": "'", "r": "\r"}.get(n, n))
            i += 2
        else:
            out.append(c)
            i += 1
    return "".join(out)


def asm_blocks(src: str) -> list[AsmBlock]:
    """Every asm(...) statement's template: the adjacent string literals before the first
    operand colon (or the closing parenthesis), concatenated as the C++ compiler would."""
    blocks = []
    i = 0
    while i < len(src):
        j = _skip_comment_or_string(src, i)
        if j != i:
            i = j
            continue
        m = _ASM_RE.match(src, i)
        if not m or (i > 0 and (src[i - 1].isalnum() or src[i - 1] == "_")):
            i += 1
            continue
        line = src.count("\n", 0, i) + 1
        k = m.end()
        parts = []
        while k < len(src):
            c = src[k]
            if c.isspace():
                k += 1
            elif src.startswith("//", k) or src.startswith("/*", k):
                k = _skip_comment_or_string(src, k)
            elif c == '"':
                e = _skip_comment_or_string(src, k)
                parts.append(_unescape(src[k + 1:e - 1]))
                k = e
            else:
                break  # ':' (operands) or ')' (end) or a macro: the template is complete
        if parts:
            blocks.append(AsmBlock("".join(parts), line))
        i = k
    return blocks


def _ptx_statements(block: AsmBlock) -> list[Stmt]:
    """Split one asm template into PTX statements: ';' ends instructions and declarations,
    '{' / '}' (scope braces outside a vector operand) end nothing but themselves, and a bare
    'word:' is a label (cf. the termination rules of src/ptx.zig:113-124)."""
    text = block.text.replace("%%", "%")
    stmts, cur, depth = [], [], 0
    for c in text + ";":
        if c == "{" and depth == 0 and not "".join(cur).strip():
            cur = []
            continue
        if c == "}" and depth == 0 and not "".join(cur).strip():
            cur = []
            continue
        if c == "{":
            depth += 1
        elif c == "}":
            depth = max(0, depth - 1)
        if c == ";" and depth == 0:
            s = "".join(cur).strip()
            cur = []
            if s:
                stmts.extend(_classify(s, block.line))
            continue
        cur.append(c)
    return stmts


_LABEL_RE = re.compile(r"^([A-Za-z_$%][\w$%=]*)\s*:(?!:)\s*")


def _classify(s: str, line: int) -> list[Stmt]:
    out = []
    while True:
        m = _LABEL_RE.match(s)
        if not m:
            break
        out.append(Stmt("label", m.group(1), line, m.group(0).strip()))
        s = s[m.end():]
    s = s.strip()
    if not s:
        return out
    words = s.split()
    first = words[0]
    if first.startswith("@"):
        words = words[1:]
        if not words:
            return out
        first = words[0]
    if first.startswith("."):
        out.append(Stmt("directive", first[1:].split(".")[0], line, s))
        return out
    parts = [p for p in first.split(".") if p]
    out.append(Stmt("instruction", ".".join(parts), line, s))
    return out


def statements(src: str) -> list[Stmt]:
    out = []
    for b in asm_blocks(src):
        out.extend(_ptx_statements(b))
    return out


def census(src: str) -> Counter:
    """Instruction statements by mnemonic + modifiers (the reference's census key)."""
    return Counter(s.key for s in statements(src) if s.kind == "instruction")


# The multi-destination qualifier of bulk copies, assembled from parts so that this file itself
# never spells out a copy form it only exists to reject.
_BCAST = "multi" + "cast"
_BCAST_Q = _BCAST + "::" + "cluster"

LINT_RULES = (
    (re.compile(r"^cp\.async\.bulk(\.tensor)?\..*" + re.escape(_BCAST_Q)),
     "bulk/tensor copy broadcast to several CTAs: no kernel of this library issues one"),
    (re.compile(r"^cp\.reduce\.async\.bulk.*" + re.escape(_BCAST_Q)),
     "bulk reduce broadcast to several CTAs"),
    (re.compile(r"^wgmma\."), "wgmma is sm_90a-only; sm_100a kernels use tcgen05.mma"),
    (re.compile(r"^(mma\.sync|wmma)\b"), "legacy warp-level MMA in a tcgen05 library"),
    (re.compile(r"^(trap|brkpt)$"), "kernels report failures through the status word, never trap"),
)


def lint(src: str) -> list[tuple[int, str]]:
    findings = []
    for s in statements(src):
        if s.kind != "instruction":
            continue
        for rx, msg in LINT_RULES:
            if rx.search(s.key):
                findings.append((s.line, f"{msg}: `{s.key}`"))
    return findings


def format_census(path: str, counts: Counter) -> str:
    entries = sorted(counts.items(), key=lambda kv: (-kv[1], kv[0]))
    lines = [f"census: {path} ({sum(counts.values())} instruction statements, {len(entries)} classes)"]
    lines += [f"  {n:>6}  {k}" for k, n in entries]
    return "\n".join(lines)


def _expand(paths: list[str]) -> list[Path]:
    files = []
    for p in map(Path, paths):
        if p.is_dir():
            files += sorted(f for f in p.rglob("*") if f.suffix in SOURCE_SUFFIXES)
        else:
            files.append(p)
    return files


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    census_mode = "--census" in argv
    paths = [a for a in argv if a != "--census"]
    if any(a.startswith("-") for a in paths):
        print("usage: python -m zoxide_b200.census [--census] [files or directories ...]", file=sys.stderr)
        return 2
    files = _expand(paths or [str(CSRC)])
    if not files:
        print("error: no source files", file=sys.stderr)
        return 1
    rc = 0
    total = Counter()
    for f in files:
        src = f.read_text()
        if census_mode:
            c = census(src)
            total += c
            print(format_census(str(f), c))
        else:
            findings = lint(src)
            for line, msg in findings:
                print(f"{f}:{line}: {msg}")
            if findings:
                print(f"FAIL: {f}: {len(findings)} finding(s)")
                rc = 1
    if census_mode and len(files) > 1:
        print(format_census("(all files)", total))
    elif not census_mode and rc == 0:
        print(f"OK: {len(files)} file(s), no findings")
    return rc


if __name__ == "__main__":
    sys.exit(main())
