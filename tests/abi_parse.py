"""Parsers for the C ABI header (include/ugb.h) and for the Rust FFI declarations shown in
INTEGRATION.md, so tests can check that the two describe the same boundary: every struct with
the same fields in the same order and of corresponding types, every prototype with the same
parameters, and the same constants.

C to Rust type rule (repr(C), x86-64 / aarch64 LP64): int / int32_t -> i32, uint32_t -> u32,
int64_t -> i64, uint64_t -> u64, size_t -> usize, float -> f32, char -> c_char, void -> c_void,
uint8_t -> u8; a pointer is *const T when what it points to is const, else *mut T."""
from __future__ import annotations

import re

SCALARS = {"int": "i32", "int32_t": "i32", "uint32_t": "u32", "int64_t": "i64", "uint64_t": "u64",
           "size_t": "usize", "float": "f32", "char": "c_char", "void": "c_void", "uint8_t": "u8",
           "ugb_status": "ugb_status", "ugb_stream": "ugb_stream"}


def strip_comments(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return re.sub(r"//[^\n]*", " ", text)


def c_to_rust(ctype: str) -> str:
    """'const void *const *' -> '*const *const c_void'; 'uint64_t[4]' -> '[u64; 4]'; a void
    return -> '()'."""
    arr = re.match(r"^(.*)\[(\d+)\]$", ctype)
    if arr:
        return f"[{c_to_rust(arr.group(1))}; {arr.group(2)}]"
    if ctype.strip() == "void":
        return "()"
    parts = ctype.replace("*", " * ").split()
    base, quals, i = [], [], 0
    while i < len(parts) and parts[i] != "*":
        base.append(parts[i])
        i += 1
    base_const = "const" in base
    base_name = [b for b in base if b not in ("const", "struct")]
    assert len(base_name) == 1, ctype
    pointee_const = base_const
    levels = []
    while i < len(parts):
        assert parts[i] == "*", ctype
        i += 1
        levels.append("*const " if pointee_const else "*mut ")
        pointee_const = i < len(parts) and parts[i] == "const"
        if pointee_const:
            i += 1
    name = SCALARS.get(base_name[0], base_name[0])
    return "".join(reversed(levels)) + name if levels else name


def _split_decl(decl: str):
    """'const void *a, *b' -> [('const void *', 'a'), ('const void *', 'b')]; an array field
    'uint64_t dims[4]' -> [('uint64_t[4]', 'dims')]."""
    decl = " ".join(decl.split())
    first = re.match(r"^(.*?)(\**)\s*(\w+)\s*(\[\d+\])?$", decl.split(",")[0].strip())
    base = first.group(1).strip()
    out = [(f"{base} {first.group(2)}".strip() + (first.group(4) or ""), first.group(3))]
    for extra in decl.split(",")[1:]:
        m = re.match(r"^\s*(\**)\s*(\w+)\s*(\[\d+\])?\s*$", extra)
        out.append((f"{base} {m.group(1)}".strip() + (m.group(3) or ""), m.group(2)))
    return out


def header_structs(text: str) -> dict:
    """struct name -> [(field, rust type)] for every typedef struct with a body."""
    text = strip_comments(text)
    out = {}
    for m in re.finditer(r"typedef\s+struct\s+(\w+)\s*\{(.*?)\}\s*(\w+)\s*;", text, flags=re.S):
        fields = []
        for decl in m.group(2).split(";"):
            if decl.strip():
                fields += [(n, c_to_rust(t)) for t, n in _split_decl(decl)]
        out[m.group(3)] = fields
    return out


def header_functions(text: str) -> dict:
    """function name -> (rust return type, [(param, rust type)])."""
    text = strip_comments(text)
    text = re.sub(r"typedef\s+(struct|enum)\s+\w*\s*\{.*?\}\s*\w+\s*;", " ", text, flags=re.S)
    text = re.sub(r"enum\s*\{.*?\}\s*;", " ", text, flags=re.S)
    text = re.sub(r"#[^\n]*", " ", text)
    out = {}
    for m in re.finditer(r"([\w\s\*]+?)\b(ugb_\w+)\s*\(([^)]*)\)\s*;", text):
        ret = " ".join(m.group(1).split())
        ret = ret.split("}")[-1].strip()
        params = []
        for p in m.group(3).split(","):
            p = p.strip()
            if p and p != "void":
                (t, n), = _split_decl(p)
                params.append((n, c_to_rust(t)))
        out[m.group(2)] = (c_to_rust(ret), params)
    return out


def header_constants(text: str) -> dict:
    """UGB_* constant -> int, from #defines with integer values and enum bodies."""
    out = {}
    for m in re.finditer(r"#define\s+(UGB_\w+)\s+(\d+)\b", text):
        out[m.group(1)] = int(m.group(2))
    body_text = strip_comments(text)
    for m in re.finditer(r"enum\s*\w*\s*\{(.*?)\}", body_text, flags=re.S):
        val = -1
        for item in m.group(1).split(","):
            item = item.strip()
            if not item:
                continue
            name, _, expr = item.partition("=")
            name = name.strip()
            if expr.strip():
                e = expr.strip()
                mm = re.match(r"^(\d+)u?\s*<<\s*(\d+)$", e)
                val = int(mm.group(1)) << int(mm.group(2)) if mm else int(e.rstrip("u"), 0)
            else:
                val += 1
            out[name] = val
    return out


def rust_block(md: str) -> str:
    m = re.search(r"```rust\n(.*?)```", md, flags=re.S)
    assert m, "no rust block"
    return m.group(1)


def rust_structs(rs: str) -> dict:
    out = {}
    for m in re.finditer(r"#\[repr\(C\)\]\s*pub struct (\w+)\s*\{(.*?)\}", rs, flags=re.S):
        body = re.sub(r"//[^\n]*", " ", m.group(2))
        fields = [(f.group(1), " ".join(f.group(2).split())) for f in re.finditer(r"pub (\w+):\s*([^,]+?)\s*(?:,|$)", body)]
        if fields:
            out[m.group(1)] = fields
    return out


def rust_functions(rs: str) -> dict:
    out = {}
    for m in re.finditer(r"pub fn (ugb_\w+)\((.*?)\)\s*(?:->\s*([^;]+))?;", rs, flags=re.S):
        params = []
        for p in re.sub(r"\s+", " ", m.group(2)).split(","):
            p = p.strip()
            if p:
                n, t = p.split(":", 1)
                params.append((n.strip(), " ".join(t.split())))
        ret = " ".join((m.group(3) or "()").split())
        out[m.group(1)] = (ret, params)
    return out


def rust_constants(rs: str) -> dict:
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"pub const (UGB_\w+):\s*\w+\s*=\s*(\d+)\s*;", rs)}
