"""The boundary document and the binding describe the header's ABI exactly (CPU only).

* INTEGRATION.md's Rust FFI block has every struct of include/ugb.h with the same fields in
  the same order and corresponding types, every entry point with the same parameters, and the
  same constant values (tests/abi_parse.py states the C-to-Rust type rule);
* a C program compiled with gcc against include/ugb.h prints each public struct's size and every
  field's offset; those equal the repr(C) layout of the Rust declarations and the layout of the
  Python binding's ctypes structures.
A host built from either document therefore hands the library structs of the size and layout
it reads."""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
import tempfile

import pytest

import abi_parse as ap
from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "ugb.h")
DOC = os.path.join(ROOT, "INTEGRATION.md")

# size and alignment of the Rust field types on LP64 (x86-64, aarch64)
RUST_SIZES = {"i32": 4, "u32": 4, "f32": 4, "i64": 8, "u64": 8, "usize": 8, "u8": 1}


def _header():
    return open(HEADER).read()


def _rust():
    return ap.rust_block(open(DOC).read())


def test_rust_structs_match_header():
    hs, rs = ap.header_structs(_header()), ap.rust_structs(_rust())
    assert set(hs) <= set(rs), f"structs missing from INTEGRATION.md: {sorted(set(hs) - set(rs))}"
    for name, fields in hs.items():
        assert rs[name] == fields, f"{name}: INTEGRATION.md {rs[name]} != header {fields}"


def test_rust_functions_match_header():
    hf, rf = ap.header_functions(_header()), ap.rust_functions(_rust())
    assert len(hf) > 40
    assert set(hf) == set(rf), f"only in header: {sorted(set(hf) - set(rf))}; only in doc: {sorted(set(rf) - set(hf))}"
    for name, sig in hf.items():
        assert rf[name] == sig, f"{name}: INTEGRATION.md {rf[name]} != header {sig}"


def test_rust_constants_match_header():
    hc, rc = ap.header_constants(_header()), ap.rust_constants(_rust())
    assert hc == rc


def _rust_size_align(ty):
    arr = __import__("re").match(r"^\[(.*); (\d+)\]$", ty)
    if arr:
        size, align = _rust_size_align(arr.group(1))
        return size * int(arr.group(2)), align
    size = 8 if ty.startswith("*") else RUST_SIZES[ty]
    return size, size


def _rust_layout(fields):
    """repr(C) offsets and size of a struct of the given Rust field types."""
    off, align, out = 0, 1, []
    for name, ty in fields:
        size, a = _rust_size_align(ty)
        off = (off + a - 1) // a * a
        out.append((name, off))
        off += size
        align = max(align, a)
    return out, (off + align - 1) // align * align


def _c_layout():
    """{struct: (size, [(field, offset)])} from a C program compiled with gcc."""
    gcc = shutil.which("gcc") or shutil.which("cc")
    if not gcc:
        pytest.skip("no C compiler")
    structs = ap.header_structs(_header())
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for name, fields in structs.items():
        lines.append(f'  printf("S {name} %zu\\n", sizeof({name}));')
        for f, _ in fields:
            lines.append(f'  printf("F {name} {f} %zu\\n", offsetof({name}, {f}));')
    lines += ["  return 0;", "}"]
    with tempfile.TemporaryDirectory() as tmp:
        src, exe = os.path.join(tmp, "layout.c"), os.path.join(tmp, "layout")
        open(src, "w").write("\n".join(lines) + "\n")
        subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-o", exe, src], check=True)
        text = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    out = {}
    for line in text.splitlines():
        kind, name, *rest = line.split()
        if kind == "S":
            out[name] = (int(rest[0]), [])
        else:
            out[name][1].append((rest[0], int(rest[1])))
    return out


def test_c_layout_equals_rust_repr_c():
    c = _c_layout()
    rs = ap.rust_structs(_rust())
    for name, (size, offs) in c.items():
        want, want_size = _rust_layout(rs[name])
        assert offs == want, f"{name}: C offsets {offs} != Rust repr(C) {want}"
        assert size == want_size, f"{name}: C size {size} != Rust {want_size}"


def test_c_layout_equals_ctypes(ugb):
    c = _c_layout()
    binding = {"ugb_job": ugb.Job, "ugb_moe_args": ugb.MoeArgs, "ugb_decoder_config": ugb.DecoderConfig,
               "ugb_layer_weights": ugb.LayerWeights, "ugb_model_weights": ugb.ModelWeights,
               "ugb_gguf_tensor": ugb.GgufTensor}
    assert set(binding) == set(c)
    for name, cls in binding.items():
        size, offs = c[name]
        assert ctypes.sizeof(cls) == size, name
        assert [(f, getattr(cls, f).offset) for f, _ in cls._fields_] == offs, name
