"""The C-ABI library loads and exports every symbol include/ugb.h declares (CPU only: no
compute calls without a GPU), and its pure host functions answer the reference's
known-answer cases."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER_DIR = os.path.join(ROOT, "include")


def declared_symbols():
    names = set()
    for fn in os.listdir(HEADER_DIR):
        if fn.endswith(".h"):
            text = open(os.path.join(HEADER_DIR, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names.update(re.findall(r"\b(ugb_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("ugb_init", "ugb_matvec", "ugb_quant_q8_1", "ugb_linear", "ugb_row_bytes"):
        assert must in names


def test_library_exports_every_declared_symbol(ugb):
    lib = ctypes.CDLL(ugb.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"libugb.so lacks {missing}"


def test_python_binding_covers_header(ugb):
    missing = [n for n in declared_symbols() if n not in ugb.SIGNATURES]
    assert not missing, f"binding lacks {missing}"


def test_row_bytes_abi(ugb):
    # frontier_core.rs:129-134 plus the configs' shapes and the other formats' block sizes
    assert ugb.row_bytes(23, 640) == -2
    assert ugb.row_bytes(20, 160) == 90
    assert ugb.row_bytes(18, 2560) == 980
    assert ugb.row_bytes(99, 256) == -1
    assert ugb.row_bytes(ugb.Q8_0, 1536) == 1632
    assert ugb.row_bytes(ugb.Q8_0, 8960) == 9520
    assert ugb.row_bytes(ugb.Q4_K, 18944) == 74 * 144
    assert ugb.row_bytes(ugb.Q3_K, 1536) == 660
    assert ugb.row_bytes(ugb.Q6_K, 4096) == 16 * 210
    assert ugb.row_bytes(ugb.IQ3_XXS, 1536) == 6 * 98
    assert ugb.row_bytes(ugb.IQ4_NL, 96) == 3 * 18
    assert ugb.row_bytes(ugb.IQ4_XS, 4096) == 16 * 136


def test_q8act_layout(ugb):
    for k, b in [(32, 1), (1536, 1), (8960, 4), (18944, 8), (96, 3)]:
        total = ugb.q8act_bytes(k, b)
        d_off, s_off = ugb.q8act_offsets(k, b)
        nbp = ((k // 32) + 3) // 4 * 4
        assert d_off >= k * b and d_off % 256 == 0
        assert s_off >= d_off + nbp * b * 4 and s_off % 256 == 0
        assert total >= s_off + nbp * b * 4
    assert ugb.q8act_bytes(33, 1) == 0
    assert ugb.q8act_bytes(32, 0) == 0


def test_init_without_gpu_fails_cleanly(ugb):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    code = ugb.lib().ugb_init(0, ctypes.byref(h))
    assert code == ugb.EBACKEND and not h.value
