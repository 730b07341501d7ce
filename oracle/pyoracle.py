"""ctypes binding of the CPU restatement (oracle/ugb_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the CPU legs of
bench.py, as the checker and the timed CPU baseline.  The product path never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")

Q8_0, Q3_K, Q4_K = 8, 11, 12
Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS = 14, 18, 20, 23  # the reference's other formats (frontier_core.rs:54-55)

_c_u8p = ctypes.POINTER(ctypes.c_uint8)
_c_i8p = ctypes.POINTER(ctypes.c_int8)
_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_i32p = ctypes.POINTER(ctypes.c_int32)


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _load(name: str) -> ctypes.CDLL:
    path = os.path.join(BUILD, name)
    if not os.path.exists(path):
        build()
    lib = ctypes.CDLL(path)
    lib.orc_half.restype = ctypes.c_float
    lib.orc_half.argtypes = [ctypes.c_uint16]
    lib.orc_row_bytes.restype = ctypes.c_long
    lib.orc_row_bytes.argtypes = [ctypes.c_uint32, ctypes.c_long]
    lib.orc_dequantize.restype = ctypes.c_int
    lib.orc_dequantize.argtypes = [ctypes.c_uint32, _c_u8p, ctypes.c_long, _c_f32p, ctypes.c_long]
    lib.orc_quant_act.restype = ctypes.c_int
    lib.orc_quant_act.argtypes = [_c_f32p, _c_i8p, _c_f32p, _c_i32p, ctypes.c_long]
    lib.orc_block_dots.restype = ctypes.c_int
    lib.orc_block_dots.argtypes = [ctypes.c_uint32, _c_u8p, _c_i8p, ctypes.c_long, _c_i32p]
    for fn in (lib.orc_matvec, lib.orc_matvec_mt, lib.orc_matvec_terms_mt):
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_uint32, _c_u8p, ctypes.c_long, _c_i8p, _c_f32p, _c_i32p, _c_f32p,
                       ctypes.c_long, ctypes.c_long, ctypes.c_long]
    lib.orc_threads.restype = ctypes.c_int
    lib.orc_matvec_dequant_f32.restype = ctypes.c_int
    lib.orc_matvec_dequant_f32.argtypes = [ctypes.c_uint32, _c_u8p, ctypes.c_long, _c_f32p,
                                           _c_f32p, ctypes.c_long, ctypes.c_long]
    lib.orc_dispatch_pack.restype = ctypes.c_long
    lib.orc_dispatch_pack.argtypes = [ctypes.c_void_p, ctypes.c_long, _c_u8p,
                                      ctypes.POINTER(ctypes.c_uint32)]
    lib.orc_moe_route.restype = ctypes.c_int
    lib.orc_moe_route.argtypes = [_c_f32p, ctypes.c_long, ctypes.c_long, _c_i32p, _c_f32p]
    lib.orc_prefill_repack_q8_0.restype = ctypes.c_int
    lib.orc_prefill_repack_q8_0.argtypes = [_c_u8p, ctypes.c_long, ctypes.c_long, ctypes.c_long,
                                            _c_i8p, _c_f32p]
    lib.orc_prefill_gemm_q8_0.restype = ctypes.c_int
    lib.orc_prefill_gemm_q8_0.argtypes = [_c_u8p, ctypes.c_long, ctypes.c_long, _c_f32p, ctypes.c_long,
                                          _c_f32p, ctypes.c_int]
    lib.orc_silu_mul.restype = ctypes.c_float
    lib.orc_silu_mul.argtypes = [ctypes.c_float, ctypes.c_float]
    lib.orc_set_iq3_grid.restype = None
    lib.orc_set_iq3_grid.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
    grid = iq3_grid()
    lib.orc_set_iq3_grid(grid.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return lib


def iq3_grid() -> np.ndarray:
    """The IQ3_XXS grid as 256 little-endian words of four magnitudes, decoded from the compact
    form the third-party gguf package (0.19.0) ships (IQ3_XXS.grid_map / grid_hex) -- an
    independent source from the table compiled into libugb."""
    from gguf import quants

    quants.IQ3_XXS.init_grid()
    g = np.asarray(quants.IQ3_XXS.grid, dtype=np.float32).reshape(256, 4).astype(np.uint32)
    return np.ascontiguousarray(g[:, 0] | (g[:, 1] << 8) | (g[:, 2] << 16) | (g[:, 3] << 24))


_LIBS: dict[str, ctypes.CDLL] = {}


def lib(mt: bool = False) -> ctypes.CDLL:
    name = "libugb_oracle_mt.so" if mt else "libugb_oracle.so"
    if name not in _LIBS:
        _LIBS[name] = _load(name)
    return _LIBS[name]


def _p(a: np.ndarray, ct):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(ct)


def half(h: int) -> float:
    return lib().orc_half(h)


def row_bytes(kind: int, n: int) -> int:
    return lib().orc_row_bytes(kind, n)


def dequantize(kind: int, raw: np.ndarray, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    rc = lib().orc_dequantize(kind, _p(raw, _c_u8p), raw.size, _p(out, _c_f32p), n)
    if rc:
        raise ValueError(f"orc_dequantize rc={rc}")
    return out


def quant_act(x: np.ndarray):
    """Block-32 activation quantisation of x [..., k] -> (q int8 [...,k], d f32 [...,k/32],
    s int32 [...,k/32], bad)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    q = np.empty(x.shape, dtype=np.int8)
    d = np.empty(x.shape[:-1] + (k // 32,), dtype=np.float32)
    s = np.empty(x.shape[:-1] + (k // 32,), dtype=np.int32)
    bad = lib().orc_quant_act(_p(x, _c_f32p), _p(q, _c_i8p), _p(d, _c_f32p), _p(s, _c_i32p), x.size)
    return q, d, s, bad


def block_dots(kind: int, row: np.ndarray, q: np.ndarray) -> np.ndarray:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    q = np.ascontiguousarray(q, dtype=np.int8)
    out = np.empty(q.size // 32, dtype=np.int32)
    rc = lib().orc_block_dots(kind, _p(row, _c_u8p), _p(q, _c_i8p), q.size, _p(out, _c_i32p))
    if rc:
        raise ValueError(f"orc_block_dots rc={rc}")
    return out


def matvec(kind: int, w: np.ndarray, row_bytes_: int, q: np.ndarray, d: np.ndarray, s: np.ndarray,
           k: int, m: int, batch: int = 1, mt: bool = False) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    q = np.ascontiguousarray(q, dtype=np.int8)
    d = np.ascontiguousarray(d, dtype=np.float32)
    s = np.ascontiguousarray(s, dtype=np.int32)
    y = np.empty((batch, m), dtype=np.float32)
    fn = lib(mt).orc_matvec_mt if mt else lib().orc_matvec
    rc = fn(kind, _p(w, _c_u8p), row_bytes_, _p(q, _c_i8p), _p(d, _c_f32p), _p(s, _c_i32p),
            _p(y, _c_f32p), k, m, batch)
    if rc:
        raise ValueError(f"orc_matvec rc={rc}")
    return y


def matvec_terms(kind: int, w: np.ndarray, row_bytes_: int, q: np.ndarray, d: np.ndarray, s: np.ndarray,
                 k: int, m: int, batch: int = 1) -> np.ndarray:
    """Per (vector, row): the sum of the magnitudes of the row's block terms."""
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    q = np.ascontiguousarray(q, dtype=np.int8)
    d = np.ascontiguousarray(d, dtype=np.float32)
    s = np.ascontiguousarray(s, dtype=np.int32)
    y = np.empty((batch, m), dtype=np.float32)
    rc = lib(True).orc_matvec_terms_mt(kind, _p(w, _c_u8p), row_bytes_, _p(q, _c_i8p), _p(d, _c_f32p),
                                       _p(s, _c_i32p), _p(y, _c_f32p), k, m, batch)
    if rc:
        raise ValueError(f"orc_matvec_terms rc={rc}")
    return y


def matvec_dequant_f32(kind: int, w: np.ndarray, row_bytes_: int, x: np.ndarray, k: int, m: int):
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(m, dtype=np.float32)
    rc = lib().orc_matvec_dequant_f32(kind, _p(w, _c_u8p), row_bytes_, _p(x, _c_f32p),
                                      _p(y, _c_f32p), k, m)
    if rc:
        raise ValueError(f"orc_matvec_dequant_f32 rc={rc}")
    return y


class Dispatch(ctypes.Structure):
    _fields_ = [("weight", ctypes.c_uint64), ("input", ctypes.c_uint64),
                ("output", ctypes.c_uint64), ("kind", ctypes.c_uint32), ("n", ctypes.c_uint32),
                ("m", ctypes.c_uint32), ("row_bytes", ctypes.c_uint32)]


def dispatch_pack(jobs):
    """jobs: list of (weight, input, output, kind, n, m, row_bytes) -> (bytes, grid) or None."""
    arr = (Dispatch * max(1, len(jobs)))(*[Dispatch(*j) for j in jobs])
    out = np.zeros(max(1, len(jobs)) * 48, dtype=np.uint8)
    grid = ctypes.c_uint32(0)
    n = lib().orc_dispatch_pack(ctypes.cast(arr, ctypes.c_void_p), len(jobs), _p(out, _c_u8p),
                                ctypes.byref(grid))
    if n < 0:
        return None
    return out[:n].tobytes(), grid.value


def moe_route(logits: np.ndarray, top_k: int):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    ids = np.empty(top_k, dtype=np.int32)
    w = np.empty(top_k, dtype=np.float32)
    rc = lib().orc_moe_route(_p(logits, _c_f32p), logits.size, top_k, _p(ids, _c_i32p),
                             _p(w, _c_f32p))
    if rc:
        return None
    return ids, w


def prefill_repack_q8_0(w: np.ndarray, n: int, k: int, n_pad: int):
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    qa = np.empty((n_pad, k), dtype=np.int8)
    sa = np.empty((k // 32, n_pad), dtype=np.float32)
    rc = lib().orc_prefill_repack_q8_0(_p(w, _c_u8p), n, k, n_pad, _p(qa, _c_i8p), _p(sa, _c_f32p))
    if rc:
        raise ValueError(f"orc_prefill_repack_q8_0 rc={rc}")
    return qa, sa


def silu_mul(g: float, u: float) -> float:
    return lib().orc_silu_mul(g, u)


def prefill_gemm_q8_0(w: np.ndarray, n: int, k: int, x: np.ndarray, threads: int = 0) -> np.ndarray:
    """y [m][n] of the Q8 prefill GEMM on GGUF Q8_0 rows w (n x k) and fp32 tokens x [m][k]."""
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
    x = np.ascontiguousarray(x, dtype=np.float32)
    m = x.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    mt = threads != 1
    l = lib(mt)
    nthr = threads if threads > 0 else (l.orc_threads() if mt else 1)
    rc = l.orc_prefill_gemm_q8_0(_p(w, _c_u8p), n, k, _p(x, _c_f32p), m, _p(y, _c_f32p), nthr)
    if rc < 0:
        raise ValueError(f"orc_prefill_gemm_q8_0 rc={rc}")
    return y
