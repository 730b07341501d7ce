"""uefi-gpu_b200 -- Python binding of libugb, the B200 quantized linear-layer hot path.

The product is the C ABI in ``include/ugb.h`` (``libugb.so``, CUDA for sm_100a).  This module
binds it with ctypes so the tests and the benchmark can drive it; PyTorch is used only to
allocate device memory and to name CUDA streams.  There is no CPU fallback: if ``libugb.so``
is missing or fails to load, importing the ops raises.

The directory name contains a hyphen, so import it with
``importlib.import_module("uefi-gpu_b200")`` after putting the repository root on sys.path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libugb.so")

F32, Q8_0, Q3_K, Q4_K = 0, 8, 11, 12
MAX_BATCH = 8

STATUS = {0: "ok", 1: "shape", 2: "non-finite", 3: "timeout", 4: "backend", 5: "alignment",
          6: "quant kind", 7: "context"}
OK, ESHAPE, ENONFINITE, ETIMEOUT, EBACKEND, EALIGN, EQUANT, ECONTEXT = range(8)

# Every symbol include/ugb.h declares, with (restype, argtypes).
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_int = ctypes.c_int
SIGNATURES = {
    "ugb_init": (_int, [_int, ctypes.POINTER(_vp)]),
    "ugb_destroy": (_int, [_vp]),
    "ugb_status_string": (ctypes.c_char_p, [_int]),
    "ugb_status_read": (_int, [_vp, _vp, ctypes.POINTER(_u32)]),
    "ugb_row_bytes": (_i64, [_u32, _i64]),
    "ugb_q8act_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "ugb_q8act_scale_offset": (ctypes.c_size_t, [_i64, _i64]),
    "ugb_q8act_sum_offset": (ctypes.c_size_t, [_i64, _i64]),
    "ugb_quant_q8_1": (_int, [_vp, _vp, _vp, _vp, _i64, _i64]),
    "ugb_matvec": (_int, [_vp, _vp, _u32, _vp, _i64, _vp, _vp, _i64, _i64, _i64]),
    "ugb_block_dots": (_int, [_vp, _vp, _u32, _vp, _i64, _vp, _vp, _i64, _i64]),
    "ugb_fill_synthetic": (_int, [_vp, _vp, _u32, _vp, _i64, _i64, _u64]),
    "ugb_linear": (_int, [_vp, _vp, _u32, _vp, _i64, _vp, _vp, _i64, _i64]),
    "ugb_set_pdl": (_int, [_vp, _int]),
    "ugb_graph_begin": (_int, [_vp, _vp]),
    "ugb_graph_end": (_int, [_vp, _vp, ctypes.POINTER(_vp)]),
    "ugb_graph_launch": (_int, [_vp, _vp]),
    "ugb_graph_destroy": (_int, [_vp]),
}


class UgbError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {STATUS.get(code, code)} ({code})")
        self.code = code


def build() -> None:
    """Compile libugb.so for sm_100a (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", "-j8", "-C", HERE], check=True)


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run build() (make -C uefi-gpu_b200)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(fn: str, code: int) -> None:
    if code != OK:
        raise UgbError(fn, code)


def row_bytes(kind: int, n: int) -> int:
    return lib().ugb_row_bytes(kind, n)


def q8act_bytes(k: int, batch: int = 1) -> int:
    return lib().ugb_q8act_bytes(k, batch)


def q8act_offsets(k: int, batch: int = 1) -> tuple[int, int]:
    return lib().ugb_q8act_scale_offset(k, batch), lib().ugb_q8act_sum_offset(k, batch)


def _ptr(t) -> int:
    return t.data_ptr()


def _stream(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class Context:
    """One libugb context on one CUDA device (ugb_init / ugb_destroy)."""

    def __init__(self, device: int = 0):
        self.device = device
        h = _vp()
        check("ugb_init", lib().ugb_init(device, ctypes.byref(h)))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            lib().ugb_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- status ----------------------------------------------------------------------------
    def status_read(self, stream=None) -> tuple[int, int]:
        bits = _u32(0)
        code = lib().ugb_status_read(self.handle, _stream(stream), ctypes.byref(bits))
        return code, bits.value

    # ---- kernels (device tensors) -----------------------------------------------------------
    def quant_q8_1(self, x, xq, k: int, batch: int = 1, stream=None) -> None:
        check("ugb_quant_q8_1", lib().ugb_quant_q8_1(self.handle, _stream(stream), _ptr(x), _ptr(xq),
                                                       k, batch))

    def matvec(self, kind: int, w, rb: int, xq, y, k: int, m: int, batch: int = 1,
               stream=None) -> None:
        check("ugb_matvec", lib().ugb_matvec(self.handle, _stream(stream), kind, _ptr(w), rb,
                                               _ptr(xq), _ptr(y), k, m, batch))

    def block_dots(self, kind: int, w, rb: int, xq, out, k: int, m: int, stream=None) -> None:
        check("ugb_block_dots", lib().ugb_block_dots(self.handle, _stream(stream), kind, _ptr(w),
                                                       rb, _ptr(xq), _ptr(out), k, m))

    def fill_synthetic(self, kind: int, w, k: int, m: int, seed: int, stream=None) -> None:
        check("ugb_fill_synthetic", lib().ugb_fill_synthetic(self.handle, _stream(stream), kind,
                                                               _ptr(w), k, m, seed))

    def set_pdl(self, enable: bool) -> None:
        check("ugb_set_pdl", lib().ugb_set_pdl(self.handle, 1 if enable else 0))

    def capture(self, fn, stream) -> "Graph":
        """Capture the ugb_* calls fn() makes on `stream` (a non-default torch stream) into a
        replayable CUDA graph."""
        import torch
        with torch.cuda.stream(stream):
            check("ugb_graph_begin", lib().ugb_graph_begin(self.handle, stream.cuda_stream))
            try:
                fn()
            finally:
                h = _vp()
                code = lib().ugb_graph_end(self.handle, stream.cuda_stream, ctypes.byref(h))
        check("ugb_graph_end", code)
        return Graph(h)

    # ---- host-buffer entry points -----------------------------------------------------------
    def linear(self, kind: int, w, rb: int, x_host, k: int, m: int, stream=None):
        """Gpu::matvec / Weights::linear equivalent: numpy x in, numpy y out (synchronous)."""
        import numpy as np
        x = np.ascontiguousarray(x_host, dtype=np.float32)
        y = np.empty(m, dtype=np.float32)
        code = lib().ugb_linear(self.handle, _stream(stream), kind, _ptr(w), rb,
                                x.ctypes.data, y.ctypes.data, k, m)
        check("ugb_linear", code)
        return y


class Graph:
    """An instantiated CUDA graph of ugb_* calls (ugb_graph_end / launch / destroy)."""

    def __init__(self, handle):
        self.handle = handle

    def launch(self, stream=None) -> None:
        check("ugb_graph_launch", lib().ugb_graph_launch(self.handle, _stream(stream)))

    def close(self) -> None:
        if self.handle:
            lib().ugb_graph_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def alloc_q8act(k: int, batch: int = 1, device: str = "cuda"):
    """Device buffer for a Q8_1 activation (ugb_q8act_bytes), as a uint8 torch tensor."""
    import torch
    return torch.empty(q8act_bytes(k, batch), dtype=torch.uint8, device=device)


def split_q8act(xq, k: int, batch: int = 1):
    """Views (q int8 [batch,k], d f32 [batch,nbp], s int32 [batch,nbp]) of a Q8_1 buffer."""
    import torch
    d_off, s_off = q8act_offsets(k, batch)
    nbp = ((k // 32) + 3) // 4 * 4
    q = xq[: batch * k].view(torch.int8).view(batch, k)
    d = xq[d_off: d_off + batch * nbp * 4].view(torch.float32).view(batch, nbp)
    s = xq[s_off: s_off + batch * nbp * 4].view(torch.int32).view(batch, nbp)
    return q, d, s
