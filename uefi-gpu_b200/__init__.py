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

F32, F16, Q8_0, Q3_K, Q4_K = 0, 1, 8, 11, 12
Q6_K, IQ3_XXS, IQ4_NL, IQ4_XS = 14, 18, 20, 23  # the reference's other block formats
MAX_BATCH = 8
LINEAR_STATIC_MAX_K, LINEAR_STATIC_MAX_M = 16384, 524288  # ugb_linear_static's fixed scratch

STATUS = {0: "ok", 1: "shape", 2: "non-finite", 3: "timeout", 4: "backend", 5: "alignment",
          6: "quant kind", 7: "context"}
OK, ESHAPE, ENONFINITE, ETIMEOUT, EBACKEND, EALIGN, EQUANT, ECONTEXT = range(8)
# Device status bits (ugb_status_read).
STATUS_NONFINITE_IN, STATUS_NONFINITE_OUT, STATUS_TIMEOUT, STATUS_BADARG = 1, 2, 4, 8

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
    "ugb_matvec_f32": (_int, [_vp, _vp, _u32, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64]),
    "ugb_matvec_multi": (_int, [_vp, _vp, _u32, ctypes.POINTER(_vp), ctypes.POINTER(_i64), _int,
                                _i64, _vp, _vp, _i64, _i64]),
    "ugb_block_dots": (_int, [_vp, _vp, _u32, _vp, _i64, _vp, _vp, _i64, _i64]),
    "ugb_fill_synthetic": (_int, [_vp, _vp, _u32, _vp, _i64, _i64, _u64]),
    "ugb_linear": (_int, [_vp, _vp, _u32, _vp, _i64, _vp, _vp, _i64, _i64]),
    "ugb_linear_static": (_int, [_vp, _vp, _u32, _vp, _i64, _vp, _vp, _i64, _i64]),
    "ugb_set_pdl": (_int, [_vp, _int]),
    "ugb_matvec_jobs": (_int, [_vp, _vp, _vp, _int, _i64]),
    "ugb_moe_route": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "ugb_moe_combine": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _int, _vp]),
    "ugb_moe_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64, _i64]),
    "ugb_moe_experts": (_int, [_vp, _vp, _vp]),
    "ugb_prefill_packed_bytes": (_i64, [_i64, _i64]),
    "ugb_prefill_repack_q8_0": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "ugb_prefill_quant": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "ugb_prefill_gemm_q8_0": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64]),
    "ugb_prefill_block_dots": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64]),
    "ugb_decoder_create": (_int, [_vp, _vp, ctypes.POINTER(_vp)]),
    "ugb_decoder_destroy": (_int, [_vp]),
    "ugb_decoder_bind": (_int, [_vp, _vp]),
    "ugb_decoder_synthetic": (_int, [_vp, _u64]),
    "ugb_decoder_step": (_int, [_vp, _vp]),
    "ugb_decoder_set_state": (_int, [_vp, _vp, ctypes.c_int32, ctypes.c_int32]),
    "ugb_decoder_set_tokens": (_int, [_vp, _vp, _vp, ctypes.c_int32]),
    "ugb_decoder_get_tokens": (_int, [_vp, _vp, _vp, ctypes.POINTER(ctypes.c_int32), _vp]),
    "ugb_decoder_tokens": (_int, [_vp, _vp, _vp, ctypes.c_int32, _vp]),
    "ugb_decoder_set_comm": (_int, [_vp, _vp]),
    "ugb_decoder_set_path": (_int, [_vp, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]),
    "ugb_comm_unique_id": (_int, [_vp]),
    "ugb_comm_init": (_int, [_vp, _int, _int, _vp, ctypes.POINTER(_vp)]),
    "ugb_comm_destroy": (_int, [_vp]),
    "ugb_comm_allreduce_f32": (_int, [_vp, _vp, _vp, _i64]),
    "ugb_comm_allreduce_max_u64": (_int, [_vp, _vp, _vp, _i64]),
    "ugb_decoder_get_state": (_int, [_vp, _vp, ctypes.POINTER(ctypes.c_int32),
                                     ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]),
    "ugb_decoder_logits": (_int, [_vp, _vp, _vp]),
    "ugb_decoder_read_kv": (_int, [_vp, _vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                   _vp, _vp]),
    "ugb_decoder_token": (_int, [_vp, _vp, ctypes.c_int32, ctypes.c_int32,
                                 ctypes.POINTER(ctypes.c_int32)]),
    "ugb_decoder_write_kv": (_int, [_vp, _vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                    _vp, _vp]),
    "ugb_decoder_set_trace": (_int, [_vp, ctypes.c_int32]),
    "ugb_decoder_set_wait_limit": (_int, [_vp, _u64]),
    "ugb_decoder_prefill_prepare": (_int, [_vp, _vp, ctypes.c_int32]),
    "ugb_decoder_prefill": (_int, [_vp, _vp, _vp, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]),
    "ugb_decoder_prefill_async": (_int, [_vp, _vp, _vp, ctypes.c_int32, ctypes.c_int32]),
    "ugb_decoder_prefill_trace_bytes": (ctypes.c_size_t, [_vp, ctypes.c_int32]),
    "ugb_decoder_read_prefill_trace": (_int, [_vp, _vp, ctypes.c_int32, ctypes.c_int32, _vp, ctypes.c_size_t]),
    "ugb_decoder_test_unreachable_wait": (_int, [_vp, ctypes.c_int32]),
    "ugb_decoder_trace_bytes": (ctypes.c_size_t, [_vp, ctypes.c_int32]),
    "ugb_decoder_read_trace": (_int, [_vp, _vp, ctypes.c_int32, ctypes.c_int32, _vp, ctypes.c_size_t]),
    "ugb_gguf_parse": (ctypes.c_int32, [_vp, ctypes.c_size_t, _u64, ctypes.POINTER(_vp)]),
    "ugb_gguf_free": (None, [_vp]),
    "ugb_gguf_info": (ctypes.c_int32, [_vp, ctypes.POINTER(_u64), ctypes.POINTER(_u64), ctypes.POINTER(_u64),
                                       ctypes.POINTER(_u64), ctypes.POINTER(_i64)]),
    "ugb_gguf_tensor_at": (ctypes.c_int32, [_vp, _i64, _vp]),
    "ugb_gguf_find_tensor": (ctypes.c_int32, [_vp, ctypes.c_char_p, _vp]),
    "ugb_gguf_tensor_rows": (ctypes.c_int32, [_vp, _u64, _u64, ctypes.POINTER(_u64), ctypes.POINTER(_u64)]),
    "ugb_gguf_tensor_expert": (ctypes.c_int32, [_vp, _u32, ctypes.POINTER(_u64), ctypes.POINTER(_u64)]),
    "ugb_gguf_meta_kind": (ctypes.c_int32, [_vp, ctypes.c_char_p, ctypes.POINTER(_u32)]),
    "ugb_gguf_meta_unsigned": (ctypes.c_int32, [_vp, ctypes.c_char_p, ctypes.POINTER(_u64)]),
    "ugb_gguf_meta_float": (ctypes.c_int32, [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float)]),
    "ugb_gguf_meta_string": (ctypes.c_int32, [_vp, ctypes.c_char_p, _vp, ctypes.c_size_t,
                                              ctypes.POINTER(ctypes.c_size_t)]),
    "ugb_gguf_meta_array": (ctypes.c_int32, [_vp, ctypes.c_char_p, ctypes.POINTER(_u32), ctypes.POINTER(_u64)]),
    "ugb_gguf_meta_array_unsigned": (ctypes.c_int32, [_vp, ctypes.c_char_p, _u64, ctypes.POINTER(_u64)]),
    "ugb_gguf_meta_array_string": (ctypes.c_int32, [_vp, ctypes.c_char_p, _u64, _vp, ctypes.c_size_t,
                                                    ctypes.POINTER(ctypes.c_size_t)]),
    "ugb_gguf_check_index": (ctypes.c_int32, [_vp, ctypes.c_int32]),
    "ugb_gguf_inventory": (ctypes.c_int32, [_vp, ctypes.c_int32, _vp]),
    "ugb_gguf_decoder_config": (ctypes.c_int32, [_vp, ctypes.c_int32, _vp]),
    "ugb_gguf_model_weights": (ctypes.c_int32, [_vp, ctypes.c_int32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ugb_graph_begin": (_int, [_vp, _vp]),
    "ugb_graph_end": (_int, [_vp, _vp, ctypes.POINTER(_vp)]),
    "ugb_graph_launch": (_int, [_vp, _vp]),
    "ugb_graph_destroy": (_int, [_vp]),
    "ugb_graph_kernels": (_int, [_vp, ctypes.POINTER(_i64)]),
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

    def matvec_f32(self, kind: int, w, rb: int, x, xq_scratch, y, k: int, m: int, batch: int = 1,
                   stream=None) -> None:
        """quant_q8_1 + matvec as one call (fused into the matvec for batch-1 staged shapes)."""
        check("ugb_matvec_f32", lib().ugb_matvec_f32(self.handle, _stream(stream), kind, _ptr(w), rb,
                                                       _ptr(x), _ptr(xq_scratch), _ptr(y), k, m, batch))

    def matvec_multi(self, kind: int, ws, rows, rb: int, xq, y, k: int, batch: int = 1,
                     stream=None) -> None:
        n = len(ws)
        wp = (_vp * n)(*[_ptr(w) for w in ws])
        rp = (_i64 * n)(*rows)
        check("ugb_matvec_multi", lib().ugb_matvec_multi(self.handle, _stream(stream), kind, wp, rp,
                                                           n, rb, _ptr(xq), _ptr(y), k, batch))

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

    # ---- MoE ----------------------------------------------------------------------------------
    def matvec_jobs(self, jobs, batch: int = 1, stream=None) -> None:
        """jobs: list of Job (device pointers)."""
        arr = (Job * len(jobs))(*jobs)
        check("ugb_matvec_jobs", lib().ugb_matvec_jobs(self.handle, _stream(stream), ctypes.cast(arr, _vp),
                                                         len(jobs), batch))

    def moe_route(self, logits, n_expert: int, top_k: int, batch: int, ids, weights, stream=None) -> None:
        check("ugb_moe_route", lib().ugb_moe_route(self.handle, _stream(stream), _ptr(logits), n_expert, top_k,
                                                     batch, _ptr(ids), _ptr(weights)))

    def moe_combine(self, values, weights, ids, top_k: int, d: int, batch: int, out, expert0: int = 0,
                    n_local: int = 1 << 30, accumulate: bool = False, stream=None) -> None:
        check("ugb_moe_combine", lib().ugb_moe_combine(self.handle, _stream(stream), _ptr(values), _ptr(weights),
                                                         _ptr(ids), top_k, d, batch, expert0, n_local,
                                                         int(accumulate), _ptr(out)))

    def moe_experts(self, args: "MoeArgs", stream=None) -> None:
        check("ugb_moe_experts", lib().ugb_moe_experts(self.handle, _stream(stream), ctypes.byref(args)))

    # ---- Q8 prefill ---------------------------------------------------------------------------
    def prefill_repack_q8_0(self, w, n: int, k: int, packed, stream=None) -> None:
        check("ugb_prefill_repack_q8_0", lib().ugb_prefill_repack_q8_0(self.handle, _stream(stream), _ptr(w),
                                                                         n, k, _ptr(packed)))

    def prefill_quant(self, x, m: int, k: int, packed, stream=None) -> None:
        check("ugb_prefill_quant", lib().ugb_prefill_quant(self.handle, _stream(stream), _ptr(x), m, k,
                                                             _ptr(packed)))

    def prefill_gemm(self, w_packed, x_packed, y, m: int, n: int, k: int, ldy: int | None = None,
                     stream=None) -> None:
        check("ugb_prefill_gemm_q8_0", lib().ugb_prefill_gemm_q8_0(
            self.handle, _stream(stream), _ptr(w_packed), _ptr(x_packed), _ptr(y), m, n, k,
            n if ldy is None else ldy))

    def prefill_block_dots(self, w_packed, x_packed, dots, y, m: int, n: int, k: int, stream=None) -> None:
        check("ugb_prefill_block_dots", lib().ugb_prefill_block_dots(
            self.handle, _stream(stream), _ptr(w_packed), _ptr(x_packed), _ptr(dots), _ptr(y), m, n, k))

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

    def linear_static(self, kind: int, w, rb: int, x_host, k: int, m: int, stream=None):
        """ugb_linear with the library's fixed device scratch (no allocation)."""
        import numpy as np
        x = np.ascontiguousarray(x_host, dtype=np.float32)
        y = np.empty(m, dtype=np.float32)
        code = lib().ugb_linear_static(self.handle, _stream(stream), kind, _ptr(w), rb,
                                       x.ctypes.data, y.ctypes.data, k, m)
        check("ugb_linear_static", code)
        return y


class Job(ctypes.Structure):
    """ugb_job: the 48-byte FrontierJob descriptor layout."""
    _fields_ = [("weights", ctypes.c_uint64), ("input", ctypes.c_uint64), ("output", ctypes.c_uint64),
                ("kind", ctypes.c_uint32), ("n", ctypes.c_uint32), ("m", ctypes.c_uint32),
                ("row_bytes", ctypes.c_uint32), ("first_row", ctypes.c_uint32), ("padding", ctypes.c_uint32)]


assert ctypes.sizeof(Job) == 48


class MoeArgs(ctypes.Structure):
    """ugb_moe_args."""
    _fields_ = [("kind", ctypes.c_uint32), ("accumulate", ctypes.c_int32),
                ("hidden", ctypes.c_int64), ("ffn", ctypes.c_int64), ("top_k", ctypes.c_int64),
                ("batch", ctypes.c_int64), ("n_expert", ctypes.c_int64), ("expert0", ctypes.c_int64),
                ("n_expert_total", ctypes.c_int64), ("gate", _vp), ("up", _vp), ("down", _vp), ("xq", _vp),
                ("ids", _vp), ("weights", _vp), ("out", _vp), ("workspace", _vp),
                ("workspace_bytes", ctypes.c_size_t)]


def moe_workspace_bytes(hidden: int, ffn: int, top_k: int, batch: int) -> int:
    return lib().ugb_moe_workspace_bytes(hidden, ffn, top_k, batch)


def moe_workspace_layout(hidden: int, ffn: int, top_k: int, batch: int) -> dict:
    """Offsets of the ugb_moe_experts workspace regions (as include/ugb.h documents them)."""
    slots = top_k * batch
    rup = lambda v: (v + 255) // 256 * 256
    hq = rup(slots * 2 * ffn * 4)
    hq_bytes = q8act_bytes(ffn, slots)
    return {"slots": slots, "gu": 0, "hq": hq, "values": hq + rup(hq_bytes)}


def prefill_packed_bytes(rows: int, k: int) -> int:
    """Bytes of a packed prefill operand (ugb_prefill_packed_bytes)."""
    v = lib().ugb_prefill_packed_bytes(rows, k)
    if v < 0:
        raise UgbError("ugb_prefill_packed_bytes", ESHAPE)
    return v


def alloc_prefill(rows: int, k: int, device=None):
    """A 16-byte aligned device buffer for a packed prefill operand."""
    import torch
    n = prefill_packed_bytes(rows, k)
    return torch.empty(n, dtype=torch.uint8, device=device or "cuda")


class DecoderConfig(ctypes.Structure):
    """ugb_decoder_config."""
    _fields_ = [("n_layer", ctypes.c_int32), ("n_embd", ctypes.c_int32), ("n_ff", ctypes.c_int32),
                ("n_head", ctypes.c_int32), ("n_head_kv", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("n_vocab", ctypes.c_int32), ("n_ctx", ctypes.c_int32),
                ("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float),
                ("kind", ctypes.c_uint32), ("head_kind", ctypes.c_uint32), ("batch", ctypes.c_int32),
                ("n_expert", ctypes.c_int32), ("top_k", ctypes.c_int32), ("n_ff_expert", ctypes.c_int32),
                ("expert_kind", ctypes.c_uint32), ("expert0", ctypes.c_int32), ("n_expert_local", ctypes.c_int32),
                ("vocab0", ctypes.c_int32), ("n_vocab_local", ctypes.c_int32), ("kv_type", ctypes.c_uint32)]


class LayerWeights(ctypes.Structure):
    """ugb_layer_weights (device pointers)."""
    _fields_ = [(n, _vp) for n in ("attn_norm", "wq", "wk", "wv", "bq", "bk", "bv", "wo",
                                   "ffn_norm", "w_gate", "w_up", "w_down",
                                   "router", "gate_exps", "up_exps", "down_exps")]


class ModelWeights(ctypes.Structure):
    """ugb_model_weights."""
    _fields_ = [("tok_embd", _vp), ("output_norm", _vp), ("output", _vp),
                ("layers", ctypes.POINTER(LayerWeights))]


# Fields of the step trace (ugb_decoder_set_trace), in the order of ugb.h's UGB_TRACE_* list.
TRACE_FIELDS = ("X", "ATTN_NORM", "ATTN_XQ", "QKV", "ATT", "ATT_XQ", "O", "FFN_NORM", "FFN_XQ", "GATE_UP", "H",
                "H_XQ", "DOWN")
TRACE = {name: i for i, name in enumerate(TRACE_FIELDS)}

COMM_ID_BYTES = 128
# How a decoder step runs (ugb_decoder_set_path): persistent token kernel where it applies, the
# per-kernel launch chain, or the persistent token kernel only.
PATH_AUTO, PATH_CHAIN, PATH_TOKEN = 0, 1, 2


class Comm:
    """ugb_comm: an NCCL communicator for a sharded decoder.  Every rank constructs it at the
    same time with the id rank 0 made (comm_unique_id)."""

    def __init__(self, ctx: "Context", rank: int, world: int, uid: bytes):
        buf = (ctypes.c_uint8 * COMM_ID_BYTES).from_buffer_copy(uid)
        h = _vp()
        check("ugb_comm_init", lib().ugb_comm_init(ctx.handle, rank, world, buf, ctypes.byref(h)))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            lib().ugb_comm_destroy(self.handle)
            self.handle = None

    def allreduce_f32(self, buf, stream=None) -> None:
        """In-place sum over the ranks of a float32 device tensor (rank order, deterministic)."""
        check("ugb_comm_allreduce_f32", lib().ugb_comm_allreduce_f32(self.handle, _stream(stream), _ptr(buf),
                                                                       buf.numel()))

    def allreduce_max_u64(self, buf, stream=None) -> None:
        """In-place maximum over the ranks of an int64 device tensor read as unsigned 64-bit."""
        check("ugb_comm_allreduce_max_u64", lib().ugb_comm_allreduce_max_u64(self.handle, _stream(stream),
                                                                               _ptr(buf), buf.numel()))


def comm_unique_id() -> bytes:
    buf = (ctypes.c_uint8 * COMM_ID_BYTES)()
    check("ugb_comm_unique_id", lib().ugb_comm_unique_id(buf))
    return bytes(buf)


QWEN25_15B = dict(n_layer=28, n_embd=1536, n_ff=8960, n_head=12, n_head_kv=2, head_dim=128,
                  n_vocab=151936, n_ctx=512, rope_theta=1e6, norm_eps=1e-6, kind=8, head_kind=8, batch=1)


class Decoder:
    """ugb_decoder: the per-token decode graph around the quantised matvecs."""

    def __init__(self, ctx: "Context", **cfg):
        self.ctx = ctx
        cfg.setdefault("batch", 1)
        self.cfg = DecoderConfig(**cfg)
        h = _vp()
        check("ugb_decoder_create", lib().ugb_decoder_create(ctx.handle, ctypes.byref(self.cfg),
                                                               ctypes.byref(h)))
        self.handle = h
        self._keep = None

    def close(self) -> None:
        if self.handle:
            lib().ugb_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synthetic(self, seed: int) -> None:
        check("ugb_decoder_synthetic", lib().ugb_decoder_synthetic(self.handle, seed))

    def bind(self, tok_embd, output_norm, output, layers) -> None:
        """layers: list of dicts of torch tensors keyed like LayerWeights (None = absent)."""
        arr = (LayerWeights * len(layers))()
        for i, L in enumerate(layers):
            for name, _ in LayerWeights._fields_:
                t = L.get(name)
                setattr(arr[i], name, t.data_ptr() if t is not None else None)
        w = ModelWeights(tok_embd.data_ptr(), output_norm.data_ptr(), output.data_ptr(), arr)
        self._keep = (arr, w, tok_embd, output_norm, output, layers)
        check("ugb_decoder_bind", lib().ugb_decoder_bind(self.handle, ctypes.byref(w)))

    def step(self, stream=None) -> None:
        check("ugb_decoder_step", lib().ugb_decoder_step(self.handle, _stream(stream)))

    def set_state(self, token: int, pos: int, stream=None) -> None:
        check("ugb_decoder_set_state", lib().ugb_decoder_set_state(self.handle, _stream(stream),
                                                                     token, pos))

    def set_tokens(self, tokens, pos: int, stream=None) -> None:
        arr = (ctypes.c_int32 * len(tokens))(*tokens)
        check("ugb_decoder_set_tokens", lib().ugb_decoder_set_tokens(self.handle, _stream(stream), arr, pos))

    def set_comm(self, comm: "Comm | None") -> None:
        check("ugb_decoder_set_comm", lib().ugb_decoder_set_comm(self.handle, comm.handle if comm else None))

    def set_path(self, path: int) -> int:
        """PATH_AUTO / PATH_CHAIN / PATH_TOKEN; returns the path the next steps take."""
        active = ctypes.c_int32()
        check("ugb_decoder_set_path", lib().ugb_decoder_set_path(self.handle, path, ctypes.byref(active)))
        return active.value

    def get_state(self, stream=None):
        t, p, n = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        check("ugb_decoder_get_state", lib().ugb_decoder_get_state(
            self.handle, _stream(stream), ctypes.byref(t), ctypes.byref(p), ctypes.byref(n)))
        return t.value, p.value, n.value

    def get_tokens(self, stream=None):
        """(tokens[batch], pos, next_tokens[batch])."""
        b = self.cfg.batch
        t, n, p = (ctypes.c_int32 * b)(), (ctypes.c_int32 * b)(), ctypes.c_int32()
        check("ugb_decoder_get_tokens", lib().ugb_decoder_get_tokens(self.handle, _stream(stream), t,
                                                                       ctypes.byref(p), n))
        return list(t), p.value, list(n)

    def logits(self, stream=None):
        import numpy as np
        n = self.cfg.n_vocab_local or self.cfg.n_vocab
        out = np.empty((self.cfg.batch, n), dtype=np.float32)
        check("ugb_decoder_logits", lib().ugb_decoder_logits(self.handle, _stream(stream), out.ctypes.data))
        return out[0] if self.cfg.batch == 1 else out

    def read_kv(self, layer: int, pos: int, count: int = 1, seq: int = 0, stream=None):
        """(keys, values), each float32 [n_head_kv, count, head_dim] (rotated keys)."""
        import numpy as np
        shape = (self.cfg.n_head_kv, count, self.cfg.head_dim)
        k = np.empty(shape, dtype=np.float32)
        v = np.empty(shape, dtype=np.float32)
        check("ugb_decoder_read_kv", lib().ugb_decoder_read_kv(self.handle, _stream(stream), seq, layer, pos,
                                                                 count, k.ctypes.data, v.ctypes.data))
        return k, v

    def write_kv(self, layer: int, pos: int, keys, values, seq: int = 0, stream=None) -> None:
        """keys, values: float32 [n_head_kv, count, head_dim] (rotated keys) into the cache."""
        import numpy as np
        k = np.ascontiguousarray(keys, dtype=np.float32)
        v = np.ascontiguousarray(values, dtype=np.float32)
        assert k.shape == v.shape and k.shape[0] == self.cfg.n_head_kv and k.shape[2] == self.cfg.head_dim
        check("ugb_decoder_write_kv", lib().ugb_decoder_write_kv(self.handle, _stream(stream), seq, layer, pos,
                                                                   k.shape[1], k.ctypes.data, v.ctypes.data))

    def set_wait_limit(self, ns: int) -> None:
        check("ugb_decoder_set_wait_limit", lib().ugb_decoder_set_wait_limit(self.handle, ns))

    def test_unreachable_wait(self, enable: bool) -> None:
        check("ugb_decoder_test_unreachable_wait",
              lib().ugb_decoder_test_unreachable_wait(self.handle, 1 if enable else 0))

    def set_trace(self, enable: bool) -> None:
        check("ugb_decoder_set_trace", lib().ugb_decoder_set_trace(self.handle, 1 if enable else 0))

    def trace(self, layer: int, field: str, stream=None):
        """One field of the last traced step: float32 [batch, len], or for a Q8_1 field
        (name ending in _XQ) the tuple (q int8 [batch, n], d f32 [batch, n/32], s int32 [batch, n/32])."""
        import numpy as np
        f = TRACE[field]
        n = lib().ugb_decoder_trace_bytes(self.handle, f)
        raw = np.empty(n, dtype=np.uint8)
        check("ugb_decoder_read_trace", lib().ugb_decoder_read_trace(self.handle, _stream(stream), layer, f,
                                                                       raw.ctypes.data, n))
        b = self.cfg.batch
        if not field.endswith("_XQ"):
            return raw.view(np.float32).reshape(b, -1)
        k = {"ATTN_XQ": self.cfg.n_embd, "FFN_XQ": self.cfg.n_embd, "ATT_XQ": self.cfg.n_head * self.cfg.head_dim,
             "H_XQ": self.cfg.n_ff}[field]
        d_off, s_off = q8act_offsets(k, b)
        nb, nbp = k // 32, (k // 32 + 3) // 4 * 4
        q = raw[: b * k].view(np.int8).reshape(b, k)
        d = raw[d_off: d_off + b * nbp * 4].view(np.float32).reshape(b, nbp)[:, :nb]
        s = raw[s_off: s_off + b * nbp * 4].view(np.int32).reshape(b, nbp)[:, :nb]
        return q, d, s

    def prefill_prepare(self, max_tokens: int, stream=None) -> None:
        check("ugb_decoder_prefill_prepare", lib().ugb_decoder_prefill_prepare(self.handle, _stream(stream), max_tokens))
        self.prefill_max = max_tokens

    def prefill(self, tokens, pos0: int = 0, stream=None) -> int:
        """Whole-prompt prefill of host tokens from position pos0; returns the greedy next token."""
        arr = (ctypes.c_int32 * len(tokens))(*[int(t) for t in tokens])
        nxt = ctypes.c_int32()
        check("ugb_decoder_prefill", lib().ugb_decoder_prefill(self.handle, _stream(stream), arr, len(tokens), pos0,
                                                                 ctypes.byref(nxt)))
        return nxt.value

    def prefill_async(self, tokens_dev, n: int, pos0: int = 0, stream=None) -> None:
        """tokens_dev: int32 device tensor of at least n tokens."""
        check("ugb_decoder_prefill_async", lib().ugb_decoder_prefill_async(self.handle, _stream(stream),
                                                                             _ptr(tokens_dev), n, pos0))

    def prefill_trace(self, layer: int, field: str, n: int, stream=None):
        """One field of the last traced prefill: float32 [n, len] (record n_layer: [1, len] of the last
        token, and ATTN_XQ as the (q, d, s) of its batch-1 Q8_1 head input)."""
        import numpy as np
        f = TRACE[field]
        final = layer == self.cfg.n_layer
        E = self.cfg.n_embd
        if field == "ATTN_XQ":
            assert final
            nbytes = q8act_bytes(E, 1)
        else:
            total = lib().ugb_decoder_prefill_trace_bytes(self.handle, f)
            nbytes = total // self.prefill_max * (1 if final else n)
        raw = np.empty(nbytes, dtype=np.uint8)
        check("ugb_decoder_read_prefill_trace", lib().ugb_decoder_read_prefill_trace(
            self.handle, _stream(stream), layer, f, raw.ctypes.data, nbytes))
        if field != "ATTN_XQ":
            return raw.view(np.float32).reshape(1 if final else n, -1)
        d_off, s_off = q8act_offsets(E, 1)
        nb = E // 32
        return (raw[:E].view(np.int8).reshape(1, E), raw[d_off:d_off + 4 * nb].view(np.float32).reshape(1, nb),
                raw[s_off:s_off + 4 * nb].view(np.int32).reshape(1, nb))

    def tokens(self, tokens, pos: int, stream=None):
        b = self.cfg.batch
        arr = (ctypes.c_int32 * b)(*tokens)
        nxt = (ctypes.c_int32 * b)()
        check("ugb_decoder_tokens", lib().ugb_decoder_tokens(self.handle, _stream(stream), arr, pos, nxt))
        return list(nxt)

    def token(self, token: int, pos: int, stream=None) -> int:
        nxt = ctypes.c_int32()
        check("ugb_decoder_token", lib().ugb_decoder_token(self.handle, _stream(stream), token, pos,
                                                             ctypes.byref(nxt)))
        return nxt.value


GGUF_ERRORS = ("ok", "truncated", "magic", "version", "limit", "type", "utf8", "alignment", "shape", "overflow",
               "tensor_bounds", "overlap", "duplicate", "missing", "split")


class GgufError(ValueError):
    def __init__(self, fn: str, code: int):
        name = GGUF_ERRORS[code] if 0 <= code < len(GGUF_ERRORS) else str(code)
        super().__init__(f"{fn} failed: {name} ({code})")
        self.code = code
        self.name = name


def _gcheck(fn: str, code: int) -> None:
    if code != 0:
        raise GgufError(fn, code)


class GgufTensor(ctypes.Structure):
    """ugb_gguf_tensor."""
    _fields_ = [("name", ctypes.c_char_p), ("dims", _u64 * 4), ("rank", _u32), ("kind", _u32),
                ("offset", _u64), ("bytes", _u64), ("row_bytes", _u64)]


class Gguf:
    """A parsed GGUF directory (ugb_gguf_parse): one file or one shard of a split model."""

    def __init__(self, prefix: bytes, logical_bytes: int | None = None):
        buf = (ctypes.c_uint8 * len(prefix)).from_buffer_copy(prefix) if prefix else None
        h = _vp()
        total = len(prefix) if logical_bytes is None else logical_bytes
        _gcheck("ugb_gguf_parse", lib().ugb_gguf_parse(buf, len(prefix), total, ctypes.byref(h)))
        self.handle = h

    @classmethod
    def open(cls, path: str) -> "Gguf":
        """Parse the directory of a file (its first 16 MiB hold it, as the format's limits require)."""
        size = os.path.getsize(path)
        with open(path, "rb") as f:
            prefix = f.read(min(size, 16 * 1024 * 1024))
        return cls(prefix, size)

    def close(self) -> None:
        if self.handle:
            lib().ugb_gguf_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> dict:
        v = [_u64() for _ in range(4)]
        n = _i64()
        _gcheck("ugb_gguf_info", lib().ugb_gguf_info(self.handle, *[ctypes.byref(x) for x in v], ctypes.byref(n)))
        return dict(data_offset=v[0].value, split_no=v[1].value, split_count=v[2].value, total_tensors=v[3].value,
                    n_tensors=n.value)

    def tensors(self) -> list:
        out = []
        for i in range(self.info()["n_tensors"]):
            t = GgufTensor()
            _gcheck("ugb_gguf_tensor_at", lib().ugb_gguf_tensor_at(self.handle, i, ctypes.byref(t)))
            out.append(t)
        return out

    def tensor(self, name: str) -> GgufTensor:
        t = GgufTensor()
        _gcheck("ugb_gguf_find_tensor", lib().ugb_gguf_find_tensor(self.handle, name.encode(), ctypes.byref(t)))
        return t

    @staticmethod
    def rows(t: GgufTensor, start: int, count: int) -> tuple[int, int]:
        o, n = _u64(), _u64()
        _gcheck("ugb_gguf_tensor_rows", lib().ugb_gguf_tensor_rows(ctypes.byref(t), start, count, ctypes.byref(o),
                                                                     ctypes.byref(n)))
        return o.value, n.value

    @staticmethod
    def expert(t: GgufTensor, eid: int) -> tuple[int, int]:
        o, n = _u64(), _u64()
        _gcheck("ugb_gguf_tensor_expert", lib().ugb_gguf_tensor_expert(ctypes.byref(t), eid, ctypes.byref(o),
                                                                         ctypes.byref(n)))
        return o.value, n.value

    def meta(self, key: str):
        """A metadata value as Python: int (unsigned kinds), float (f32), str, or list (arrays of
        unsigned or string elements)."""
        k = key.encode()
        kind = _u32()
        _gcheck("ugb_gguf_meta_kind", lib().ugb_gguf_meta_kind(self.handle, k, ctypes.byref(kind)))
        if kind.value in (0, 2, 4, 10):
            v = _u64()
            _gcheck("ugb_gguf_meta_unsigned", lib().ugb_gguf_meta_unsigned(self.handle, k, ctypes.byref(v)))
            return v.value
        if kind.value == 6:
            f = ctypes.c_float()
            _gcheck("ugb_gguf_meta_float", lib().ugb_gguf_meta_float(self.handle, k, ctypes.byref(f)))
            return f.value
        if kind.value == 8:
            return self._string(lambda buf, cap, n: lib().ugb_gguf_meta_string(self.handle, k, buf, cap, n))
        if kind.value == 9:
            ek, count = _u32(), _u64()
            _gcheck("ugb_gguf_meta_array", lib().ugb_gguf_meta_array(self.handle, k, ctypes.byref(ek),
                                                                       ctypes.byref(count)))
            out = []
            for i in range(count.value):
                if ek.value == 8:
                    out.append(self._string(lambda buf, cap, n, i=i: lib().ugb_gguf_meta_array_string(
                        self.handle, k, i, buf, cap, n)))
                else:
                    v = _u64()
                    _gcheck("ugb_gguf_meta_array_unsigned",
                            lib().ugb_gguf_meta_array_unsigned(self.handle, k, i, ctypes.byref(v)))
                    out.append(v.value)
            return out
        raise GgufError("meta", 5)

    @staticmethod
    def _string(call) -> str:
        n = ctypes.c_size_t()
        _gcheck("ugb_gguf_meta_string", call(None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(max(1, n.value))
        _gcheck("ugb_gguf_meta_string", call(buf, n.value, ctypes.byref(n)))
        return buf.raw[:n.value].decode()


def _handles(shards):
    return (_vp * len(shards))(*[s.handle for s in shards])


def gguf_check_index(shards) -> None:
    _gcheck("ugb_gguf_check_index", lib().ugb_gguf_check_index(_handles(shards), len(shards)))


def gguf_inventory(shards) -> list:
    out = (_u64 * 3)()
    _gcheck("ugb_gguf_inventory", lib().ugb_gguf_inventory(_handles(shards), len(shards), out))
    return list(out)


def gguf_decoder_config(shards) -> dict:
    cfg = DecoderConfig()
    _gcheck("ugb_gguf_decoder_config", lib().ugb_gguf_decoder_config(_handles(shards), len(shards),
                                                                       ctypes.byref(cfg)))
    return {name: getattr(cfg, name) for name, _ in DecoderConfig._fields_}


def gguf_model_weights(shards, dev_bases, base_offsets, dev_sizes, cfg: dict):
    """(ModelWeights, LayerWeights array) pointing into the shards' device copies."""
    n = len(shards)
    c = DecoderConfig(**cfg)
    layers = (LayerWeights * c.n_layer)()
    w = ModelWeights()
    _gcheck("ugb_gguf_model_weights", lib().ugb_gguf_model_weights(
        _handles(shards), n, (_vp * n)(*dev_bases), (_u64 * n)(*base_offsets), (_u64 * n)(*dev_sizes),
        ctypes.byref(c), ctypes.byref(w), layers))
    return w, layers


def load_gguf_decoder(ctx: "Context", path: str, **overrides) -> "Decoder":
    """A decoder bound to the weights of a GGUF file: the directory is parsed, the data section
    is copied to the device once (owned by the returned decoder), and every tensor is bound in
    place.  overrides replace configuration fields (e.g. n_ctx, batch, kv_type)."""
    import numpy as np
    import torch
    g = Gguf.open(path)
    info = g.info()
    cfg = gguf_decoder_config([g])
    cfg.update(overrides)
    data = np.fromfile(path, dtype=np.uint8, offset=info["data_offset"])
    dev = torch.from_numpy(data).to(torch.device("cuda", ctx.device))
    w, layers = gguf_model_weights([g], [dev.data_ptr()], [info["data_offset"]], [dev.numel()], cfg)
    dec = Decoder(ctx, **cfg)
    check("ugb_decoder_bind", lib().ugb_decoder_bind(dec.handle, ctypes.byref(w)))
    dec._keep = (w, layers, dev, g)
    return dec


class Graph:
    """An instantiated CUDA graph of ugb_* calls (ugb_graph_end / launch / destroy)."""

    def __init__(self, handle):
        self.handle = handle

    def launch(self, stream=None) -> None:
        check("ugb_graph_launch", lib().ugb_graph_launch(self.handle, _stream(stream)))

    def kernels(self) -> int:
        """Kernel launches per replay (ugb_graph_kernels)."""
        n = _i64(0)
        check("ugb_graph_kernels", lib().ugb_graph_kernels(self.handle, ctypes.byref(n)))
        return n.value

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
