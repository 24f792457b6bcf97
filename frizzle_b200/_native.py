"""ctypes bindings of the C ABI (include/frizzle_b200.h).

The library is built in-tree (frizzle_b200/_lib/libfrizzle_b200.so).  There
is no CPU fallback: if the library cannot be loaded or built, importing the
bindings raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libfrizzle_b200.so")

_lock = threading.Lock()
_lib = None

OK = 0
STATUS = {0: "OK", 1: "ARGUMENT", 2: "CUDA", 3: "INDEX", 4: "ARCHITECTURE", 5: "FIT", 6: "UPLOAD", 7: "STATE",
          8: "EDITS", 9: "TRUNCATED", 10: "DEVICE_LOST", 11: "NOT_SUPPORTED"}


class FzError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status
        self.message = message


class Step(C.Structure):
    _fields_ = [("position", C.c_uint32), ("tokens", C.c_uint32), ("logits", C.c_uint32), ("fed", C.c_uint32),
                ("seed", C.c_uint32 * 2), ("top_k", C.c_uint32), ("temperature", C.c_float), ("top_p", C.c_float),
                ("min_p", C.c_float), ("log_min_p", C.c_float), ("capture", C.c_uint32),
                ("padding", C.c_uint32 * 4)]


class Record(C.Structure):
    _fields_ = [("token", C.c_uint32), ("failed", C.c_uint32), ("u", C.c_float), ("padding", C.c_uint32)]


class ModelInfo(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("layers", "hidden", "ffn", "heads", "kv_heads", "head_dim", "vocab",
                                           "window", "pattern", "context")] + \
               [("eps", C.c_float), ("rope_global", C.c_float), ("rope_local", C.c_float),
                ("weight_bytes", C.c_uint64)]


class Plan(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("sequences", "context", "rollback", "rows")] + \
               [(n, C.c_uint64) for n in ("budget", "weight_bytes", "copy_bytes", "scratch_bytes", "cache_bytes",
                                           "total_bytes")]


class CaptureSlot(C.Structure):
    _fields_ = [("first", C.c_uint32), ("width", C.c_uint32)]


class CaptureSlots(C.Structure):
    _fields_ = [(n, CaptureSlot) for n in ("neurons", "residual", "attention_added", "mlp_added", "query",
                                             "weights", "stats", "readout")] + \
               [(n, C.c_uint32) for n in ("keys", "query_heads", "window", "full_attention")]


# Every symbol the header declares, with its signature.
VP = C.c_void_p
U32 = C.c_uint32
SIGNATURES = {
    "fz_last_error": (C.c_char_p, []),
    "fz_device_open": (C.c_int, [C.c_int, C.POINTER(VP)]),
    "fz_device_close": (C.c_int, [VP]),
    "fz_device_stream": (VP, [VP]),
    "fz_model_index_check": (C.c_int, [VP, C.c_uint64, C.c_uint64, C.POINTER(ModelInfo)]),
    "fz_model_load_begin": (C.c_int, [VP, VP, C.c_uint64, C.c_uint64, C.POINTER(VP)]),
    "fz_model_index_needed": (C.c_uint64, []),
    "fz_model_load_write": (C.c_int, [VP, C.c_uint64, VP, C.c_uint64]),
    "fz_model_load_finish": (C.c_int, [VP]),
    "fz_model_info_get": (C.c_int, [VP, C.POINTER(ModelInfo)]),
    "fz_model_free": (C.c_int, [VP]),
    "fz_batch_create": (C.c_int, [VP, U32, U32, U32, C.POINTER(VP)]),
    "fz_batch_free": (C.c_int, [VP]),
    "fz_batch_set_edits": (C.c_int, [VP, U32, VP, C.c_size_t]),
    "fz_batch_step": (C.c_int, [VP, C.POINTER(Step), VP, VP]),
    "fz_batch_wait": (C.c_int, [VP, VP]),
    "fz_batch_wait_oldest": (C.c_int, [VP, VP]),
    "fz_batch_read_logits": (C.c_int, [VP, U32, VP, C.c_size_t]),
    "fz_capture_floats": (C.c_size_t, [VP]),
    "fz_batch_read_capture": (C.c_int, [VP, U32, VP, C.c_size_t]),
    "fz_capture_layout": (C.c_int, [VP, U32, C.POINTER(CaptureSlots)]),
    "fz_batch_cache": (C.c_int, [VP, U32, U32, C.c_int, C.POINTER(VP), C.POINTER(U32)]),
    "fz_batch_truncate": (C.c_int, [VP, U32, C.POINTER(U32)]),
    "fz_batch_cache_state": (C.c_int, [VP, C.POINTER(U32), C.POINTER(U32)]),
    "fz_cache_truncate_keeps": (C.c_int, [VP, VP, U32, U32, U32]),
    "fz_batch_trace": (C.c_int, [VP, C.c_int]),
    "fz_batch_set_wait_limit": (C.c_int, [VP, C.c_uint32]),
    "fz_batch_time_decode": (C.c_int, [VP, C.c_int]),
    "fz_batch_cache_advance": (C.c_int, [VP, C.c_uint32]),
    "fz_model_plan": (C.c_int, [VP, C.POINTER(Plan)]),
    "fz_model_index_plan": (C.c_int, [VP, C.c_uint64, C.c_uint64, C.POINTER(Plan)]),
    "fz_batch_decode_time": (C.c_int, [VP, C.POINTER(C.c_float)]),
    "fz_batch_inject_stale_epoch": (C.c_int, [VP, C.c_int]),
    "fz_batch_read_trace": (C.c_int, [VP, VP, C.c_size_t, C.POINTER(U32), C.POINTER(U32)]),
    "fz_q4_0_codes_bytes": (C.c_size_t, [U32, U32]),
    "fz_q4_0_scales_bytes": (C.c_size_t, [U32, U32]),
    "fz_q4_0_repack": (C.c_int, [VP, U32, U32, VP, VP, VP]),
    "fz_q4_0_rows": (C.c_int, [VP, VP, U32, U32, VP, U32, C.c_float, VP, VP]),
    "fz_q4_0_matvec": (C.c_int, [VP, VP, U32, U32, VP, U32, VP, VP]),
    "fz_q4_0_gated": (C.c_int, [VP, VP, VP, VP, U32, U32, VP, U32, VP, U32, U32, VP, VP]),
    "fz_q4_0_head": (C.c_int, [VP, VP, U32, U32, VP, U32, VP, VP, VP]),
    "fz_q8_0_codes_bytes": (C.c_size_t, [U32, U32]),
    "fz_q8_0_scales_bytes": (C.c_size_t, [U32, U32]),
    "fz_q4_1_codes_bytes": (C.c_size_t, [U32, U32]),
    "fz_q4_1_scales_bytes": (C.c_size_t, [U32, U32]),
    "fz_q8_0_repack": (C.c_int, [VP, U32, U32, VP, VP, VP]),
    "fz_q4_1_repack": (C.c_int, [VP, U32, U32, VP, VP, VP]),
    "fz_q8_0_rows": (C.c_int, [VP, VP, U32, U32, VP, U32, C.c_float, VP, VP]),
    "fz_q4_1_rows": (C.c_int, [VP, VP, U32, U32, VP, U32, C.c_float, VP, VP]),
    "fz_q8_0_matvec": (C.c_int, [VP, VP, U32, U32, VP, U32, VP, VP]),
    "fz_q4_1_matvec": (C.c_int, [VP, VP, U32, U32, VP, U32, VP, VP]),
    "fz_q4_0_gemm": (C.c_int, [VP, VP, U32, U32, VP, VP, U32, U32, VP, VP, VP]),
    "fz_q4_0_to_f16": (C.c_int, [VP, VP, U32, U32, VP, VP, VP]),
    "fz_f16_gemm": (C.c_int, [VP, VP, U32, U32, VP, VP, U32, U32, VP, VP, VP]),
    "fz_f16_gemm_gated": (C.c_int, [VP, VP, VP, VP, U32, U32, VP, VP, U32, U32, VP, U32, U32, VP, VP, VP, VP, VP]),
    "fz_q4_0_gemm_gated": (C.c_int, [VP, VP, VP, VP, U32, U32, VP, VP, U32, U32, VP, U32, U32, VP, VP, VP, VP, VP]),
    "fz_split_f16": (C.c_int, [VP, C.c_size_t, VP, VP, VP]),
    "fz_attention": (C.c_int, [VP, VP, VP, U32, U32, U32, U32, U32, U32, U32, VP, VP, VP, VP, VP]),
    "fz_attention_splits": (U32, [U32, U32, U32]),
    "fz_attention_wide": (C.c_int, [VP, VP, VP, U32, U32, U32, U32, U32, U32, U32, VP, VP, VP, VP, VP, VP]),
    "fz_attention_static": (C.c_int, [VP, VP, VP, U32, U32, U32, U32, U32, U32, U32, VP, VP]),
}


def load(build_if_missing: bool = True):
    """The loaded library; builds it first when it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            if not build_if_missing:
                raise OSError(f"{LIB_PATH} is not built")
            from . import build
            build.build()
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != OK:
        raise FzError(status, load().fz_last_error().decode("utf-8", "replace"))
