"""ctypes face of the CPU oracle (``oracle/oracle.c``): TEST INFRASTRUCTURE ONLY.

Only tests, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this package, as the checker of the CUDA path.  The product never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

_lib = None

ROLES = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_q_norm", "attn_k_norm", "attn_output",
         "post_attention_norm", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down", "post_ffw_norm")


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE, "CC=gcc"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        try:
            _lib = C.CDLL(LIB_PATH)
        except OSError:
            subprocess.run(["make", "-s", "-C", HERE, "clean"], check=True)
            build()
            _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


class Shape(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "hidden", "ffn", "heads", "kv_heads", "head_dim", "vocab",
                                        "window", "pattern")] + \
               [("rope_global", C.c_float), ("rope_local", C.c_float), ("eps", C.c_float), ("context", C.c_int)]


P = C.c_void_p
F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
U32P = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
U8P = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def _declare(L):
    L.oracle_f16_to_f32.argtypes = [C.c_uint16]; L.oracle_f16_to_f32.restype = C.c_float
    L.oracle_f32_to_f16.argtypes = [C.c_float]; L.oracle_f32_to_f16.restype = C.c_uint16
    L.oracle_f16_pack.argtypes = [C.c_float]; L.oracle_f16_pack.restype = C.c_uint16
    L.oracle_q4_0_dequant.argtypes = [U8P, C.c_int64, F32P]
    L.oracle_matmul.argtypes = [U8P, C.c_int, C.c_int, F32P, C.c_int, F32P]
    L.oracle_matmul_fmt.argtypes = [C.c_int, U8P, C.c_int, C.c_int, F32P, C.c_int, F32P]
    L.oracle_matmul_fmt.restype = C.c_int
    L.oracle_blocks_dequant.argtypes = [C.c_int, U8P, C.c_int64, F32P]
    L.oracle_blocks_dequant.restype = C.c_int
    L.oracle_gated.argtypes = [U8P, U8P, C.c_int, C.c_int, F32P, C.c_int, F32P]
    L.oracle_exp_nonpositive.argtypes = [C.c_float]; L.oracle_exp_nonpositive.restype = C.c_float
    L.oracle_gelu.argtypes = [C.c_float]; L.oracle_gelu.restype = C.c_float
    L.oracle_norm_row.argtypes = [F32P, P, P, F32P, C.c_int, C.c_float, F32P, P]
    L.oracle_rope_turns.argtypes = [C.c_float, C.c_int, F32P]
    L.oracle_attention.argtypes = [F32P, P, P, C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_uint32, C.c_float,
                                   C.c_uint32, C.c_int, F32P]
    L.oracle_edit_apply.argtypes = [P, C.c_uint32, C.c_uint32, C.c_int, C.c_int, F32P]
    L.oracle_topk_key.argtypes = [C.c_uint32]; L.oracle_topk_key.restype = C.c_uint32
    L.oracle_topk64.argtypes = [F32P, C.c_int64, U32P]
    L.oracle_philox.argtypes = [U32P, U32P, U32P]
    L.oracle_draw.argtypes = [U32P, C.c_uint32, C.c_float, C.c_float, C.c_float, C.c_float, U32P,
                              C.c_uint32, U32P]
    L.oracle_ctx_new.argtypes = [C.POINTER(Shape), P, P, C.POINTER(C.c_void_p), C.c_uint32, C.c_uint32]
    L.oracle_ctx_new.restype = P
    L.oracle_ctx_free.argtypes = [P]
    L.oracle_ctx_slots.argtypes = [P, C.c_int]; L.oracle_ctx_slots.restype = C.c_uint32
    L.oracle_ctx_keys.argtypes = [P, C.c_int]; L.oracle_ctx_keys.restype = P
    L.oracle_ctx_values.argtypes = [P, C.c_int]; L.oracle_ctx_values.restype = P
    L.oracle_capture_floats.argtypes = [C.POINTER(Shape)]; L.oracle_capture_floats.restype = C.c_int64
    L.oracle_capture_slots.argtypes = [C.POINTER(Shape), C.c_int, P, P]
    L.oracle_capture_slots.restype = C.c_int64
    L.oracle_step.argtypes = [P, C.c_uint32, C.c_int, U32P, P, P, P]
    L.oracle_threads.restype = C.c_int
    L.oracle_ctx_set_types.argtypes = [P, C.c_int, P]
    L.oracle_ctx_set_types.restype = C.c_int
    L.oracle_set_threads.argtypes = [C.c_int]


# ------------------------------------------------------------ small helpers

def matmul(blocks: np.ndarray, n: int, k: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = np.empty((x.shape[0], n), dtype=np.float32)
    lib().oracle_matmul(np.ascontiguousarray(blocks, dtype=np.uint8), n, k, x, x.shape[0], y)
    return y


def gated(gate: np.ndarray, up: np.ndarray, f: int, k: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = np.empty((x.shape[0], f), dtype=np.float32)
    lib().oracle_gated(np.ascontiguousarray(gate, dtype=np.uint8), np.ascontiguousarray(up, dtype=np.uint8),
                       f, k, x, x.shape[0], y)
    return y


# GGUF type numbers (gguf::TensorType) and block bytes of the formats the
# oracle restates.
TYPE_Q4_0, TYPE_Q4_1, TYPE_Q8_0 = 2, 3, 8
BLOCK_BYTES = {TYPE_Q4_0: 18, TYPE_Q4_1: 20, TYPE_Q8_0: 34}


def matmul_fmt(gguf_type: int, blocks: np.ndarray, n: int, k: int, x: np.ndarray) -> np.ndarray:
    """y = x W^T over blocks of any restated format, in the reference's order."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = np.empty((x.shape[0], n), dtype=np.float32)
    rc = lib().oracle_matmul_fmt(gguf_type, np.ascontiguousarray(blocks, dtype=np.uint8), n, k, x, x.shape[0], y)
    if rc != 0:
        raise ValueError(f"type {gguf_type} is not restated")
    return y


def dequant_fmt(gguf_type: int, blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    nb = b.size // BLOCK_BYTES[gguf_type]
    out = np.empty(nb * 32, dtype=np.float32)
    if lib().oracle_blocks_dequant(gguf_type, b, nb, out) != 0:
        raise ValueError(f"type {gguf_type} is not restated")
    return out


def dequant(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(b.size // 18 * 32, dtype=np.float32)
    lib().oracle_q4_0_dequant(b, b.size // 18, out)
    return out


def topk64(logits: np.ndarray) -> np.ndarray:
    l = np.ascontiguousarray(logits, dtype=np.float32)
    out = np.empty(128, dtype=np.uint32)
    lib().oracle_topk64(l, l.size, out)
    return out


def philox(counter, key) -> np.ndarray:
    out = np.empty(4, dtype=np.uint32)
    lib().oracle_philox(np.asarray(counter, dtype=np.uint32), np.asarray(key, dtype=np.uint32), out)
    return out


def draw(candidates: np.ndarray, top_k: int, temperature: float, top_p: float, min_p: float, seed, counter: int):
    rec = np.empty(4, dtype=np.uint32)
    log_min_p = float(np.log(np.float32(min_p))) if min_p > 0 else 0.0
    lib().oracle_draw(np.ascontiguousarray(candidates, dtype=np.uint32), top_k, temperature, top_p, min_p,
                      log_min_p, np.asarray(seed, dtype=np.uint32), counter, rec)
    return rec


def attention(q, kc, vc, slots, kv_heads, window, scale_log2e, position):
    """q [rows][heads][d] f32; kc, vc [slots][kv_heads][d] uint16 (f16 bits)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    rows, heads, d = q.shape
    kc = np.ascontiguousarray(kc, dtype=np.uint16)
    vc = np.ascontiguousarray(vc, dtype=np.uint16)
    out = np.empty_like(q)
    lib().oracle_attention(q, kc.ctypes.data, vc.ctypes.data, slots, heads, kv_heads, d, window, scale_log2e,
                           position, rows, out)
    return out


def edit_apply(table, layer: int, position: int, activation: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(activation, dtype=np.float32).copy()
    rows, width = a.shape
    t = None if table is None else np.ascontiguousarray(table, dtype=np.uint32)
    lib().oracle_edit_apply(None if t is None else t.ctypes.data, layer, position, rows, width, a)
    return a


# ------------------------------------------------------------ the model

class OracleModel:
    """The whole forward pass over one GGUF file's bytes, one sequence."""

    def __init__(self, gguf_path: str, context: int = 4096, rollback: int = 4096):
        from frizzle_b200 import gguf, synth
        self.data = np.memmap(gguf_path, dtype=np.uint8, mode="r")
        self.index = gguf.read_index(self.data[: 64 << 20])
        self.shape = synth.shape_of(self.index)
        s = self.shape
        self.cshape = Shape(s.layers, s.hidden, s.ffn, s.heads, s.kv_heads, s.head_dim, s.vocab, s.window,
                            s.pattern, s.rope_global, s.rope_local, s.eps, s.context)
        self._keep = []
        ptrs = []
        for l in range(s.layers):
            for role in ROLES:
                ptrs.append(self._ptr(f"blk.{l}.{role}.weight"))
        arr = (C.c_void_p * len(ptrs))(*ptrs)
        self._keep.append(arr)
        self.ctx = lib().oracle_ctx_new(C.byref(self.cshape), self._ptr("token_embd.weight"),
                                        self._ptr("output_norm.weight"), arr, context, rollback)
        self.capture_floats = lib().oracle_capture_floats(C.byref(self.cshape))
        # The tensors' formats (the pinned file's Q8_0 embedding, Q4_1 ffn_down).
        embd = self.index.tensors["token_embd.weight"].ggml_type
        downs = np.array([self.index.tensors[f"blk.{l}.ffn_down.weight"].ggml_type for l in range(s.layers)],
                         dtype=np.int32)
        if embd != 2 or np.any(downs != 2):
            if lib().oracle_ctx_set_types(self.ctx, embd, downs.ctypes.data) != 0:
                raise ValueError("a tensor format the oracle does not restate")

    def tensor(self, name: str) -> np.ndarray:
        a, b = self.index.tensor_range(name)
        return self.data[a:b]

    def _ptr(self, name: str) -> int:
        t = np.ascontiguousarray(self.tensor(name))
        self._keep.append(t)
        return t.ctypes.data

    def step(self, position: int, ids, logits: bool = True, edit_table=None, capture: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.empty(self.shape.vocab, dtype=np.float32) if logits else None
        cap = np.zeros(self.capture_floats, dtype=np.float32) if capture else None
        table = None if edit_table is None else np.ascontiguousarray(edit_table, dtype=np.uint32)
        lib().oracle_step(self.ctx, position, ids.size, ids,
                          None if table is None else table.ctypes.data,
                          None if out is None else out.ctypes.data,
                          None if cap is None else cap.ctypes.data)
        return out, cap

    def slots(self, layer: int) -> int:
        return lib().oracle_ctx_slots(self.ctx, layer)

    def cache(self, layer: int):
        n = self.slots(layer) * self.shape.kv_heads * self.shape.head_dim
        k = np.ctypeslib.as_array(C.cast(lib().oracle_ctx_keys(self.ctx, layer), C.POINTER(C.c_uint16)), (n,))
        v = np.ctypeslib.as_array(C.cast(lib().oracle_ctx_values(self.ctx, layer), C.POINTER(C.c_uint16)), (n,))
        return k.copy(), v.copy()

    def write_cache(self, layer: int, keys: np.ndarray, values: np.ndarray) -> None:
        """Overwrites the layer's key and value rings ([slots][kv_heads][d]
        f16 bits) with the given ones (a test's seeded cache)."""
        n = self.slots(layer) * self.shape.kv_heads * self.shape.head_dim
        for ptr, src in ((lib().oracle_ctx_keys(self.ctx, layer), keys), (lib().oracle_ctx_values(self.ctx, layer),
                                                                           values)):
            dst = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint16)), (n,))
            dst[:] = np.ascontiguousarray(src, dtype=np.uint16).reshape(-1)

    def close(self):
        if self.ctx:
            lib().oracle_ctx_free(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


CAPTURE_SLOTS = ("neurons", "residual", "attention_added", "mlp_added", "query", "weights", "stats", "readout")


def cshape(shape) -> Shape:
    return Shape(shape.layers, shape.hidden, shape.ffn, shape.heads, shape.kv_heads, shape.head_dim, shape.vocab,
                 shape.window, shape.pattern, shape.rope_global, shape.rope_local, shape.eps, shape.context)


def capture_layout(shape):
    """The oracle's capture layout: per layer {slot: first word} and its keys,
    and the store's size in words (capture/capture.cpp:31-73)."""
    cs = cshape(shape)
    layers = []
    for l in range(shape.layers):
        first = (C.c_int64 * 8)()
        keys = C.c_uint32()
        words = lib().oracle_capture_slots(C.byref(cs), l, C.cast(first, C.c_void_p), C.cast(C.byref(keys), C.c_void_p))
        d = dict(zip(CAPTURE_SLOTS, list(first)))
        d["keys"] = keys.value
        layers.append(d)
    return layers, int(words)
