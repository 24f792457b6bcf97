"""Seeded synthetic Gemma-3-shaped models in GGUF Q4_0, and random Q4_0 matrices.

The benchmark configurations use random-init weights (there is no network for
the pinned checkpoint).  A model is a GGUF v3 file with the tensor names,
hyperparameter keys and tied embedding that Frizzle's Gemma 3 description
reads (``src/core/arch/gemma3/gemma3.cpp:21-35``, ``src/core/arch/describe.cpp:205-320``):

- every linear weight and the tied ``token_embd`` drawn N(0, 0.02) and
  quantised to Q4_0;
- every norm gain stored as ``1 + N(0, 0.1)`` in F32, since the engine
  multiplies by the stored gain and the file convention is ``1 + w``;
- a synthetic vocabulary of ``t<i>`` strings (bos 2, eos 106).

Each tensor (and each 4 Mi-element slice of a large one) draws from its own
``numpy.random.default_rng([seed, tensor, slice])`` stream, so generation is
parallel and any tensor can be regenerated alone.
"""
from __future__ import annotations

import os
import tempfile
from concurrent.futures import ThreadPoolExecutor
from dataclasses import asdict, dataclass, replace

import numpy as np

from . import gguf


@dataclass(frozen=True)
class ModelShape:
    layers: int
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    window: int = 512
    pattern: int = 6          # every pattern-th layer attends globally
    rope_global: float = 1e6
    rope_local: float = 1e4
    eps: float = 1e-6
    context: int = 32768
    # "q4_0": every linear and the tied embedding Q4_0.  "pinned": the
    # pinned file's mix (docs/architecture/logical-overview.md:63-64): the
    # tied embedding Q8_0, ffn_down Q4_1 in the first three layers, the
    # rest Q4_0.
    mix: str = "q4_0"

    def is_global(self, layer: int) -> bool:
        return layer % self.pattern == self.pattern - 1

    def layer_window(self, layer: int) -> int:
        return self.context if self.is_global(layer) else self.window

    @property
    def q_width(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim

    def tag(self) -> str:
        vals = asdict(self)
        if vals["mix"] == "q4_0":
            del vals["mix"]   # (the Q4_0 files keep their names)
        return "_".join(str(v).replace(".", "p") for v in vals.values())


GEMMA3_1B = ModelShape(layers=26, hidden=1152, ffn=6912, heads=4, kv_heads=1,
                       head_dim=256, vocab=262144)
# Small enough for the CPU oracle in milliseconds, shaped like Gemma 3 1B where
# the kernels care: d = 256, 4:1 grouped queries, one global layer (5) among
# window layers, K a multiple of 64 for every product.
TINY = ModelShape(layers=7, hidden=512, ffn=1024, heads=4, kv_heads=1,
                  head_dim=256, vocab=4096, window=16, context=4096)
# The same shapes with the pinned file's format mix.
GEMMA3_1B_PINNED = replace(GEMMA3_1B, mix="pinned")
TINY_PINNED = replace(TINY, mix="pinned")

SLICE = 1 << 22


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """Q4_0 blocks (fp16 scale d, then 16 code bytes) of a float32 array.

    Per block of 32 the scale is chosen so the value of largest magnitude, m,
    lands on code 0: d = m / -8; each value's code is round-half-up of
    x / d + 8, clamped to 15; a block of zeros has d = 0 and codes 8.  Byte j
    of the codes holds code j in its low nibble and code j + 16 in its high
    nibble (``src/core/formats/q4_0/q4_0.h:21-23``).
    """
    b = x.reshape(-1, 32).astype(np.float32, copy=False)
    i = np.abs(b).argmax(axis=1)
    m = np.take_along_axis(b, i[:, None], 1)[:, 0]
    d = m / np.float32(-8.0)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.minimum(15, np.floor(b * inv[:, None] + np.float32(8.5))).astype(np.uint8)
    out = np.empty((b.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Q8_0 blocks (fp16 scale d, then 32 signed codes) of a float32 array:
    per block of 32, d = (largest magnitude) / 127 and each code is x / d
    rounded half away from zero; a block of zeros has d = 0, codes 0.  Weight
    j is code j x d (``src/core/formats/q8_0/q8_0.h:19-21``)."""
    b = x.reshape(-1, 32).astype(np.float32, copy=False)
    d = np.abs(b).max(axis=1) / np.float32(127.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d[:, None] != 0, np.round(b / d[:, None]), 0)
    q = np.clip(q, -127, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize_q4_1(x: np.ndarray) -> np.ndarray:
    """Q4_1 blocks (fp16 scale d, fp16 minimum m, then 16 code bytes) of a
    float32 array: per block of 32, m = the smallest value, d = (largest -
    m) / 15, each code (x - m) / d rounded to nearest and clamped to [0, 15];
    byte j holds code j low and code j + 16 high.  Weight j is code j x d + m
    (``src/core/formats/q4_1/q4_1.h:20-23``)."""
    b = x.reshape(-1, 32).astype(np.float32, copy=False)
    lo, hi = b.min(axis=1), b.max(axis=1)
    d = (hi - lo) / np.float32(15.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d[:, None] != 0, np.round((b - lo[:, None]) / d[:, None]), 0)
    q = np.clip(q, 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], 20), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = lo.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 4:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def dequantize_q4_0(blocks: np.ndarray) -> np.ndarray:
    """The weights a Q4_0 byte array holds: (code - 8) x d, exact in f32."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 18)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    qs = b[:, 2:]
    codes = np.concatenate([qs & 0xF, qs >> 4], axis=1).astype(np.float32)
    return ((codes - 8.0) * d[:, None]).reshape(-1).astype(np.float32)


def random_q4_0(rows: int, k: int, seed: int, scale_sigma: float = 0.005) -> np.ndarray:
    """Q4_0 blocks with codes uniform in [0, 15] and fp16 scales |N(0, sigma)|."""
    rng = np.random.default_rng([seed, rows, k])
    n = rows * k // 32
    out = np.empty((n, 18), dtype=np.uint8)
    d = np.abs(rng.standard_normal(n, dtype=np.float32) * np.float32(scale_sigma))
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = rng.integers(0, 256, size=(n, 16), dtype=np.uint8)
    return out.reshape(-1)


def random_q8_0(rows: int, k: int, seed: int, scale_sigma: float = 0.0005) -> np.ndarray:
    """Q8_0 blocks (fp16 d, 32 signed codes) with codes uniform in [-128, 127]
    and fp16 scales |N(0, sigma)|: weights of Q4_0's magnitude at 16x the
    resolution."""
    rng = np.random.default_rng([seed, rows, k, 8])
    n = rows * k // 32
    out = np.empty((n, 34), dtype=np.uint8)
    d = np.abs(rng.standard_normal(n, dtype=np.float32) * np.float32(scale_sigma))
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = rng.integers(0, 256, size=(n, 32), dtype=np.uint8)
    return out.reshape(-1)


def random_q4_1(rows: int, k: int, seed: int, scale_sigma: float = 0.005) -> np.ndarray:
    """Q4_1 blocks (fp16 d, fp16 m, 16 code bytes) with codes uniform in
    [0, 15], d = |N(0, sigma)| and m = -8 d + N(0, sigma): a block's minimum
    near its centred range, as a quantiser sets it."""
    rng = np.random.default_rng([seed, rows, k, 3])
    n = rows * k // 32
    out = np.empty((n, 20), dtype=np.uint8)
    d = np.abs(rng.standard_normal(n, dtype=np.float32) * np.float32(scale_sigma))
    m = -8.0 * d + rng.standard_normal(n, dtype=np.float32) * np.float32(scale_sigma)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = m.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 4:] = rng.integers(0, 256, size=(n, 16), dtype=np.uint8)
    return out.reshape(-1)


def tensor_plan(shape: ModelShape):
    """(name, dims innermost first, ggml type, kind) in file order."""
    H, F, Q, KV, D = shape.hidden, shape.ffn, shape.q_width, shape.kv_width, shape.head_dim
    pinned = shape.mix == "pinned"
    embd = (gguf.TYPE_Q8_0, "q8_0") if pinned else (gguf.TYPE_Q4_0, "linear")
    plan = [("token_embd.weight", (H, shape.vocab), embd[0], embd[1])]
    for l in range(shape.layers):
        p = f"blk.{l}."
        down = (gguf.TYPE_Q4_1, "q4_1") if pinned and l < 3 else (gguf.TYPE_Q4_0, "linear")
        plan += [
            (p + "attn_norm.weight", (H,), gguf.TYPE_F32, "norm"),
            (p + "attn_q.weight", (H, Q), gguf.TYPE_Q4_0, "linear"),
            (p + "attn_k.weight", (H, KV), gguf.TYPE_Q4_0, "linear"),
            (p + "attn_v.weight", (H, KV), gguf.TYPE_Q4_0, "linear"),
            (p + "attn_q_norm.weight", (D,), gguf.TYPE_F32, "norm"),
            (p + "attn_k_norm.weight", (D,), gguf.TYPE_F32, "norm"),
            (p + "attn_output.weight", (Q, H), gguf.TYPE_Q4_0, "linear"),
            (p + "post_attention_norm.weight", (H,), gguf.TYPE_F32, "norm"),
            (p + "ffn_norm.weight", (H,), gguf.TYPE_F32, "norm"),
            (p + "ffn_gate.weight", (H, F), gguf.TYPE_Q4_0, "linear"),
            (p + "ffn_up.weight", (H, F), gguf.TYPE_Q4_0, "linear"),
            (p + "ffn_down.weight", (F, H), down[0], down[1]),
            (p + "post_ffw_norm.weight", (H,), gguf.TYPE_F32, "norm"),
        ]
    plan.append(("output_norm.weight", (H,), gguf.TYPE_F32, "norm"))
    return plan


def _slice_job(args):
    seed, index, part, count, kind = args
    rng = np.random.default_rng([seed, index, part])
    if kind == "norm":
        return (np.float32(1.0) + rng.standard_normal(count, dtype=np.float32) * np.float32(0.1)).tobytes()
    x = rng.standard_normal(count, dtype=np.float32) * np.float32(0.02)
    if kind == "q8_0":
        return quantize_q8_0(x).tobytes()
    if kind == "q4_1":
        return quantize_q4_1(x).tobytes()
    return quantize_q4_0(x).tobytes()


def model_header(shape: ModelShape = GEMMA3_1B, seed: int = 0) -> tuple:
    """The GGUF head ``write_model`` writes for (shape, seed) -- metadata and
    tensor infos, padded to the data section -- and the whole file's size,
    without generating the tensor data."""
    w = _writer(None, shape, seed)
    for name, dims, ttype, _ in tensor_plan(shape):
        w.add_tensor(name, dims, ttype)
    head = w._header()
    return head, len(head) + w._next


def _writer(path, shape: ModelShape, seed: int):
    w = gguf.GgufWriter(path)
    a = "gemma3."
    w.add("general.architecture", gguf.STRING, "gemma3")
    w.add("general.name", gguf.STRING, f"synthetic-gemma3-seed{seed}")
    w.add(a + "block_count", gguf.U32, shape.layers)
    w.add(a + "context_length", gguf.U32, shape.context)
    w.add(a + "embedding_length", gguf.U32, shape.hidden)
    w.add(a + "feed_forward_length", gguf.U32, shape.ffn)
    w.add(a + "attention.head_count", gguf.U32, shape.heads)
    w.add(a + "attention.head_count_kv", gguf.U32, shape.kv_heads)
    w.add(a + "attention.key_length", gguf.U32, shape.head_dim)
    w.add(a + "attention.value_length", gguf.U32, shape.head_dim)
    w.add(a + "attention.layer_norm_rms_epsilon", gguf.F32, shape.eps)
    w.add(a + "rope.freq_base", gguf.F32, shape.rope_global)
    w.add(a + "rope.freq_base_swa", gguf.F32, shape.rope_local)
    w.add(a + "attention.sliding_window", gguf.U32, shape.window)
    w.add(a + "attention.sliding_window_pattern", gguf.U32, shape.pattern)
    w.add("tokenizer.ggml.model", gguf.STRING, "llama")
    w.add("tokenizer.ggml.tokens", gguf.ARRAY, (gguf.STRING, [f"t{i}" for i in range(shape.vocab)]))
    w.add("tokenizer.ggml.bos_token_id", gguf.U32, 2)
    w.add("tokenizer.ggml.eos_token_id", gguf.U32, 106)
    return w


def write_model(path: str, shape: ModelShape = GEMMA3_1B, seed: int = 0, threads: int | None = None) -> None:
    w = _writer(path, shape, seed)
    plan = tensor_plan(shape)
    jobs = []
    for index, (name, dims, ttype, kind) in enumerate(plan):
        w.add_tensor(name, dims, ttype)
        n = int(np.prod(dims))
        parts = [(seed, index, p, min(SLICE, n - p * SLICE), kind) for p in range(-(-n // SLICE))]
        jobs.append(parts)
    w.begin_data()
    with ThreadPoolExecutor(threads or os.cpu_count() or 4) as ex:
        for parts in jobs:
            w.write_tensor_data(b"".join(ex.map(_slice_job, parts)))
    w.close()


def cache_dir() -> str:
    d = os.environ.get("FRIZZLE_B200_CACHE") or os.path.join(tempfile.gettempdir(), "frizzle_b200_cache")
    os.makedirs(d, exist_ok=True)
    return d


def model_path(shape: ModelShape = GEMMA3_1B, seed: int = 0) -> str:
    """The cached synthetic model for (shape, seed), written on first use."""
    path = os.path.join(cache_dir(), f"gemma3_{shape.tag()}_seed{seed}.gguf")
    if not os.path.exists(path):
        tmp = f"{path}.{os.getpid()}.tmp"
        write_model(tmp, shape, seed)
        os.replace(tmp, path)
    return path


def shape_of(index: gguf.GgufIndex) -> ModelShape:
    """The shape a GGUF index declares (the keys ``write_model`` writes)."""
    m = index.metadata
    a = "gemma3."
    return ModelShape(
        layers=int(m[a + "block_count"]), hidden=int(m[a + "embedding_length"]),
        ffn=int(m[a + "feed_forward_length"]), heads=int(m[a + "attention.head_count"]),
        kv_heads=int(m[a + "attention.head_count_kv"]), head_dim=int(m[a + "attention.key_length"]),
        vocab=len(m["tokenizer.ggml.tokens"]), window=int(m.get(a + "attention.sliding_window", 0)),
        pattern=int(m.get(a + "attention.sliding_window_pattern", 6)),
        rope_global=float(m[a + "rope.freq_base"]), rope_local=float(m.get(a + "rope.freq_base_swa", 1e4)),
        eps=float(m[a + "attention.layer_norm_rms_epsilon"]), context=int(m[a + "context_length"]))
