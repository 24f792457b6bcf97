"""The C ABI without a GPU: the library loads, exports every symbol the header
declares, refuses to open a device cleanly, and parses/describes GGUF indexes
(LoadError::Index / ::Architecture behaviour of src/core/runtime/engine.h)."""
import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

from frizzle_b200 import _native, gguf, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "frizzle_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fz_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    names = declared_symbols()
    assert len(names) >= 25
    for name in names:
        assert hasattr(lib, name), name
        assert name in _native.SIGNATURES, f"{name} has no binding"


def test_struct_sizes_match_header():
    assert C.sizeof(_native.Step) == 64
    assert C.sizeof(_native.Record) == 16


def test_layout_sizes():
    lib = _native.load()
    assert lib.fz_q4_0_codes_bytes(1536, 1152) == 1536 * 1152 // 2
    assert lib.fz_q4_0_scales_bytes(1536, 1152) == 1536 * 1152 // 16


def test_device_open_fails_loudly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _native.load()
    h = C.c_void_p()
    st = lib.fz_device_open(0, C.byref(h))
    assert st != 0
    assert lib.fz_last_error()


def _index_check(head: bytes, size: int):
    lib = _native.load()
    info = _native.ModelInfo()
    buf = C.create_string_buffer(head, len(head))
    st = lib.fz_model_index_check(buf, len(head), size, C.byref(info))
    return st, lib.fz_last_error().decode(), info


def test_index_check_describes_tiny_model(tiny_model_path):
    size = os.path.getsize(tiny_model_path)
    head = open(tiny_model_path, "rb").read(1 << 20)
    st, msg, info = _index_check(head, size)
    assert st == 0, msg
    s = synth.TINY
    assert (info.layers, info.hidden, info.ffn, info.heads, info.kv_heads, info.head_dim, info.vocab) == \
        (s.layers, s.hidden, s.ffn, s.heads, s.kv_heads, s.head_dim, s.vocab)
    assert info.window == s.window and info.context == s.context


def test_index_check_truncated_asks_for_more(tiny_model_path):
    size = os.path.getsize(tiny_model_path)
    head = open(tiny_model_path, "rb").read(100)
    st, _, _ = _index_check(head, size)
    assert st == 9
    assert _native.load().fz_model_index_needed() > 100


def _write(tmp_path, mutate=None, arch="gemma3", tensors=None, align=32):
    w = gguf.GgufWriter(str(tmp_path / "m.gguf"), alignment=align)
    w.add("general.architecture", gguf.STRING, arch)
    for k, v in [("block_count", 1), ("context_length", 64), ("embedding_length", 64), ("feed_forward_length", 128),
                 ("attention.head_count", 1), ("attention.head_count_kv", 1), ("attention.key_length", 256)]:
        w.add("gemma3." + k, gguf.U32, v)
    w.add("gemma3.attention.layer_norm_rms_epsilon", gguf.F32, 1e-6)
    w.add("gemma3.rope.freq_base", gguf.F32, 1e6)
    if mutate:
        mutate(w)
    for name, dims, t in tensors or [("token_embd.weight", (64, 32), gguf.TYPE_Q4_0)]:
        w.add_tensor(name, dims, t)
    w.begin_data()
    for info in w.infos:
        w.write_tensor_data(b"\0" * info.nbytes)
    w.close()
    data = open(str(tmp_path / "m.gguf"), "rb").read()
    return data


def test_index_refusals(tmp_path):
    data = _write(tmp_path)
    # A well formed index of a file missing its layers: refused as Architecture.
    st, msg, _ = _index_check(data, len(data))
    assert st == 4, msg
    assert _index_check(b"GGUX" + data[4:], len(data))[0] == 3            # bad magic
    assert _index_check(data[:4] + struct.pack("<I", 2) + data[8:], len(data))[0] == 3  # version 2
    st, msg, _ = _index_check(_write(tmp_path, arch="llama"), len(data))
    assert st == 4 and "gemma3" in msg
    st, msg, _ = _index_check(data, 64)                                    # data past the end of the file
    assert st == 3


def test_index_refuses_duplicates_and_bad_alignment(tmp_path):
    dup = _write(tmp_path, tensors=[("a", (32,), gguf.TYPE_F32), ("a", (32,), gguf.TYPE_F32)])
    assert _index_check(dup, len(dup))[0] == 3
    def bad_align(w):
        w.add("general.alignment", gguf.U32, 24)
    bad = _write(tmp_path, mutate=bad_align)
    assert _index_check(bad, len(bad))[0] == 3


def test_index_refuses_offset_that_wraps(tmp_path):
    # Tensor b's offset rewritten to 2^64 - 64: offset + 128 bytes wraps to 64, which would pass the
    # data-in-file and overlap checks if the parser let it through.  Refused as an index error.
    data = _write(tmp_path, tensors=[("a", (32,), gguf.TYPE_F32), ("b", (32,), gguf.TYPE_F32)])
    info_b = gguf._pack_string("b") + struct.pack("<IQ", 1, 32)
    at = data.index(info_b + struct.pack("<IQ", gguf.TYPE_F32, 128))
    field = at + len(info_b) + 4
    bad = data[:field] + struct.pack("<Q", (1 << 64) - 64) + data[field + 8:]
    st, msg, _ = _index_check(bad, len(bad))
    assert st == 3 and "out of range" in msg, msg
    # The same file untouched is well formed (refused only for missing layers).
    assert _index_check(data, len(data))[0] == 4


def test_index_refuses_softcapping(tmp_path):
    def cap(w):
        w.add("gemma3.final_logit_softcapping", gguf.F32, 30.0)
    data = _write(tmp_path, mutate=cap)
    st, msg, _ = _index_check(data, len(data))
    assert st == 4 and "softcapping" in msg


def test_gguf_reader_round_trip(tiny_model_path):
    idx = gguf.read_index(open(tiny_model_path, "rb").read(1 << 22))
    assert idx.metadata["general.architecture"] == "gemma3"
    assert len(idx.metadata["tokenizer.ggml.tokens"]) == synth.TINY.vocab
    t = idx.tensors["blk.0.ffn_gate.weight"]
    assert t.dims == (synth.TINY.hidden, synth.TINY.ffn) and t.ggml_type == gguf.TYPE_Q4_0
    assert t.offset % 32 == 0


def test_attention_wide_refuses_bad_arguments_before_any_launch():
    """fz_attention_wide checks its arguments on the host, before it encodes
    tensor maps or launches anything, so these refusals need no GPU: null
    pointers, maps not 64-byte aligned, caches not 16-byte aligned, a head
    group other than 1, 2, 4 or 8, a slot count that is not whole 32-key
    tiles, zero rows, and split scratch without its counters."""
    lib = _native.load()
    P = 0x10000          # a 64-byte-aligned stand-in address; nothing is dereferenced
    ok = dict(q=P, k=P, v=P, slots=2048, heads=4, kv=1, d=256, window=32768, position=0, rows=64,
              maps=P, split=None, counters=None, out=P)

    def call(**kw):
        c = dict(ok, **kw)
        return lib.fz_attention_wide(c["q"], c["k"], c["v"], c["slots"], c["heads"], c["kv"], c["d"], c["window"],
                                     c["position"], c["rows"], c["maps"], c["split"], c["counters"], c["out"],
                                     None, None)

    for bad in (dict(q=None), dict(out=None), dict(maps=None), dict(maps=P + 32), dict(k=P + 8),
                dict(heads=3), dict(d=128), dict(slots=1000), dict(rows=0), dict(split=P),
                dict(position=(1 << 24) - 10, rows=64)):
        st = call(**bad)
        assert st == 1, (bad, st)   # FZ_ERR_ARGUMENT
        assert lib.fz_last_error(), bad
