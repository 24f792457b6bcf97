"""GGUF v3 files: a writer for seeded synthetic models and an index reader.

The engine's own loader parses the index natively (``csrc/gguf_index.cpp``);
this module exists so tests and benchmarks can write the files the engine
reads and look inside them from Python.  The format is GGUF v3 as Frizzle's
reader accepts it (``src/core/gguf/reader.h:185``, value types
``src/core/gguf/types.h:136-166``): little-endian, the magic ``GGUF``,
version 3, tensor and metadata counts as u64, metadata key/value pairs, tensor
infos (name, dimension count, dimensions innermost first, ggml type, offset
relative to the aligned data section), then the data section aligned to
``general.alignment`` (32 when absent).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

# Metadata value types.
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i",
           F32: "<f", BOOL: "<?", U64: "<Q", I64: "<q", F64: "<d"}

# Tensor types (ggml numbering) and their block geometry: (elements, bytes).
TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q4_1, TYPE_Q8_0 = 0, 1, 2, 3, 8
BLOCK = {TYPE_F32: (1, 4), TYPE_F16: (1, 2), TYPE_Q4_0: (32, 18),
         TYPE_Q4_1: (32, 20), TYPE_Q8_0: (32, 34)}

DEFAULT_ALIGNMENT = 32


class GgufError(ValueError):
    pass


def tensor_bytes(ggml_type: int, elements: int) -> int:
    per, size = BLOCK[ggml_type]
    if elements % per:
        raise GgufError(f"{elements} elements is not a whole number of blocks")
    return elements // per * size


@dataclass
class TensorInfo:
    name: str
    dims: tuple          # innermost first, as stored
    ggml_type: int
    offset: int          # relative to the data section

    @property
    def elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        return tensor_bytes(self.ggml_type, self.elements)


@dataclass
class GgufIndex:
    version: int
    metadata: dict
    tensors: dict = field(default_factory=dict)  # name -> TensorInfo, file order
    alignment: int = DEFAULT_ALIGNMENT
    data_offset: int = 0                          # absolute start of the data section

    def tensor_range(self, name: str) -> tuple:
        t = self.tensors[name]
        start = self.data_offset + t.offset
        return start, start + t.nbytes


# ---------------------------------------------------------------- writing

def _pack_string(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _pack_value(vtype: int, value) -> bytes:
    if vtype == STRING:
        return _pack_string(value)
    if vtype == ARRAY:
        etype, items = value
        head = struct.pack("<IQ", etype, len(items))
        if etype == STRING:
            return head + b"".join(_pack_string(s) for s in items)
        return head + np.asarray(items, dtype=np.dtype(_SCALAR[etype])).tobytes()
    return struct.pack(_SCALAR[vtype], value)


class GgufWriter:
    """Streams a GGUF v3 file: metadata and tensor infos first, then data.

    Tensors are declared with their byte size up front (``add_tensor``), then
    their bytes written in the same order (``write_tensor_data``), so a model
    of several hundred MB never has to be held whole in memory.
    """

    def __init__(self, path: str, alignment: int = DEFAULT_ALIGNMENT):
        self.path = path
        self.alignment = alignment
        self.kv = []         # (key, vtype, value)
        self.infos = []      # TensorInfo
        self._next = 0
        self._written = 0
        self._fh = None

    def add(self, key: str, vtype: int, value) -> None:
        self.kv.append((key, vtype, value))

    def add_tensor(self, name: str, dims: tuple, ggml_type: int) -> TensorInfo:
        info = TensorInfo(name, tuple(int(d) for d in dims), ggml_type, self._next)
        self.infos.append(info)
        self._next += -(-info.nbytes // self.alignment) * self.alignment
        return info

    def _header(self) -> bytes:
        kv = list(self.kv)
        if self.alignment != DEFAULT_ALIGNMENT and not any(k == "general.alignment" for k, _, _ in kv):
            kv.insert(0, ("general.alignment", U32, self.alignment))
        out = [b"GGUF", struct.pack("<IQQ", 3, len(self.infos), len(kv))]
        for key, vtype, value in kv:
            out += [_pack_string(key), struct.pack("<I", vtype), _pack_value(vtype, value)]
        for t in self.infos:
            out += [_pack_string(t.name), struct.pack("<I", len(t.dims)),
                    struct.pack(f"<{len(t.dims)}Q", *t.dims),
                    struct.pack("<IQ", t.ggml_type, t.offset)]
        head = b"".join(out)
        pad = -len(head) % self.alignment
        return head + b"\0" * pad

    def begin_data(self) -> None:
        self._fh = open(self.path, "wb")
        self._fh.write(self._header())

    def write_tensor_data(self, data: bytes | np.ndarray) -> None:
        info = self.infos[self._written]
        raw = data.tobytes() if isinstance(data, np.ndarray) else bytes(data)
        if len(raw) != info.nbytes:
            raise GgufError(f"{info.name}: {len(raw)} bytes for {info.nbytes}")
        self._fh.write(raw)
        self._fh.write(b"\0" * (-len(raw) % self.alignment))
        self._written += 1

    def close(self) -> None:
        if self._written != len(self.infos):
            raise GgufError(f"{len(self.infos) - self._written} tensors left unwritten")
        self._fh.close()


# ---------------------------------------------------------------- reading

class _Reader:
    def __init__(self, buf):
        self.buf = memoryview(buf)
        self.at = 0

    def take(self, n: int) -> memoryview:
        if self.at + n > len(self.buf):
            raise GgufError("truncated index")
        v = self.buf[self.at:self.at + n]
        self.at += n
        return v

    def scalar(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.scalar("<Q")
        return bytes(self.take(n)).decode("utf-8")

    def value(self, vtype: int, depth: int = 0):
        if vtype == STRING:
            return self.string()
        if vtype == ARRAY:
            if depth:
                raise GgufError("nested array")
            etype = self.scalar("<I")
            count = self.scalar("<Q")
            if etype == STRING:
                return [self.string() for _ in range(count)]
            if etype not in _SCALAR:
                raise GgufError(f"array of unknown type {etype}")
            dt = np.dtype(_SCALAR[etype])
            return np.frombuffer(self.take(count * dt.itemsize), dtype=dt).copy()
        if vtype not in _SCALAR:
            raise GgufError(f"unknown value type {vtype}")
        return self.scalar(_SCALAR[vtype])


def read_index(buf) -> GgufIndex:
    """Parses the header, metadata and tensor infos of a GGUF v3 buffer."""
    r = _Reader(buf)
    if bytes(r.take(4)) != b"GGUF":
        raise GgufError("bad magic")
    version = r.scalar("<I")
    if version != 3:
        raise GgufError(f"version {version}")
    n_tensors = r.scalar("<Q")
    n_kv = r.scalar("<Q")
    meta = {}
    for _ in range(n_kv):
        key = r.string()
        vtype = r.scalar("<I")
        if key in meta:
            raise GgufError(f"duplicate key {key}")
        meta[key] = r.value(vtype)
    align = int(meta.get("general.alignment", DEFAULT_ALIGNMENT))
    if align <= 0 or align & (align - 1):
        raise GgufError("alignment not a power of two")
    idx = GgufIndex(version, meta, alignment=align)
    for _ in range(n_tensors):
        name = r.string()
        nd = r.scalar("<I")
        dims = struct.unpack(f"<{nd}Q", r.take(8 * nd))
        ttype = r.scalar("<I")
        off = r.scalar("<Q")
        if name in idx.tensors:
            raise GgufError(f"duplicate tensor {name}")
        idx.tensors[name] = TensorInfo(name, dims, ttype, off)
    idx.data_offset = -(-r.at // align) * align
    return idx
