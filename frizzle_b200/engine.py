"""The engine API over the C ABI, in the shape of Frizzle's C++ engine.

``Device``, ``Model`` (``begin_load``/``write``/``finish_load`` as
``Engine::begin_load/write/finish_load``, src/core/runtime/engine.h:366-412),
``Batch`` (sequences stepped together: ``Program::run`` per step,
src/core/kernels/program.h:380-388) and ``generate`` (the turn loop of
``Runtime::run_planned``/``Turn::next``, src/core/runtime/runtime.cpp:89-114,
turn.cpp:22-39: prefill blocks, the last asking for logits, then fed
one-token decode steps).  Token identifiers go in directly: the tokenizer is
outside this path.
"""
from __future__ import annotations

import ctypes as C
import math
import os
from dataclasses import dataclass, field

import numpy as np

from . import edits as E
from . import prefix as P
from ._native import CaptureSlots, FzError, ModelInfo, Record, Step, check, load
from .capture import SLOTS, Capture
from .capture import layout as capture_layout

MAX_ROWS = 16  # sequences x tokens the skinny (matvec) path takes in one step
PREFILL_BLOCK = 512  # prompt tokens a step (residency::kPrefillBlock, src/core/residency/plan.h:175)


class Device:
    def __init__(self, ordinal: int = 0):
        self.lib = load()
        h = C.c_void_p()
        check(self.lib.fz_device_open(ordinal, C.byref(h)))
        self.handle = h
        self.ordinal = ordinal

    @property
    def stream(self) -> int:
        return self.lib.fz_device_stream(self.handle) or 0

    def close(self):
        if self.handle:
            self.lib.fz_device_close(self.handle)
            self.handle = None


class Model:
    """A model loaded from GGUF bytes, in chunks (Upload::begin/write/finish)."""

    def __init__(self, device: Device):
        self.device = device
        self.lib = device.lib
        self.handle = None
        self.info = None

    def begin_load(self, head: bytes, file_bytes: int) -> None:
        h = C.c_void_p()
        buf = C.create_string_buffer(bytes(head), len(head))
        check(self.lib.fz_model_load_begin(self.device.handle, buf, len(head), file_bytes, C.byref(h)))
        self.handle = h

    def write(self, offset: int, chunk) -> None:
        mv = memoryview(chunk)
        arr = (C.c_char * mv.nbytes).from_buffer_copy(mv) if mv.readonly else (C.c_char * mv.nbytes).from_buffer(mv)
        check(self.lib.fz_model_load_write(self.handle, offset, arr, mv.nbytes))

    def finish_load(self) -> None:
        check(self.lib.fz_model_load_finish(self.handle))
        info = ModelInfo()
        check(self.lib.fz_model_info_get(self.handle, C.byref(info)))
        self.info = info

    @classmethod
    def from_file(cls, device: Device, path: str, chunk: int = 64 << 20) -> "Model":
        m = cls(device)
        size = os.path.getsize(path)
        with open(path, "rb") as f:
            head = f.read(min(size, 1 << 20))
            while True:
                try:
                    m.begin_load(head, size)
                    break
                except FzError as e:
                    if e.status != 9:  # TRUNCATED: read as much as the index asks for
                        raise
                    need = max(int(m.lib.fz_model_index_needed()), 2 * len(head))
                    f.seek(0)
                    head = f.read(min(size, need))
            data = np.memmap(path, dtype=np.uint8, mode="r")
            for off in range(0, size, chunk):
                part = np.ascontiguousarray(data[off:off + chunk])
                check(m.lib.fz_model_load_write(m.handle, off, part.ctypes.data, part.size))
            del data
        m.finish_load()
        return m

    @property
    def capture_floats(self) -> int:
        return int(self.lib.fz_capture_floats(self.handle))

    def capture_layout(self, layer: int) -> dict:
        """fz_capture_layout: the layer's slots as {name: (first, width)} and its attention."""
        out = CaptureSlots()
        check(self.lib.fz_capture_layout(self.handle, layer, C.byref(out)))
        d = {n: (getattr(out, n).first, getattr(out, n).width) for n in SLOTS}
        d.update(keys=out.keys, query_heads=out.query_heads, window=out.window,
                 full_attention=bool(out.full_attention))
        return d

    def free(self):
        if self.handle:
            self.lib.fz_model_free(self.handle)
            self.handle = None


@dataclass
class Sampling:
    """policy::SamplingSettings as the draw reads them; temperature 0 is greedy."""
    temperature: float = 0.0
    top_k: int = 64
    top_p: float = 1.0
    min_p: float = 0.0
    seed: tuple = (0, 0)


class Batch:
    """Sequences stepped together, each with its own KV cache, edits and seed."""

    def __init__(self, model: Model, sequences: int = 1, context: int = 4096, rollback: int = 4096):
        self.model = model
        self.lib = model.lib
        self.sequences = sequences
        h = C.c_void_p()
        check(self.lib.fz_batch_create(model.handle, sequences, context, rollback, C.byref(h)))
        self.handle = h
        self.context = context

    def set_edits(self, sequence: int, words) -> None:
        if words is None or len(words) == 0:
            check(self.lib.fz_batch_set_edits(self.handle, sequence, None, 0))
            return
        arr = np.ascontiguousarray(words, dtype=np.uint32)
        check(self.lib.fz_batch_set_edits(self.handle, sequence, arr.ctypes.data, arr.size))

    def step(self, position: int, ids=None, tokens: int = 1, logits: bool = True, fed: bool = False,
             sampling: Sampling = Sampling(), seeds=None, capture: bool = False) -> None:
        st = Step()
        st.position = position
        st.tokens = tokens
        st.logits = 1 if logits else 0
        st.fed = 1 if fed else 0
        st.seed[0], st.seed[1] = sampling.seed
        st.top_k = sampling.top_k
        st.temperature = sampling.temperature
        st.top_p = sampling.top_p
        st.min_p = sampling.min_p
        st.log_min_p = math.log(sampling.min_p) if sampling.min_p > 0 else 0.0
        st.capture = 1 if capture else 0
        idp = None
        if not fed:
            ids = np.ascontiguousarray(ids, dtype=np.uint32).reshape(-1)
            if ids.size != tokens * self.sequences:
                raise ValueError("ids must hold sequences x tokens identifiers")
            idp = ids.ctypes.data
            self._ids = ids
        sp = None
        if seeds is not None:
            self._seeds = np.ascontiguousarray(seeds, dtype=np.uint32).reshape(-1)
            sp = self._seeds.ctypes.data
        check(self.lib.fz_batch_step(self.handle, C.byref(st), idp, sp))

    def wait(self) -> np.ndarray:
        recs = (Record * self.sequences)()
        check(self.lib.fz_batch_wait(self.handle, recs))
        return np.array([(r.token, r.failed, r.u) for r in recs], dtype=object)

    def wait_oldest(self) -> np.ndarray:
        """The records of the oldest step not yet reported (two steps may be in
        flight; steps report in the order they ran)."""
        recs = (Record * self.sequences)()
        check(self.lib.fz_batch_wait_oldest(self.handle, recs))
        return np.array([(r.token, r.failed, r.u) for r in recs], dtype=object)

    def tokens(self) -> list:
        recs = (Record * self.sequences)()
        check(self.lib.fz_batch_wait(self.handle, recs))
        return [int(r.token) for r in recs]

    def logits(self, sequence: int = 0) -> np.ndarray:
        v = self.model.info.vocab
        out = np.empty(v, dtype=np.float32)
        check(self.lib.fz_batch_read_logits(self.handle, sequence, out.ctypes.data, v))
        return out

    def capture(self, sequence: int = 0) -> np.ndarray:
        n = self.model.capture_floats
        out = np.empty(n, dtype=np.float32)
        check(self.lib.fz_batch_read_capture(self.handle, sequence, out.ctypes.data, n))
        return out

    def capture_view(self, sequence: int = 0) -> Capture:
        """The sequence's capture store read through its layout."""
        info = self.model.info
        return Capture(self.capture(sequence), capture_layout(info), info.head_dim)

    def truncate(self, tokens: int) -> int:
        """KvCache::truncate (clamped to the length): the tokens kept."""
        kept = C.c_uint32()
        check(self.lib.fz_batch_truncate(self.handle, tokens, C.byref(kept)))
        return kept.value

    def cache_state(self):
        """(tokens held, high-water mark) of the batch's KV cache."""
        length, written = C.c_uint32(), C.c_uint32()
        check(self.lib.fz_batch_cache_state(self.handle, C.byref(length), C.byref(written)))
        return length.value, written.value

    def cache(self, sequence: int, layer: int, values: bool = False):
        p = C.c_void_p()
        slots = C.c_uint32()
        check(self.lib.fz_batch_cache(self.handle, sequence, layer, 1 if values else 0, C.byref(p), C.byref(slots)))
        return p.value, slots.value

    def free(self):
        if self.handle:
            self.lib.fz_batch_free(self.handle)
            self.handle = None


@dataclass
class Turn:
    tokens: list = field(default_factory=list)      # per sequence, the reply's tokens
    records: list = field(default_factory=list)
    logits: list = field(default_factory=list)      # per step, per sequence (when kept)


def generate(batch: Batch, prompts, steps: int, sampling: Sampling = Sampling(), edit_sets=None,
             seeds=None, keep_logits: bool = False, capture: bool = False, start: int = 0) -> Turn:
    """Prefill every sequence's prompt (same length) then `steps` fed decode steps.

    ``edit_sets[s]`` is sequence s's list of ``edits.Edit`` with ranges in steps
    from the prompt's last position (origin = prompt length - 1, as
    Engine::generate places them).  The prefill starts at `start`: the
    tokens before it are the ones the cache already holds (``Session``).
    Returns each sequence's drawn tokens.
    """
    S = batch.sequences
    prompts = [list(p) for p in prompts]
    if len(prompts) != S or len({len(p) for p in prompts}) != 1:
        raise ValueError("one prompt a sequence, all the same length")
    n = len(prompts[0])
    origin = n - 1
    layers = batch.model.info.layers
    for s in range(S):
        es = (edit_sets or [None] * S)[s]
        if es:
            chk = E.check(es, layers, batch.model.info.ffn)
            if not chk.ok:
                raise FzError(8, chk.subject)
            batch.set_edits(s, E.table(es, layers, origin))
        else:
            batch.set_edits(s, None)
    block = max(1, PREFILL_BLOCK // S)
    turn = Turn(tokens=[[] for _ in range(S)])
    if not 0 <= start < n:
        raise ValueError("the prefill must start inside the prompt")
    pos = start
    while pos < n:
        t = min(block, n - pos)
        last = pos + t == n
        ids = np.array([p[pos:pos + t] for p in prompts], dtype=np.uint32)
        batch.step(pos, ids, tokens=t, logits=last, sampling=sampling, seeds=seeds, capture=capture and last)
        pos += t
    for i in range(steps):
        rec = batch.tokens()
        for s in range(S):
            turn.tokens[s].append(rec[s])
        if keep_logits:
            turn.logits.append([batch.logits(s) for s in range(S)])
        if i + 1 < steps:
            batch.step(n + i, fed=True, tokens=1, logits=True, sampling=sampling, seeds=seeds)
    return turn


class Session:
    """Turns on one batch that reuse its KV cache across runs.

    Runtime::start with Engine::generate's rewind (runtime.cpp:236-275,
    engine.cpp:690-701): each sequence's held tokens, and the placed edits of
    the run that wrote its cache, are kept between turns.  A turn keeps what
    every sequence may reuse (``prefix.reusable``: the common prefix, cut at
    the first edit difference and short of the prompt's last token), which
    the cache's window rule may still empty (``Batch.truncate``), and
    prefills the rest.  The reply's tokens fed back in stay cached, so the
    next turn's prompt may extend this one's conversation, or the same
    prompt may run again with other edits from the position they change."""

    def __init__(self, batch: Batch):
        self.batch = batch
        self.held = [[] for _ in range(batch.sequences)]
        self.held_edits = [[] for _ in range(batch.sequences)]
        self.reused = 0

    def run(self, prompts, steps: int, sampling: Sampling = Sampling(), edit_sets=None, seeds=None,
            keep_logits: bool = False, capture: bool = False) -> Turn:
        S = self.batch.sequences
        prompts = [[int(t) for t in p] for p in prompts]
        if len(prompts) != S or len({len(p) for p in prompts}) != 1 or not prompts[0]:
            raise ValueError("one non-empty prompt a sequence, all the same length")
        origin = len(prompts[0]) - 1
        sets = list(edit_sets or [None] * S)
        placed = [E.placed(es, origin) if es else [] for es in sets]
        keep = min(P.reusable(self.held[s], self.held_edits[s], prompts[s], placed[s]) for s in range(S))
        self.reused = self.batch.truncate(keep)
        turn = generate(self.batch, prompts, steps, sampling, sets, seeds, keep_logits, capture,
                        start=self.reused)
        for s in range(S):
            self.held[s] = prompts[s] + turn.tokens[s][:steps - 1]
            self.held_edits[s] = placed[s]
        return turn

