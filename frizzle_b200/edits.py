"""Steering edits: the reference's Edit, its checks and its u32 table.

A restatement of ``src/core/edit/edit.cpp`` (``check`` :105-145, ``table``
:147-170, ``apply`` :93-104, ``placed`` :172-179) and ``edit.h``'s layout
(:50-60): per layer [first, count], then five words an edit
{neuron, kind, value bits, first position, end position}, sorted by
(layer, neuron, from, index), ranges placed at ``origin`` and saturating at
``TO_THE_END``.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass

SET, SCALE, ZERO = 0, 1, 2
TO_THE_END = 0xFFFFFFFF
MAX_EDITS = 4096
EDIT_WORDS = 5

# EditError (edit.h:140-150).
OK, KIND, LAYER, NEURON, NOT_FINITE, ZERO_VALUE, RANGE, OVERLAP, TOO_MANY = range(9)


@dataclass(frozen=True)
class Edit:
    layer: int
    neuron: int
    kind: int
    value: float
    start: int             # the first step it applies at (the reference's `from`)
    until: int = TO_THE_END


@dataclass
class EditCheck:
    error: int = OK
    index: int = 0
    subject: str = ""

    @property
    def ok(self) -> bool:
        return self.error == OK


def _f32(v: float) -> float:
    return struct.unpack("<f", struct.pack("<f", v))[0]


def _bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", v))[0]


def place(step: int, origin: int) -> int:
    """Step s at position origin + s, saturating at TO_THE_END (edit.cpp:29-33)."""
    if step == TO_THE_END or step > TO_THE_END - origin:
        return TO_THE_END
    return step + origin


def apply(kind: int, value: float, neuron: float) -> float:
    if kind == SET:
        return value
    if kind == SCALE:
        return _f32(neuron * value)
    if kind == ZERO:
        return 0.0
    return neuron


def _range(e: Edit) -> str:
    return f"[{e.start}, {'end' if e.until == TO_THE_END else e.until})"


def check(edits, layers: int, width) -> EditCheck:
    """The first fault of a set of edits, or OK; `width` is the FFN width (int or per-layer list)."""
    widths = [width] * layers if isinstance(width, int) else list(width)
    if len(edits) > MAX_EDITS:
        return EditCheck(TOO_MANY, MAX_EDITS, f"{len(edits)} edits; at most {MAX_EDITS}")
    for i, e in enumerate(edits):
        if e.kind not in (SET, SCALE, ZERO):
            return EditCheck(KIND, i, f"edit {i}: kind {e.kind} is not Set, Scale or Zero")
        if e.layer >= layers:
            return EditCheck(LAYER, i, f"edit {i}: layer {e.layer} is past the model's {layers} layers")
        if e.neuron >= widths[e.layer]:
            return EditCheck(NEURON, i, f"edit {i}: neuron {e.neuron} is past layer {e.layer}'s "
                                        f"{widths[e.layer]} neurons")
        if not math.isfinite(e.value):
            return EditCheck(NOT_FINITE, i, f"edit {i}: the value is not finite")
        if e.kind == ZERO and e.value != 0.0:
            return EditCheck(ZERO_VALUE, i, f"edit {i}: a Zero edit's value is not 0")
        if e.start >= e.until:
            return EditCheck(RANGE, i, f"edit {i}: layer {e.layer} neuron {e.neuron}'s steps {_range(e)} hold no step")
    # Ranges of one neuron held so far never overlap, so an edit overlaps one of
    # them exactly when it overlaps its neighbour before or after its key.
    held = []  # sorted (layer, neuron, start, index)
    import bisect
    for i, e in enumerate(edits):
        key = (e.layer, e.neuron, e.start)
        at = bisect.bisect_left(held, key + (-1,))
        other = None
        if at < len(held):
            o = edits[held[at][3]]
            if o.layer == e.layer and o.neuron == e.neuron and o.start < e.until:
                other = held[at][3]
        if other is None and at > 0:
            o = edits[held[at - 1][3]]
            if o.layer == e.layer and o.neuron == e.neuron and e.start < o.until:
                other = held[at - 1][3]
        if other is not None:
            return EditCheck(OVERLAP, i, f"edit {i}: layer {e.layer} neuron {e.neuron}'s steps {_range(e)} "
                                         f"overlap edit {other}'s {_range(edits[other])}")
        if at < len(held) and held[at][:3] == key:
            continue  # same key already held: the map keeps the first
        held.insert(at, key + (i,))
    return EditCheck()


def table(edits, layers: int, origin: int) -> list:
    """The u32 words the kernels read (edit.cpp:147-170).  Precondition: check passed."""
    words = [0] * (2 * layers + EDIT_WORDS * len(edits))
    at = 2 * layers
    order = sorted(range(len(edits)), key=lambda i: (edits[i].layer, edits[i].neuron, edits[i].start, i))
    for i in order:
        e = edits[i]
        head = 2 * e.layer
        if words[head + 1] == 0:
            words[head] = at
        words[head + 1] += 1
        words[at:at + 5] = [e.neuron, e.kind, _bits(e.value), place(e.start, origin), place(e.until, origin)]
        at += EDIT_WORDS
    return words


def placed(edits, origin: int) -> list:
    return [Edit(e.layer, e.neuron, e.kind, e.value, place(e.start, origin), place(e.until, origin)) for e in edits]
