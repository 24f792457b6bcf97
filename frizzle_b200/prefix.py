"""How much of a new run the KV cache already holds (cache/prefix.h:87-92).

Attention is causal, so a position's keys and values depend only on the
tokens up to it and on the edits in force at those positions.  A run may
reuse the cache up to the first position where either differs from the run
that wrote it: ``min(longest_common_prefix, first_edit_difference)``, less
one when that is the whole prompt, because the first draw needs the last
prompt token's logits, which the cache does not hold
(src/core/runtime/runtime.cpp:257-262, engine.cpp:690-701).
"""
from __future__ import annotations

import struct

TO_END = 0xFFFFFFFF  # edit::kToTheEnd


def longest_common_prefix(cached, incoming) -> int:
    """How many leading tokens the two sequences share."""
    n = 0
    for a, b in zip(cached, incoming):
        if a != b:
            break
        n += 1
    return n


def _fields(e):
    if hasattr(e, "layer"):
        return e.layer, e.neuron, e.kind, e.value, e.start, e.until
    return tuple(e)


def _bits(v) -> int:
    return struct.unpack("<I", struct.pack("<f", float(v)))[0]


def first_edit_difference(cached, incoming) -> int:
    """The least position at which the edits in force differ, or TO_END.

    Both are placed edit sets (positions, not steps: ``edits.placed``).  The
    edits in force at a position are those whose range [start, until) holds
    it, each with its kind and value bits, per (layer, neuron); how a set's
    ranges are ordered or split does not matter.  Each neuron's in-force edit
    is constant between the starts and ends of its ranges, so the two sets
    are compared at those points only, in order."""
    per = {}
    for side, edits in ((0, cached), (1, incoming)):
        for e in edits:
            layer, neuron, kind, value, start, until = _fields(e)
            per.setdefault((layer, neuron), ([], []))[side].append((start, until, kind, _bits(value)))
    least = TO_END
    for ranges in per.values():
        points = sorted({p for side in ranges for r in side for p in r[:2]})
        for p in points:
            if p >= least:
                break
            here = [next(((k, b) for s, u, k, b in side if s <= p < u), None) for side in ranges]
            if here[0] != here[1]:
                least = p
                break
    return least


def reusable(cached_tokens, cached_edits, prompt, placed_edits) -> int:
    """Tokens of `prompt` a cache written by (cached_tokens, cached_edits) may
    keep: the common prefix, cut at the first edit difference and short of
    the prompt's last token (before the cache's own window rule)."""
    keep = min(longest_common_prefix(cached_tokens, prompt), max(len(prompt) - 1, 0))
    return min(keep, first_edit_difference(cached_edits, placed_edits))
