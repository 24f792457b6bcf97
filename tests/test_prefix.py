"""Prefix reuse and the KV cache's bookkeeping without a GPU, against the
reference's own code (golden fixtures written by tests/golden/make_golden.py
from src/core/cache/prefix.cpp and src/core/cache/kv.cpp): the token and edit
differences, and KvCache's truncate/advance histories replayed through the C
ABI's fz_cache_truncate_keeps."""
import ctypes as C
import json
import os

import numpy as np
import pytest

from frizzle_b200 import _native, prefix
from frizzle_b200.edits import Edit

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "prefix.json")))


def _edit(rec):
    l, n, k, v, f, u = rec
    return (l, n, k, float("nan") if v == "nan" else float(v), f, u)


@pytest.mark.parametrize("i", range(len(GOLDEN["lcp"])))
def test_longest_common_prefix_matches_reference(i):
    a, b, want = GOLDEN["lcp"][i]
    assert prefix.longest_common_prefix(a, b) == want


@pytest.mark.parametrize("i", range(len(GOLDEN["fed"])))
def test_first_edit_difference_matches_reference(i):
    a, b, want = GOLDEN["fed"][i]
    assert prefix.first_edit_difference([_edit(x) for x in a], [_edit(x) for x in b]) == want


def test_first_edit_difference_takes_edit_records():
    a = [Edit(13, 7, 0, 4.0, 3, 5), Edit(13, 7, 0, 4.0, 5, 9)]
    assert prefix.first_edit_difference(a, [Edit(13, 7, 0, 4.0, 3, 9)]) == prefix.TO_END
    assert prefix.first_edit_difference(a, [Edit(13, 7, 0, 4.0, 3, 8)]) == 8


class Kv:
    """KvCache's counts driven through the ABI's truncate rule."""

    def __init__(self, windows, slots):
        self.lib = _native.load()
        self.w = (C.c_uint32 * len(windows))(*windows)
        self.s = (C.c_uint32 * len(slots))(*slots)
        self.n = len(windows)
        self.length = self.written = 0

    def advance(self, n):
        self.length += n
        self.written = max(self.written, self.length)
        return self.length

    def truncate(self, t):
        if t > 0 and self.lib.fz_cache_truncate_keeps(C.cast(self.w, C.c_void_p), C.cast(self.s, C.c_void_p),
                                                      self.n, self.written, t):
            self.length = t
        else:
            self.length = self.written = 0
        return self.length


@pytest.mark.parametrize("i", range(len(GOLDEN["kv"])))
def test_kv_cache_histories_match_reference(i):
    case = GOLDEN["kv"][i]
    kv = Kv(case["windows"], case["slots"])
    for (kind, arg), (want, length) in zip(case["ops"], case["results"]):
        got = kv.advance(arg) if kind == 0 else kv.truncate(arg)
        assert (got, kv.length) == (want, length), (kind, arg)


def test_histories_cover_kept_and_emptied_truncations():
    kept = emptied = 0
    for case in GOLDEN["kv"]:
        for (kind, arg), (res, _) in zip(case["ops"], case["results"]):
            if kind == 1 and arg > 0:
                kept += res == arg
                emptied += res == 0
    assert kept >= 10 and emptied >= 10


def test_reusable():
    p = [5, 6, 7, 8]
    assert prefix.reusable([], [], p, []) == 0
    assert prefix.reusable(p, [], p, []) == 3               # the last token is recomputed
    assert prefix.reusable(p + [9, 10], [], p + [9, 11], []) == 5
    e = [Edit(2, 1, 0, 1.0, 2, prefix.TO_END)]
    assert prefix.reusable(p + [9], [], p + [9, 4], e) == 2  # edits start at position 2
