"""Steering edits: the host's check/table against the reference's own edit.cpp
(golden fixtures written by tests/golden/make_golden.py), and the oracle's edit
launch against the reference's apply() on the edit kernel's known answers
(tests/contracts/kernels/edit_kernel_test.cpp's activation pattern)."""
import json
import os
import struct

import numpy as np
import pytest

import oracle
from frizzle_b200 import edits as E

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "edits.json")))
CASES = sorted(k for k in GOLDEN if not k.startswith("_"))


def _edits(rec):
    out = []
    for layer, neuron, kind, value, start, until in rec["edits"]:
        v = float("nan") if value == "nan" else float("inf") if value == "inf" else float(value)
        out.append(E.Edit(layer, neuron, kind, v, start, until))
    return out


@pytest.mark.parametrize("name", CASES)
def test_check_and_table_match_reference(name):
    rec = GOLDEN[name]
    edits = _edits(rec)
    got = E.check(edits, rec["layers"], rec["width"])
    assert (got.error, got.index) == (rec["error"], rec["index"])
    if rec["error"] == 0:
        assert E.table(edits, rec["layers"], rec["origin"]) == rec["table"]
    else:
        assert got.subject


def test_apply_matches_reference():
    for kind, value, neuron, want_bits in GOLDEN["_apply"]:
        got = E.apply(kind, value, neuron)
        assert struct.unpack("<I", struct.pack("<f", got))[0] == want_bits


def kat_activation(rows=5, width=200):
    """(i % 97) * 0.375 - 13, with a subnormal at neuron 7 and -0 at neuron 8."""
    a = (np.arange(rows * width) % 97).astype(np.float32) * np.float32(0.375) - np.float32(13.0)
    a = a.reshape(rows, width)
    a[:, 7] = np.array([0x123], dtype=np.uint32).view(np.float32)[0]
    a[:, 8] = np.float32(-0.0)
    return a


def expected(before, edits, layer, origin, position, rows):
    out = before.copy()
    for e in E.placed(edits, origin):
        if e.layer != layer:
            continue
        for r in range(rows):
            p = position + r
            if e.start <= p < e.until:
                if e.kind == E.SCALE and e.value == 1.0:
                    continue  # the kernel keeps the bits
                out[r, e.neuron] = np.float32(E.apply(e.kind, e.value, float(out[r, e.neuron])))
    return out


@pytest.mark.parametrize("case,position,rows", [
    ("kernel_kat_all", 36, 5),      # a block ending at the origin: only its last row is edited
    ("kernel_kat_from_2", 40, 5),   # a range starting inside the block
    ("kernel_kat_until_3", 40, 5),  # a range ending inside the block
    ("kernel_kat_until_6", 45, 1),  # a decode step inside the range
    ("kernel_kat_until_6", 46, 1),  # past its end: nothing
    ("kernel_kat_all", 0, 5),       # a block before every range
    ("one_neuron_three_ranges", 40, 5),
])
def test_oracle_edit_launch_known_answers(case, position, rows):
    rec = GOLDEN[case]
    edits = _edits(rec)
    before = kat_activation(rows)
    got = oracle.edit_apply(rec["table"], 1, position, before)
    want = expected(before, edits, 1, rec["origin"], position, rows)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # Scale x 1 keeps the subnormal and the negative zero, bit for bit.
    assert np.array_equal(got[:, 7:9].view(np.uint32), before[:, 7:9].view(np.uint32))


def test_no_edits_change_nothing():
    before = kat_activation()
    got = oracle.edit_apply(GOLDEN["empty"]["table"][:6], 1, 40, before)
    assert np.array_equal(got.view(np.uint32), before.view(np.uint32))
