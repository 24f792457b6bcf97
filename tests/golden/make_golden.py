"""Writes tests/golden/edits.json and capture_layout.json from the reference's
own edit and capture code.

Runs Frizzle's ``edit::check`` and ``edit::table`` (src/core/edit/edit.cpp)
and ``capture::layout`` (src/core/capture/capture.cpp), compiled in place into
oracle/_ref/libfrizzle_ref.so by ``make -C oracle ref``, over the edit sets
and model shapes below, and records what they return.  The sets cover the
cases the reference's edit tests cover (every fault with its index, overlap
naming the later edit, touching ranges, placement and saturation, the edit
kernel's 150-edit known-answer set); the sets themselves are written here.

Needs the reference checkout; the JSON it writes is committed so the tests
run without it.
"""
import ctypes as C
import json
import os
import struct
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
LIB = os.path.join(ROOT, "oracle", "_ref", "libfrizzle_ref.so")

TO_END = 0xFFFFFFFF
SET, SCALE, ZERO = 0, 1, 2
LAYERS, WIDTH = 26, 6912


class RefEdit(C.Structure):
    _fields_ = [("layer", C.c_uint32), ("neuron", C.c_uint32), ("kind", C.c_uint32), ("value", C.c_float),
                ("start", C.c_uint32), ("until", C.c_uint32)]


def e(layer, neuron, kind, value, start=0, until=TO_END):
    return [layer, neuron, kind, value, start, until]


def bits(v):
    return struct.unpack("<I", struct.pack("<f", v))[0]


def kernel_kat_edits(start=0, until=TO_END):
    """The edit kernel's known-answer set: layer 1 holds 150 mixed edits of
    neurons 10..159 plus Scale x 1 on neurons 7 and 8; layers 0 and 2 hold
    edits the layer-1 launch must ignore."""
    out = []
    for n in range(10, 160):
        kind = n % 3
        if kind == 0:
            out.append(e(1, n, SET, n * 0.5, start, until))
        elif kind == 1:
            out.append(e(1, n, SCALE, -1.75, start, until))
        else:
            out.append(e(1, n, ZERO, 0.0, start, until))
    out += [e(1, 7, SCALE, 1.0, start, until), e(1, 8, SCALE, 1.0, start, until),
            e(0, 3, SET, 999.0), e(2, 4, SET, -999.0), e(0, 20, ZERO, 0.0)]
    return out


def cases():
    good = e(3, 10, SET, 1.0)
    c = {
        "empty": ([], LAYERS, WIDTH, 0),
        "full": ([e(i % LAYERS, i, SCALE, 2.0) for i in range(4096)], LAYERS, WIDTH, 7),
        "two_valid": ([e(LAYERS - 1, WIDTH - 1, ZERO, 0.0), e(0, 0, SET, -3.5, 4, 5)], LAYERS, WIDTH, 3),
        "bad_kind": ([good, e(0, 0, 7, 1.0)], LAYERS, WIDTH, 0),
        "bad_layer": ([good, e(LAYERS, 0, SET, 1.0)], LAYERS, WIDTH, 0),
        "bad_neuron": ([good, e(2, WIDTH, SET, 1.0)], LAYERS, WIDTH, 0),
        "nan_value": ([e(1, 1, SCALE, float("nan"))], LAYERS, WIDTH, 0),
        "inf_value": ([e(1, 1, SET, float("inf"))], LAYERS, WIDTH, 0),
        "zero_with_value": ([e(1, 1, ZERO, 0.5)], LAYERS, WIDTH, 0),
        "empty_range": ([good, e(1, 1, SET, 1.0, 7, 7)], LAYERS, WIDTH, 0),
        "reversed_range": ([e(1, 1, SET, 1.0, 8, 7)], LAYERS, WIDTH, 0),
        "unranged": ([e(3, 10, SET, 1.0, 0, 0)], LAYERS, WIDTH, 0),
        "too_many": ([good] * 4097, LAYERS, WIDTH, 0),
        "overlap_later_named": ([e(5, 7, SET, 1.0, 0, 10), e(9, 2, SET, 1.0, 3, TO_END), e(9, 2, SCALE, 2.0, 0, 4),
                                 e(5, 7, ZERO, 0.0, 9, TO_END)], LAYERS, WIDTH, 0),
        "overlap_inside": ([e(1, 1, SET, 1.0, 4, 6), e(1, 1, SET, 2.0, 0, 20)], LAYERS, WIDTH, 0),
        "touching_ranges": ([e(5, 7, SET, 1.0, 0, 6), e(5, 7, SCALE, 3.0, 6, 9), e(5, 7, ZERO, 0.0, 9, TO_END),
                             e(5, 8, SET, 1.0, 2, 4)], LAYERS, WIDTH, 10),
        "fault_before_overlap": ([e(5, 7, SET, 1.0), e(5, 7, SET, 1.0), e(LAYERS, 0, SET, 1.0),
                                  e(1, WIDTH, SET, 1.0)], LAYERS, WIDTH, 0),
        "table_order": ([e(12, 4031, SET, 8.0, 3, 9), e(3, 900, SCALE, -2.0), e(12, 17, ZERO, 0.0, 5, TO_END),
                         e(25, 6911, SCALE, 1.0, 0, 1), e(12, 4031, SCALE, 2.0, 0, 3)], LAYERS, WIDTH, 41),
        "saturating": ([e(0, 0, SET, 1.0, 2, TO_END - 1)], LAYERS, WIDTH, 100),
        "kernel_kat_all": (kernel_kat_edits(), 3, 200, 40),
        "kernel_kat_from_2": (kernel_kat_edits(2), 3, 200, 40),
        "kernel_kat_until_3": (kernel_kat_edits(0, 3), 3, 200, 40),
        "kernel_kat_until_6": (kernel_kat_edits(0, 6), 3, 200, 40),
        "one_neuron_three_ranges": ([e(1, 50, SET, 1.0, 0, 2), e(1, 50, SET, 2.0, 2, 4),
                                     e(1, 50, SCALE, -3.0, 4, TO_END)], 3, 200, 40),
    }
    return c


def main():
    if not os.path.exists(LIB):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref"], check=True)
    lib = C.CDLL(LIB)
    lib.ref_edit_check.restype = C.c_int
    lib.ref_edit_check.argtypes = [C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint32, C.POINTER(C.c_size_t),
                                   C.c_char_p, C.c_size_t]
    lib.ref_edit_table.restype = C.c_size_t
    lib.ref_edit_table.argtypes = [C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p,
                                   C.c_size_t]
    out = {}
    for name, (edits, layers, width, origin) in cases().items():
        arr = (RefEdit * max(1, len(edits)))(*[RefEdit(*x) for x in edits])
        index = C.c_size_t()
        subject = C.create_string_buffer(512)
        err = lib.ref_edit_check(arr, len(edits), layers, width, C.byref(index), subject, 512)
        rec = {"edits": [[a, b, c_, ("nan" if v != v else ("inf" if v == float("inf") else v)), s, u]
                         for a, b, c_, v, s, u in edits],
               "layers": layers, "width": width, "origin": origin, "error": err, "index": index.value}
        if err == 0:
            n = lib.ref_edit_table(arr, len(edits), layers, width, origin, None, 0)
            words = (C.c_uint32 * max(1, n))()
            lib.ref_edit_table(arr, len(edits), layers, width, origin, words, n)
            rec["table"] = list(words)[:n]
        out[name] = rec
    # apply(): Scale x 1 keeps bits, Set stores, Zero stores +0.
    apply_cases = []
    lib.ref_edit_apply.restype = C.c_float
    lib.ref_edit_apply.argtypes = [C.c_uint32, C.c_float, C.c_float]
    for kind, value, neuron in [(SET, 4.25, -1.0), (SCALE, 3.0, 0.5), (ZERO, 0.0, -7.0), (SCALE, 1.0, -0.0),
                                (SCALE, 1.0, 1.401298464324817e-45), (SCALE, -1.75, 3.0)]:
        apply_cases.append([kind, value, neuron, bits(lib.ref_edit_apply(kind, value, neuron))])
    out["_apply"] = apply_cases
    with open(os.path.join(HERE, "edits.json"), "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    print("wrote", len(out), "cases", file=sys.stderr)
    # capture::layout over Gemma 3 1B's shape and the tiny test model's.
    lib.ref_capture_layout.restype = C.c_uint64
    lib.ref_capture_layout.argtypes = [C.c_uint32] * 8 + [C.c_void_p]
    shapes = {"gemma3_1b": dict(layers=26, width=1152, ffn=6912, heads=4, head_dim=256, window=512, pattern=6,
                                context=32768),
              "tiny": dict(layers=7, width=512, ffn=1024, heads=4, head_dim=256, window=16, pattern=6,
                           context=4096)}
    lay = {}
    for name, sh in shapes.items():
        words = (C.c_uint32 * (20 * sh["layers"]))()
        total = lib.ref_capture_layout(sh["layers"], sh["width"], sh["ffn"], sh["heads"], sh["head_dim"],
                                       sh["window"], sh["pattern"], sh["context"], words)
        lay[name] = {"shape": sh, "words": total,
                     "layers": [list(words)[20 * l:20 * l + 20] for l in range(sh["layers"])]}
    with open(os.path.join(HERE, "capture_layout.json"), "w") as f:
        json.dump(lay, f, indent=0, sort_keys=True)
    print("wrote capture layouts", {k: v["words"] for k, v in lay.items()}, file=sys.stderr)


if __name__ == "__main__":
    main()
