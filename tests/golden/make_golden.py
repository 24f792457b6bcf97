"""Writes tests/golden/edits.json, capture_layout.json and prefix.json from
the reference's own edit, capture and cache code.

Runs Frizzle's ``edit::check`` and ``edit::table`` (src/core/edit/edit.cpp),
``capture::layout`` (src/core/capture/capture.cpp), ``longest_common_prefix``
and ``first_edit_difference`` (src/core/cache/prefix.cpp) and
``KvCache::truncate``/``advance`` (src/core/cache/kv.cpp), compiled in place
into oracle/_ref/libfrizzle_ref.so by ``make -C oracle ref``, over the edit
sets, model shapes, token sequences and cache histories below, and records
what they return.  The sets cover the
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
        # The checkout's root: FRIZZLE_REFERENCE, or the path BASELINE.json records.
        sys.path.insert(0, ROOT)
        import __graft_entry__
        ref = __graft_entry__.reference_checkout()
        if not ref:
            sys.exit("make_golden.py needs the reference checkout (set FRIZZLE_REFERENCE)")
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", f"REF={ref}"], check=True)
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
    write_prefix(lib)


def prefix_cases():
    """(cached, incoming) token sequences and placed edit sets."""
    import random
    rng = random.Random(7)
    seq = [rng.randrange(2, 262144) for _ in range(300)]
    tokens = [([], []), (seq[:10], []), ([], seq[:10]), (seq, seq), (seq[:120], seq), (seq, seq[:120]),
              (seq[:50] + [1] + seq[51:], seq), ([5] + seq[1:], seq), (seq[:299] + [3], seq)]
    A = e(13, 7, SET, 4.0, 3, 9)
    edits = [
        ([], []),
        ([A], [A]),
        ([A], [e(13, 7, SET, 4.5, 3, 9)]),                            # value differs: its start
        ([e(13, 7, SET, 4.0, 3, 5), e(13, 7, SET, 4.0, 5, 9)], [A]),  # split ranges are one edit
        ([A], [e(13, 7, SCALE, 4.0, 3, 9)]),                          # kind differs
        ([A], [e(13, 7, SET, 4.0, 3, 7)]),                            # shorter range: its end
        ([A], [e(13, 7, SET, 4.0, 5, 9)]),                            # later start
        ([A], []), ([], [A]),                                          # only in one set
        ([e(2, 1, SET, 0.0, 0, 4)], [e(2, 1, SET, -0.0, 0, 4)]),      # value bits differ
        ([e(2, 1, SET, float("nan"), 0, 4)], [e(2, 1, SET, float("nan"), 0, 4)]),
        ([A, e(2, 1, ZERO, 0.0, 10, TO_END)], [e(2, 1, ZERO, 0.0, 10, TO_END), A]),  # order does not matter
        ([A, e(2, 1, ZERO, 0.0, 10, TO_END)], [A, e(2, 1, ZERO, 0.0, 12, TO_END)]),
        ([e(0, 0, SET, 1.0, 0, TO_END)], [e(0, 0, SET, 1.0, 0, 100)]),
        ([e(4, 9, SCALE, 2.0, 20, 30), e(4, 9, SCALE, 2.0, 40, 50)], [e(4, 9, SCALE, 2.0, 20, 30)]),
    ]
    for trial in range(12):
        base = []
        for _ in range(rng.randrange(1, 40)):
            a = rng.randrange(0, 300)
            base.append(e(rng.randrange(26), rng.randrange(6912), rng.randrange(3), float(rng.randrange(-8, 9)) / 2,
                          a, a + rng.randrange(1, 60) if rng.random() < 0.8 else TO_END))
        other = list(base)
        rng.shuffle(other)
        if trial % 3:
            i = rng.randrange(len(other))
            l, n, k, v, a, u = other[i]
            other[i] = (l, n, k, v + 0.5, a, u) if trial % 3 == 1 else (l, n, k, v, a + 1, u)
        edits.append((base, other))
    return tokens, edits


def kv_cases():
    """KvCache histories: (windows, slots, capacity, operations)."""
    import random
    rng = random.Random(11)
    g_win = [32768 if l % 6 == 5 else 512 for l in range(26)]
    g_slots = [8192 if w == 32768 else 5120 for w in g_win]
    t_win = [4096 if l % 6 == 5 else 16 for l in range(7)]
    t_slots = [2048 if w == 4096 else 544 for w in t_win]
    out = []
    for windows, slots, cap in ((g_win, g_slots, 8192), (t_win, t_slots, 2048)):
        for trial in range(6):
            ops, length = [], 0
            for _ in range(40):
                if length and rng.random() < 0.45:
                    t = rng.choice([0, length, rng.randrange(length + 1), max(0, length - rng.randrange(1, 700))])
                    ops.append((1, t))
                    length = t  # provisional: the reference's answer decides
                else:
                    n = min(cap - length, rng.choice([1, 16, 300, 1500, rng.randrange(1, 4000)]))
                    if n <= 0:
                        continue
                    ops.append((0, n))
                    length += n
            out.append([windows, slots, cap, ops])
    return out


def write_prefix(lib):
    lib.ref_longest_common_prefix.restype = C.c_size_t
    lib.ref_longest_common_prefix.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
    lib.ref_first_edit_difference.restype = C.c_uint32
    lib.ref_first_edit_difference.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
    lib.ref_kv_run.restype = None
    lib.ref_kv_run.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_size_t, C.c_void_p]
    tokens, edits = prefix_cases()
    out = {"lcp": [], "fed": [], "kv": []}
    for a, b in tokens:
        x = (C.c_uint32 * max(1, len(a)))(*a)
        y = (C.c_uint32 * max(1, len(b)))(*b)
        out["lcp"].append([a, b, lib.ref_longest_common_prefix(x, len(a), y, len(b))])
    for a, b in edits:
        x = (RefEdit * max(1, len(a)))(*[RefEdit(*r) for r in a])
        y = (RefEdit * max(1, len(b)))(*[RefEdit(*r) for r in b])
        enc = lambda rs: [[l, n, k, ("nan" if v != v else v), f, u] for l, n, k, v, f, u in rs]
        out["fed"].append([enc(a), enc(b), lib.ref_first_edit_difference(x, len(a), y, len(b))])
    # The histories' truncations may be refused (the cache empties): replay
    # them so each later operation stays within the reference's length.
    for windows, slots, cap, ops in kv_cases():
        fixed, res = [], []
        for op in ops:
            trial = fixed + [op]
            w = (C.c_uint32 * len(windows))(*windows)
            s_ = (C.c_uint32 * len(slots))(*slots)
            o = (C.c_uint32 * (2 * len(trial)))(*[v for p in trial for v in p])
            r = (C.c_uint32 * (2 * len(trial)))()
            length = 0 if not fixed else res[-1][1]
            if op[0] == 1 and op[1] > length:
                op = (1, length)
            if op[0] == 0 and length + op[1] > cap:
                continue
            trial = fixed + [op]
            o = (C.c_uint32 * (2 * len(trial)))(*[v for p in trial for v in p])
            lib.ref_kv_run(w, s_, len(windows), cap, o, len(trial), r)
            fixed = trial
            res = [(r[2 * i], r[2 * i + 1]) for i in range(len(trial))]
        out["kv"].append({"windows": windows, "slots": slots, "capacity": cap,
                          "ops": [list(p) for p in fixed], "results": [list(p) for p in res]})
    with open(os.path.join(HERE, "prefix.json"), "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    print("wrote prefix cases", {k: len(v) for k, v in out.items()}, file=sys.stderr)


if __name__ == "__main__":
    main()
