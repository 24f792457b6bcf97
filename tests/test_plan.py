"""The residency plan for one batch (plan_residency / place_cache,
src/core/residency/plan.cpp:321-419, restated for one B200 and a batch of
sequences), from a Gemma-3-1B-shaped file's index, without a device.

Checked against budgets computed here by hand: the weights are every
tensor's bytes plus the RoPE turns, the f16 prefill copies two halves of
every layer product, the rings window + 512 + rollback slots rounded up to
32 (a global layer's the context) of f16 keys and values a sequence; the
bisection's context is the brute-force largest that fits."""
import ctypes as C

import numpy as np
import pytest

from frizzle_b200 import _native, gguf, synth

S = synth.GEMMA3_1B
ROLLBACK = 4096


def plan(budget, sequences=1, context=0, rows=0, rollback=ROLLBACK, shape=S):
    head, size = synth.model_header(shape)
    p = _native.Plan(sequences=sequences, context=context, rollback=rollback, rows=rows, budget=budget)
    buf = C.create_string_buffer(head, len(head))
    st = _native.load().fz_model_index_plan(buf, len(head), size, C.byref(p))
    return st, p


def ring(window, context, rollback=ROLLBACK):
    return min(context, -(-(window + 512 + rollback) // 32) * 32)


def cache_bytes(context, sequences, shape=S, rollback=ROLLBACK):
    total = 0
    for layer in range(shape.layers):
        window = shape.context if layer % shape.pattern == shape.pattern - 1 else shape.window
        total += 2 * ring(window, context, rollback) * shape.kv_heads * shape.head_dim * 2 * sequences
    return total


def test_weights_and_copies_by_hand():
    head, _ = synth.model_header(S)
    idx = gguf.read_index(head)
    weights = sum(t.nbytes for t in idx.tensors.values()) + S.layers * (S.head_dim // 2) * 4
    q, kv = S.heads * S.head_dim, S.kv_heads * S.head_dim
    copies = S.layers * ((q + 2 * kv) * S.hidden + S.hidden * q + 3 * S.ffn * S.hidden) * 4
    st, p = plan(180 << 30)
    assert st == 0, _native.load().fz_last_error()
    assert p.weight_bytes == weights
    assert p.copy_bytes == copies == 2_791_047_168
    # Everything fits 180 GB: the trained context for the one sequence.
    assert p.context == S.context and p.sequences == 1
    assert p.cache_bytes == cache_bytes(S.context, 1)


def test_cache_bytes_at_given_contexts():
    for context, seqs in ((512, 1), (4096, 2), (5119, 3), (32768, 16)):
        st, p = plan(180 << 30, sequences=seqs, context=context)
        assert st == 0
        assert (p.context, p.sequences) == (context, seqs)
        assert p.cache_bytes == cache_bytes(context, seqs)
        assert p.total_bytes == p.weight_bytes + p.copy_bytes + p.scratch_bytes + p.cache_bytes + (1 << 26)


def test_largest_context_by_bisection_matches_brute_force():
    # A budget that lands between the shortest and the trained context for 8 sequences.
    st, hi = plan(180 << 30, sequences=8, context=20000)
    budget = hi.total_bytes - 1
    st, p = plan(budget, sequences=8)
    assert st == 0
    assert p.context == 19999
    # Brute force over a neighbourhood: the plan's context fits, the next one does not.
    for ctx, fits in ((p.context, True), (p.context + 1, False)):
        s2, q = plan(180 << 30, sequences=8, context=ctx)
        assert (q.total_bytes <= budget) == fits


def test_most_sequences_at_a_context():
    st, four = plan(180 << 30, sequences=4, context=32768)
    st, five = plan(180 << 30, sequences=5, context=32768)
    budget = (four.total_bytes + five.total_bytes) // 2
    st, p = plan(budget, sequences=0, context=32768)
    assert st == 0 and p.sequences == 4 and p.context == 32768


def test_budget_below_the_shortest_context_is_refused():
    st, p = plan(1 << 30)   # 1 GiB: the weights and copies alone are 3.4 GB
    assert st == 5          # FZ_ERR_FIT
    assert b"ExceedsBudget" in _native.load().fz_last_error()
    assert p.total_bytes > 1 << 30


def test_refusals():
    assert plan(180 << 30, sequences=17)[0] == 1
    assert plan(180 << 30, context=S.context + 1)[0] == 1
    assert plan(0)[0] == 1   # no device: a budget is required


def test_pinned_mix_weights():
    # The pinned file's Q8_0 embedding takes its file bytes on the device; each
    # Q4_1 block of ffn_down (20 bytes) becomes a Q4_0 block and a 4-byte
    # correction (22).
    P = synth.GEMMA3_1B_PINNED
    head, _ = synth.model_header(P)
    idx = gguf.read_index(head)
    q4_1 = [t for t in idx.tensors.values() if t.ggml_type == gguf.TYPE_Q4_1]
    assert len(q4_1) == 3 and idx.tensors["token_embd.weight"].ggml_type == gguf.TYPE_Q8_0
    weights = sum(t.nbytes for t in idx.tensors.values()) + sum(t.nbytes // 10 for t in q4_1)
    weights += P.layers * (P.head_dim // 2) * 4
    st, p = plan(180 << 30, shape=P)
    assert st == 0, _native.load().fz_last_error()
    assert p.weight_bytes == weights
    assert p.copy_bytes == 2_791_047_168
