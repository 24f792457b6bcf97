"""The capture store without a GPU: its layout against the reference's own
capture::layout (golden fixtures written by tests/golden/make_golden.py from
src/core/capture/capture.cpp), and the oracle's weights, statistics and
readouts against their definitions (capture/weights.h:24-62, capture.h:26-33)
on the tiny model."""
import json
import os

import numpy as np
import pytest

import oracle
from frizzle_b200 import capture, synth

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "capture_layout.json")))
SHAPES = {"gemma3_1b": synth.GEMMA3_1B, "tiny": synth.TINY}


def golden_layer(rec, l):
    w = rec["layers"][l]
    slots = {n: (w[2 * i], w[2 * i + 1]) for i, n in enumerate(capture.SLOTS)}
    return slots, w[16], w[17], w[18], bool(w[19])


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_layout_matches_reference(name):
    rec, shape = GOLDEN[name], SHAPES[name]
    lay = capture.layout(shape)
    assert lay.words == rec["words"]
    for l in range(shape.layers):
        slots, keys, heads, window, full = golden_layer(rec, l)
        got = lay.layers[l]
        for n in capture.SLOTS:
            assert getattr(got, n) == slots[n], (l, n)
        assert (got.keys, got.query_heads, got.window, got.full_attention) == (keys, heads, window, full)


def test_gemma_layout_counts_of_the_reference_header():
    # capture.h:52-59: neurons 179,712 words, the store 869,072 (3.3 MiB).
    lay = capture.layout(synth.GEMMA3_1B)
    assert lay.neuron_words == 179_712 and lay.words == 869_072
    globals_ = [l for l, s in enumerate(lay.layers) if s.full_attention]
    assert globals_ == [5, 11, 17, 23]


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_oracle_layout_matches_reference(name):
    rec, shape = GOLDEN[name], SHAPES[name]
    layers, words = oracle.capture_layout(shape)
    assert words == rec["words"]
    for l in range(shape.layers):
        slots, keys, _, _, _ = golden_layer(rec, l)
        for n in capture.SLOTS:
            assert layers[l][n] == slots[n][0], (l, n)
        assert layers[l]["keys"] == keys


def test_reader_views():
    shape = synth.TINY
    lay = capture.layout(shape)
    store = np.arange(lay.words, dtype=np.float32)
    pairs = np.zeros((64, 2), dtype=np.uint32)
    pairs[:, 0] = np.arange(64, dtype=np.float32)[::-1].view(np.uint32)
    pairs[:, 1] = np.arange(64) * 7
    first = lay.layers[3].readout[0]
    store[first:first + 128] = pairs.ravel().view(np.float32)
    cap = capture.Capture(store, lay, shape.head_dim)
    assert cap.weights(5).shape == (shape.heads, shape.context)
    assert cap.weights(0).shape == (shape.heads, shape.window)
    assert cap.query(2)[1, 0] == lay.layers[2].query[0] + shape.head_dim
    logits, tokens = cap.readout(3)
    assert logits[0] == 63.0 and tokens[5] == 35


@pytest.fixture(scope="module")
def tiny_capture(tiny_model_path):
    orc = oracle.OracleModel(tiny_model_path, context=512)
    ids = np.random.default_rng(5).integers(2, synth.TINY.vocab, size=40).astype(np.uint32)
    logits, cap = orc.step(0, ids, logits=True, capture=True)
    yield orc, ids, logits, capture.Capture(cap, capture.layout(synth.TINY), synth.TINY.head_dim)
    orc.close()


def test_oracle_weights_are_a_softmax(tiny_capture):
    _, ids, _, cap = tiny_capture
    s = synth.TINY
    p = len(ids) - 1
    for l in range(s.layers):
        keys = cap.layout.layers[l].keys
        count = min(p + 1, keys)
        w = cap.weights(l)
        assert np.all(w[:, count:] == 0)
        assert np.all(w[:, :count] > 0)
        np.testing.assert_allclose(w[:, :count].sum(axis=1, dtype=np.float64), 1.0, atol=1e-5)
        m, lsum = cap.stats(l).T
        assert np.all(lsum >= 1.0)
        # The largest weight is 1 / l: its key scored m.
        np.testing.assert_allclose(w.max(axis=1), 1.0 / lsum, rtol=1e-6)


def test_oracle_weights_follow_the_scores(tiny_capture):
    """Weights recomputed in f64 from q (the captured query) and the cached keys."""
    orc, ids, _, cap = tiny_capture
    s = synth.TINY
    p = len(ids) - 1
    scale = np.float64(np.float32(np.float64(1.0 / np.sqrt(np.float32(s.head_dim))) * 1.4426950408889634))
    for l in (0, 5):
        kc, _ = orc.cache(l)
        slots = orc.slots(l)
        k = oracle_f16(kc).reshape(slots, s.kv_heads, s.head_dim)
        keys = cap.layout.layers[l].keys
        count = min(p + 1, keys)
        pos = np.arange(p + 1 - count, p + 1)
        q = cap.query(l).astype(np.float64) * scale
        sc = q @ k[pos % slots, 0].T.astype(np.float64)
        w = np.exp2(sc - sc.max(axis=1, keepdims=True))
        w /= w.sum(axis=1, keepdims=True)
        np.testing.assert_allclose(cap.weights(l)[:, :count], w, rtol=2e-5, atol=1e-7)


def oracle_f16(words):
    return np.asarray(words, dtype=np.uint16).view(np.float16).astype(np.float32)


def test_oracle_readouts(tiny_capture):
    orc, _, logits, cap = tiny_capture
    s = synth.TINY
    lt, tt = cap.readout(s.layers - 1)
    want = oracle.topk64(logits)
    assert np.array_equal(np.stack([lt.view(np.uint32), tt], axis=1).ravel(), want.ravel())
    embd = oracle.dequant(orc.tensor("token_embd.weight")).reshape(s.vocab, s.hidden).astype(np.float64)
    gain = orc.tensor("output_norm.weight").view(np.float32).astype(np.float64)
    for l in range(s.layers - 1):
        x = cap.residual(l + 1).astype(np.float64)
        normed = x / np.sqrt(np.mean(x * x) + s.eps) * gain
        ref = embd @ normed
        rl, rt = cap.readout(l)
        # Logits within f32 rounding of an f64 product; order descending.
        np.testing.assert_allclose(rl, ref[rt], rtol=1e-4, atol=1e-4)
        assert np.all(np.diff(rl) <= 0)
        # Every token outside the readout scores no higher than its last.
        outside = np.setdiff1d(np.arange(s.vocab), rt)
        assert ref[outside].max() <= rl[-1] + 1e-4
