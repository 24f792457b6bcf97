"""Model-level parity through the C ABI on the GPU against the CPU oracle.

The north-star bar: per-layer activations and logits within 1e-2 max-abs and
1e-3 relative RMS of the oracle's f32, and identical greedy tokens over the
whole run, unsteered and steered.  BASELINE config 1 is the 26-layer
Gemma-3-1B-shaped Q4_0 model (seed 0) with 32 prompt tokens, 32-token prefill
then 32 greedy decode steps; the tiny model runs the same path in seconds."""
import numpy as np
import pytest

import oracle
from frizzle_b200 import capture as C
from frizzle_b200 import engine, synth
from frizzle_b200.edits import Edit, SET, SCALE, ZERO, check, table

from conftest import max_abs, rel_rms

pytestmark = pytest.mark.gpu

MAX_ABS, REL_RMS = 1e-2, 1e-3


def prompt(shape, n, seed=0):
    return np.random.default_rng([seed, n]).integers(2, shape.vocab, size=n).astype(np.uint32)


def compare_capture(got, want, shape, got_logits=None):
    """Two capture stores slot kind by slot kind: the activations (neurons,
    residuals, additions, queries) and the attention weights against the
    north-star bars; the statistics (m in log2 units within the max-abs bar,
    the sums l within the relative-RMS bar over every layer and head); each
    readout's logits in order, and its tokens wherever the oracle's logits
    stand more than twice the logit bar from their neighbours; and the last
    layer's readout against the top 64 of the GPU's own logits, bit for bit."""
    lay = C.layout(shape)
    g, w = C.Capture(got, lay, shape.head_dim), C.Capture(want, lay, shape.head_dim)
    L = shape.layers
    r = {"act_rms": rel_rms(g.activations(), w.activations()), "act_abs": max_abs(g.activations(), w.activations())}
    gw = np.concatenate([g.weights(l).ravel() for l in range(L)])
    ww = np.concatenate([w.weights(l).ravel() for l in range(L)])
    r["w_rms"], r["w_abs"] = rel_rms(gw, ww), max_abs(gw, ww)
    r["w_zeros"] = bool(np.array_equal(gw == 0, ww == 0))
    gs = np.stack([g.stats(l) for l in range(L)])
    ws = np.stack([w.stats(l) for l in range(L)])
    r["m_abs"] = max_abs(gs[..., 0], ws[..., 0])
    r["l_rms"] = rel_rms(gs[..., 1], ws[..., 1])
    r["l_rel_max"] = float(np.max(np.abs(gs[..., 1] / ws[..., 1] - 1)))
    r["readout_abs"], r["readout_tokens"] = 0.0, True
    for l in range(L):
        gl, gt = g.readout(l)
        wl, wt = w.readout(l)
        r["readout_abs"] = max(r["readout_abs"], max_abs(gl, wl))
        gap = np.minimum(np.abs(np.diff(wl, prepend=np.inf)), np.abs(np.diff(wl, append=-np.inf)))
        clear = gap > 2 * MAX_ABS
        r["readout_tokens"] &= bool(np.array_equal(gt[clear], wt[clear]))
    if got_logits is not None:
        gl, gt = g.readout(L - 1)
        mine = oracle.topk64(got_logits).reshape(64, 2)
        r["last_readout_own"] = bool(np.array_equal(gl.view(np.uint32), mine[:, 0]) and np.array_equal(gt, mine[:, 1]))
    return r


def run_both(path, shape, n_prompt, steps, edits=None, capture=True, context=4096, block=16):
    """Greedy decode on the GPU and the oracle; returns per-step comparisons.
    The prompt is prefilled in steps of `block` tokens: up to 16 rows run the
    skinny tensor-core matvec, more rows the tcgen05 GEMM path."""
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, path)
    batch = engine.Batch(model, 1, context)
    orc = oracle.OracleModel(path, context=context)
    ids = prompt(shape, n_prompt)
    words = None
    if edits:
        assert check(edits, shape.layers, shape.ffn).ok
        words = np.array(table(edits, shape.layers, n_prompt - 1), dtype=np.uint32)
        batch.set_edits(0, words)
    out = {"tokens_gpu": [], "tokens_cpu": [], "logit_rms": [], "logit_abs": [], "captures": []}
    # Prefill in blocks, the last asking for logits.
    pos = 0
    while pos < n_prompt:
        t = min(block, n_prompt - pos)
        last = pos + t == n_prompt
        batch.step(pos, ids[pos:pos + t], tokens=t, logits=last, capture=capture and last)
        pos += t
    want_logits, want_cap = orc.step(0, ids, logits=True, edit_table=words, capture=capture)
    for i in range(steps):
        tok = batch.tokens()[0]
        got = batch.logits(0)
        out["tokens_gpu"].append(tok)
        out["tokens_cpu"].append(int(np.argmax(want_logits)))
        out["logit_rms"].append(rel_rms(got, want_logits))
        out["logit_abs"].append(max_abs(got, want_logits))
        if capture and i < 2 and want_cap is not None:
            # The prompt's last step, then the first decode step (one row).
            cap = batch.capture(0)
            out["captures"].append(compare_capture(cap, want_cap, shape, got))
            if i == 0:
                out["cap_layers"] = (cap, want_cap)
        if i + 1 < steps:
            nxt = out["tokens_cpu"][-1]
            cap_now = capture and i == 0
            batch.step(n_prompt + i, fed=True, tokens=1, logits=True, capture=cap_now)
            want_logits, want_cap = orc.step(n_prompt + i, [nxt], logits=True, edit_table=words, capture=cap_now)
    kv = []
    for layer in (0, shape.pattern - 1):
        ptr, slots = batch.cache(0, layer)
        kv.append((layer, ptr, slots))
    orc.close()
    batch.free()
    model.free()
    dev.close()
    return out


def assert_parity(out):
    assert out["tokens_gpu"] == out["tokens_cpu"], (out["tokens_gpu"], out["tokens_cpu"])
    assert max(out["logit_rms"]) < REL_RMS, max(out["logit_rms"])
    assert max(out["logit_abs"]) < MAX_ABS, max(out["logit_abs"])
    for c in out["captures"]:
        assert c["act_rms"] < REL_RMS and c["act_abs"] < MAX_ABS, c
        assert c["w_rms"] < REL_RMS and c["w_abs"] < MAX_ABS and c["w_zeros"], c
        assert c["m_abs"] < MAX_ABS and c["l_rms"] < REL_RMS, c
        assert c["readout_abs"] < MAX_ABS and c["readout_tokens"], c
        assert c["last_readout_own"], c


def test_tiny_model_greedy(tiny_model_path):
    assert_parity(run_both(tiny_model_path, synth.TINY, 21, 12))


def test_tiny_model_steered(tiny_model_path):
    s = synth.TINY
    edits = [Edit(3, 5, SET, 8.0, 0), Edit(3, 100, SCALE, -2.5, 1), Edit(3, 900, ZERO, 0.0, 0, 3),
             Edit(6, 17, SET, -10.0, 2, 5)]
    out = run_both(tiny_model_path, s, 9, 8, edits=edits)
    assert_parity(out)
    cap, _ = out["cap_layers"]
    neurons = C.Capture(cap, C.layout(s), s.head_dim).neurons(3)
    assert neurons[5] == np.float32(8.0) and neurons[900] == 0.0


def test_tiny_model_long_prompt_wraps_window(tiny_model_path):
    # 70 prompt tokens: the window layers (16 keys) read a sliding range and the
    # prefill crosses several 16-token blocks.
    assert_parity(run_both(tiny_model_path, synth.TINY, 70, 6))


def test_gemma_1b_config1_greedy(gemma_model_path):
    out = run_both(gemma_model_path, synth.GEMMA3_1B, 32, 32, capture=True)
    assert_parity(out)


def test_gemma_1b_config1_steered(gemma_model_path):
    s = synth.GEMMA3_1B
    rng = np.random.default_rng(13)
    idx = rng.choice(s.ffn, size=8, replace=False)
    vals = rng.uniform(-10, 10, size=8).astype(np.float32)
    edits = [Edit(13, int(i), SET, float(v), 0) for i, v in zip(idx, vals)]
    out = run_both(gemma_model_path, s, 32, 32, edits=edits, capture=True)
    assert_parity(out)


def test_tiny_model_sampled_draw(tiny_model_path):
    """Temperature 1, top-k 64 (config 4's sampling): the GPU's top-64 selection
    and Philox draw against the oracle's on the oracle's own logits; the uniform
    must be the same bits (Philox is integer arithmetic) and the token the same
    unless the uniform falls within float rounding of a cumulative boundary."""
    s = synth.TINY
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, tiny_model_path)
    batch = engine.Batch(model, 1, 512)
    orc = oracle.OracleModel(tiny_model_path, context=512)
    samp = engine.Sampling(temperature=1.0, top_k=64, top_p=1.0, min_p=0.0, seed=(7, 9))
    ids = prompt(s, 12, seed=3)
    batch.step(0, ids, tokens=12, logits=True, sampling=samp)
    want_logits, _ = orc.step(0, ids, logits=True)
    agree = 0
    for i in range(10):
        rec = batch.wait()[0]
        tok, failed, u = int(rec[0]), int(rec[1]), float(rec[2])
        cand = oracle.topk64(want_logits)
        want = oracle.draw(cand, 64, 1.0, 1.0, 0.0, (7, 9), 12 + i)
        assert failed == 0
        assert np.float32(u).view(np.uint32) == want[2]
        agree += tok == int(want[0])
        batch.step(12 + i, fed=True, tokens=1, logits=True, sampling=samp)
        want_logits, _ = orc.step(12 + i, [tok], logits=True)
    batch.wait()
    assert agree >= 9
    orc.close()
    batch.free()
    model.free()
    dev.close()


def test_tiny_model_wide_prefill(tiny_model_path):
    # A 40-token prompt in one step: every product on the tcgen05 GEMM path.
    assert_parity(run_both(tiny_model_path, synth.TINY, 40, 8, block=40))


def test_tiny_model_wide_prefill_steered(tiny_model_path):
    edits = [Edit(3, 5, SET, 8.0, 0), Edit(3, 100, SCALE, -2.5, 0), Edit(4, 900, ZERO, 0.0, 0, 3)]
    out = run_both(tiny_model_path, synth.TINY, 33, 6, edits=edits, block=33)
    assert_parity(out)


def test_gemma_1b_config1_one_step_prefill(gemma_model_path):
    # Config 1's 32-token prompt as one step (32 rows: the GEMM path), then decode.
    assert_parity(run_both(gemma_model_path, synth.GEMMA3_1B, 32, 32, block=32))


def test_gemma_1b_config1_one_step_prefill_steered(gemma_model_path):
    s = synth.GEMMA3_1B
    rng = np.random.default_rng(13)
    idx = rng.choice(s.ffn, size=8, replace=False)
    vals = rng.uniform(-10, 10, size=8).astype(np.float32)
    edits = [Edit(13, int(i), SET, float(v), 0) for i, v in zip(idx, vals)]
    assert_parity(run_both(gemma_model_path, s, 32, 32, edits=edits, block=32))


def test_gemma_1b_256_token_prefill(gemma_model_path):
    # A 256-token prompt in one step, two 128-row tiles of the GEMM, then decode.
    assert_parity(run_both(gemma_model_path, synth.GEMMA3_1B, 256, 8, block=256))


def run_batch(path, shape, S, n_prompt, steps, edit_sets=None, context=4096, block=None):
    """S sequences stepped together (one decode launch serves them all), each
    against its own oracle run; prompts differ per sequence.  The prompt goes in
    steps of `block` tokens a sequence (default: 16 rows a step)."""
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, path)
    batch = engine.Batch(model, S, context)
    prompts = [prompt(shape, n_prompt, seed=11 + s) for s in range(S)]
    words = []
    for s in range(S):
        es = (edit_sets or [None] * S)[s]
        w = np.array(table(es, shape.layers, n_prompt - 1), dtype=np.uint32) if es else None
        batch.set_edits(s, w)
        words.append(w)
    block = block or max(1, 16 // S)
    pos = 0
    while pos < n_prompt:
        t = min(block, n_prompt - pos)
        ids = np.array([p[pos:pos + t] for p in prompts], dtype=np.uint32)
        batch.step(pos, ids, tokens=t, logits=pos + t == n_prompt)
        pos += t
    got_tokens, got_logits = [], []
    for i in range(steps):
        got_tokens.append(batch.tokens())
        got_logits.append([batch.logits(s) for s in range(S)])
        if i + 1 < steps:
            batch.step(n_prompt + i, fed=True, tokens=1, logits=True)
    batch.free()
    model.free()
    dev.close()
    worst_rms = worst_abs = 0.0
    for s in range(S):
        orc = oracle.OracleModel(path, context=context)
        want, _ = orc.step(0, prompts[s], logits=True, edit_table=words[s])
        for i in range(steps):
            tok = int(np.argmax(want))
            assert got_tokens[i][s] == tok, (s, i, got_tokens[i][s], tok)
            worst_rms = max(worst_rms, rel_rms(got_logits[i][s], want))
            worst_abs = max(worst_abs, max_abs(got_logits[i][s], want))
            if i + 1 < steps:
                want, _ = orc.step(n_prompt + i, [tok], logits=True, edit_table=words[s])
        orc.close()
    assert worst_rms < REL_RMS, worst_rms
    assert worst_abs < MAX_ABS, worst_abs


@pytest.mark.parametrize("S", [2, 8])
def test_tiny_model_chunked_wide_prefill(tiny_model_path, S):
    # Config 5 in small: S sequences whose 700-token prompts go in 256-token
    # steps (GEMM and tensor-core attention reading the keys of earlier steps
    # from the cache, the window layers sliding), then batched decode whose
    # global layers split 700+ keys over many CTAs and fold the splits.
    s = synth.TINY
    edits = [[Edit(3, 5, SET, 8.0, 0)]] + [None] * (S - 1)
    run_batch(tiny_model_path, s, S, 700, 6, edit_sets=edits, block=256)


@pytest.mark.parametrize("n_prompt,block", [(2048, 2048), (2100, 1024)])
def test_tiny_model_split_key_ranges(tiny_model_path, n_prompt, block):
    # Long causal blocks of the global layer (5) split their keys over two CTAs
    # of the tensor-core attention and the second to finish merges: a
    # 2048-token step (blocks of up to 64 key tiles), and 1024-token steps
    # whose later blocks start past position 1024 (the third step's 52 rows
    # at position 2048, ~66 tiles each).
    assert_parity(run_both(tiny_model_path, synth.TINY, n_prompt, 4, block=block))


@pytest.mark.parametrize("S", [3, 6])
def test_tiny_model_batch_decode(tiny_model_path, S):
    # 3 sequences: one column quad of the decode kernel's fragments; 6: two.
    edit_sets = [None] * S
    edit_sets[1] = [Edit(3, 5, SET, 8.0, 0), Edit(4, 900, ZERO, 0.0, 0, 3)]
    run_batch(tiny_model_path, synth.TINY, S, 12, 8, edit_sets=edit_sets)


def test_tiny_model_layered_decode(tiny_model_path, monkeypatch):
    # The per-operation launches (FRIZZLE_B200_LAYERED=1) stay a working path.
    monkeypatch.setenv("FRIZZLE_B200_LAYERED", "1")
    assert_parity(run_both(tiny_model_path, synth.TINY, 21, 8))


def test_tiny_model_decode_attention_splits(tiny_model_path):
    # 700 prompt tokens: the global layer's decode attention spans two
    # 512-key splits, folded by the last CTA.
    assert_parity(run_both(tiny_model_path, synth.TINY, 700, 4, block=700))


def test_gemma_1b_steered_pair_decode(gemma_model_path):
    # A steered sequence and its unsteered twin stepped together (config 4's pairing).
    s = synth.GEMMA3_1B
    rng = np.random.default_rng(4)
    idx = rng.choice(s.ffn, size=5, replace=False)
    vals = rng.uniform(-10, 10, size=5).astype(np.float32)
    edits = [Edit(13, int(i), SET, float(v), 0) for i, v in zip(idx, vals)]
    run_batch(gemma_model_path, s, 2, 32, 8, edit_sets=[edits, None])


def test_two_steps_in_flight_report_in_order(tiny_model_path):
    """Greedy decode with the next step enqueued before the previous step's
    records are read (wait_oldest): the same tokens, in order, as one step at
    a time, and the oracle's greedy tokens."""
    s = synth.TINY
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, tiny_model_path)
    ids = prompt(s, 10, seed=21)
    got = []
    for pipelined in (False, True):
        batch = engine.Batch(model, 1, 512)
        batch.step(0, ids, tokens=10, logits=True)
        toks = [int(batch.wait()[0][0])]
        n = 12
        if pipelined:
            batch.step(10, fed=True, tokens=1, logits=True)
            for i in range(n):
                if i + 1 < n:
                    batch.step(11 + i, fed=True, tokens=1, logits=True)
                toks.append(int(batch.wait_oldest()[0][0]))
            with pytest.raises(RuntimeError):
                batch.wait_oldest()
        else:
            for i in range(n):
                batch.step(10 + i, fed=True, tokens=1, logits=True)
                toks.append(int(batch.wait()[0][0]))
        got.append(toks)
        batch.free()
    assert got[0] == got[1], got
    orc = oracle.OracleModel(tiny_model_path, context=512)
    want, _ = orc.step(0, ids, logits=True)
    expect = [int(np.argmax(want))]
    for i in range(12):
        want, _ = orc.step(10 + i, [expect[-1]], logits=True)
        expect.append(int(np.argmax(want)))
    orc.close()
    model.free()
    dev.close()
    assert got[1] == expect, (got[1], expect)


@pytest.mark.parametrize("path_fixture,shape", [("tiny_model_path", synth.TINY),
                                                ("gemma_model_path", synth.GEMMA3_1B)])
def test_capture_layout_through_the_abi(request, path_fixture, shape):
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, request.getfixturevalue(path_fixture))
    lay = C.layout(shape)
    assert model.capture_floats == lay.words
    for l in range(shape.layers):
        got = model.capture_layout(l)
        want = lay.layers[l]
        for n in C.SLOTS:
            assert got[n] == getattr(want, n), (l, n)
        assert (got["keys"], got["query_heads"], got["window"], got["full_attention"]) == \
            (want.keys, want.query_heads, want.window, want.full_attention)
    model.free()
    dev.close()


@pytest.mark.parametrize("S", [3])
def test_tiny_model_batch_capture(tiny_model_path, S):
    """Each sequence's store against its own oracle run: the prompt's last
    step (rows of three sequences) and a one-row decode step (the persistent
    decode kernel), one sequence steered."""
    s = synth.TINY
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, tiny_model_path)
    batch = engine.Batch(model, S, 512)
    prompts = [prompt(s, 12, seed=21 + q) for q in range(S)]
    words = [None] * S
    words[1] = np.array(table([Edit(3, 5, SET, 8.0, 0)], s.layers, 11), dtype=np.uint32)
    batch.set_edits(1, words[1])
    batch.step(0, np.array(prompts, dtype=np.uint32), tokens=12, logits=True, capture=True)
    toks = batch.tokens()
    caps = [batch.capture(q) for q in range(S)]
    logits = [batch.logits(q) for q in range(S)]
    batch.step(12, fed=True, tokens=1, logits=True, capture=True)
    batch.tokens()
    caps2 = [batch.capture(q) for q in range(S)]
    logits2 = [batch.logits(q) for q in range(S)]
    batch.free()
    model.free()
    dev.close()
    for q in range(S):
        orc = oracle.OracleModel(tiny_model_path, context=512)
        want_logits, want_cap = orc.step(0, prompts[q], logits=True, edit_table=words[q], capture=True)
        assert toks[q] == int(np.argmax(want_logits))
        _, want_cap2 = orc.step(12, [toks[q]], logits=True, edit_table=words[q], capture=True)
        orc.close()
        for c in (compare_capture(caps[q], want_cap, s, logits[q]), compare_capture(caps2[q], want_cap2, s, logits2[q])):
            assert c["act_rms"] < REL_RMS and c["act_abs"] < MAX_ABS, (q, c)
            assert c["w_rms"] < REL_RMS and c["w_abs"] < MAX_ABS and c["w_zeros"], (q, c)
            assert c["m_abs"] < MAX_ABS and c["l_rms"] < REL_RMS, (q, c)
            assert c["readout_abs"] < MAX_ABS and c["readout_tokens"] and c["last_readout_own"], (q, c)


def oracle_greedy(path, ids, steps, edits=None, context=512):
    """The oracle's greedy tokens and first logits for a prompt from position 0."""
    orc = oracle.OracleModel(path, context=context)
    words = None
    if edits:
        words = np.array(table(edits, synth.TINY.layers, len(ids) - 1), dtype=np.uint32)
    logits, _ = orc.step(0, np.asarray(ids, dtype=np.uint32), logits=True, edit_table=words)
    first = logits
    toks = [int(np.argmax(logits))]
    for i in range(steps - 1):
        logits, _ = orc.step(len(ids) + i, [toks[-1]], logits=True, edit_table=words)
        toks.append(int(np.argmax(logits)))
    orc.close()
    return toks, first


def test_session_reuses_the_cache_across_turns(tiny_model_path):
    """Runtime::start's reuse: a turn extending the last one's conversation
    prefills only its new tokens; the same prompt with edits from a later
    position recomputes from there; a rewind past the rollback reserve empties
    the cache.  Every turn's tokens are the oracle's from scratch."""
    s = synth.TINY
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, tiny_model_path)
    batch = engine.Batch(model, 1, 1024, rollback=0)
    sess = engine.Session(batch)
    a = list(prompt(s, 20, seed=31))
    t1 = sess.run([a], 6, keep_logits=True)
    assert sess.reused == 0
    assert t1.tokens[0] == oracle_greedy(tiny_model_path, a, 6)[0]
    assert batch.cache_state()[0] == 25
    # The conversation goes on: the held prompt and reply, then new tokens.
    b = a + t1.tokens[0][:5] + list(prompt(s, 7, seed=32))
    t2 = sess.run([b], 6, keep_logits=True)
    assert sess.reused == 25
    want, first = oracle_greedy(tiny_model_path, b, 6)
    assert t2.tokens[0] == want
    assert rel_rms(t2.logits[0][0], first) < REL_RMS and max_abs(t2.logits[0][0], first) < MAX_ABS
    # The same prompt, steered from its last position: only that position is recomputed.
    edits = [Edit(3, 5, SET, 8.0, 0), Edit(4, 900, ZERO, 0.0, 0)]
    t3 = sess.run([b], 4, edit_sets=[edits])
    assert sess.reused == len(b) - 1
    assert t3.tokens[0] == oracle_greedy(tiny_model_path, b, 4, edits)[0]
    # A step past the cached tokens is refused.
    with pytest.raises(engine.FzError):
        batch.step(batch.cache_state()[0] + 1, [1], tokens=1)
    # Past the reserve: 600 more tokens, then a prompt sharing only 10 of them.
    long = b + list(prompt(s, 600, seed=33))
    sess.run([long], 2)
    assert sess.reused == len(b) - 1   # the last turn's edits were in force from there
    short = long[:10] + list(prompt(s, 5, seed=34))
    t5 = sess.run([short], 3)
    assert sess.reused == 0        # the window layers' rings have moved on
    assert t5.tokens[0] == oracle_greedy(tiny_model_path, short, 3)[0]
    batch.free()
    model.free()
    dev.close()
