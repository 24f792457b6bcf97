"""Parity at BASELINE.json's larger configs, through the C ABI on the GPU
against the CPU oracle, at the bars the north star states: logits and
per-layer captures within 1e-2 max-abs and 1e-3 relative RMS, identical greedy
tokens; products within the kernel tests' bars.

- Config 2: the tied head's 262,144 x 1152 product at M = 8 (the skinny
  head kernel), 64 and 512 rows (the tcgen05 GEMM, f32-level).
- Config 3: one 4096-token prefill step of the 26-layer model (the global
  layers attend over the whole prompt, the local ones over their window),
  the last row's logits, greedy token and per-layer capture.  The oracle's
  4096-row forward pass takes a few minutes on the host: marked slow, still
  collected by `-m gpu`.
- Config 5: a decode step at position 32,512 through the persistent decode
  kernel.  Both sides' key/value caches are filled with the same seeded f16
  keys and values for positions 0..32,511 (fz_batch_cache on the GPU, the
  oracle's rings on the host; KvCache::advance declares them held), so the
  oracle need not prefill 32k tokens; then a second, fed step.
- Config 4's sampling on the Gemma-shaped model: a steered sequence and its
  unsteered twin in one batch under the same seed, temperature 1 and top-k
  64, each draw against the oracle's own draw over its own logits."""
import numpy as np
import pytest

import oracle
from frizzle_b200 import _native, engine, synth
from frizzle_b200.edits import Edit, SET, check, table

from conftest import max_abs, rel_rms
from test_gpu_kernels import repacked, split_dev, stream, torch_cuda
from test_gpu_model import MAX_ABS, REL_RMS, assert_parity, prompt, run_both

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m", [8, 64, 512])
def test_c2_head_rows(m):
    torch = torch_cuda()
    lib = _native.load()
    n, k = 262144, 1152
    blocks = synth.random_q4_0(n, k, seed=5)
    codes, scales = repacked(blocks, n, k)
    x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    if m <= 16:
        am = torch.zeros(m, dtype=torch.int64, device="cuda")
        xd = torch.from_numpy(x).cuda()
        _native.check(lib.fz_q4_0_head(codes.data_ptr(), scales.data_ptr(), n, k, xd.data_ptr(), m, y.data_ptr(),
                                       am.data_ptr(), stream()))
        bar = 1e-5
    else:
        hi, lo = split_dev(x)
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        _native.check(lib.fz_q4_0_gemm(codes.data_ptr(), scales.data_ptr(), n, k, hi.data_ptr(), lo.data_ptr(), 1, m,
                                       y.data_ptr(), err.data_ptr(), stream()))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        bar = 5e-5   # the f32-level tensor-core product's bar (its own f32 accumulation)
    got = y.cpu().numpy()
    want = oracle.matmul(blocks, n, k, x)
    assert np.isfinite(got).all()
    assert rel_rms(got, want) < bar, rel_rms(got, want)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


@pytest.mark.slow
def test_c3_prefill_4096(gemma_model_path):
    # One 4096-token step (the tcgen05 path for every product, the tensor-core prefill attention),
    # then two decode steps.
    out = run_both(gemma_model_path, synth.GEMMA3_1B, 4096, 3, block=4096, capture=True, context=8192)
    assert_parity(out)


def _to_device(dst: int, host: np.ndarray) -> None:
    """Copies a host array to a raw device pointer (the CUDA runtime through
    cuda-python)."""
    from cuda.bindings import runtime as rt
    host = np.ascontiguousarray(host)
    err, = rt.cudaMemcpy(dst, host.ctypes.data, host.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice)
    assert err == rt.cudaError_t.cudaSuccess, err


def _seeded_caches(shape, batch, orc, upto, seed=17):
    """Writes the same seeded f16 keys and values for positions 0..upto-1 into
    the GPU batch's rings and the oracle's (slot p mod slots on each side),
    only the positions each ring still holds at the end."""
    per = shape.kv_heads * shape.head_dim
    for layer in range(shape.layers):
        g_slots = batch.cache(0, layer)[1]
        o_slots = orc.slots(layer)
        first = max(0, upto - min(g_slots, o_slots))
        rng = np.random.default_rng([seed, layer])
        keys = (rng.standard_normal((upto - first, per), dtype=np.float32) * np.float32(0.5)).astype(np.float16)
        vals = rng.standard_normal((upto - first, per), dtype=np.float32).astype(np.float16)
        pos = np.arange(first, upto)
        for values, src in ((False, keys), (True, vals)):
            ptr, slots = batch.cache(0, layer, values=values)
            ring = np.zeros((slots, per), dtype=np.uint16)
            ring[pos % slots] = src.view(np.uint16)
            _to_device(ptr, ring)
        k_ring = np.zeros((o_slots, per), dtype=np.uint16)
        v_ring = np.zeros((o_slots, per), dtype=np.uint16)
        k_ring[pos % o_slots] = keys.view(np.uint16)
        v_ring[pos % o_slots] = vals.view(np.uint16)
        orc.write_cache(layer, k_ring, v_ring)


@pytest.mark.slow
def test_c5_decode_at_32k(gemma_model_path):
    s = synth.GEMMA3_1B
    upto = 32768 - 256
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, gemma_model_path)
    batch = engine.Batch(model, 1, 32768)
    orc = oracle.OracleModel(gemma_model_path, context=32768)
    _seeded_caches(s, batch, orc, upto)
    _native.check(batch.lib.fz_batch_cache_advance(batch.handle, upto))
    tok0 = int(prompt(s, 1, seed=9)[0])
    batch.step(upto, np.array([tok0], dtype=np.uint32), tokens=1, logits=True)
    want, _ = orc.step(upto, [tok0], logits=True)
    got = batch.logits(0)
    tok = batch.tokens()[0]
    assert tok == int(np.argmax(want))
    assert rel_rms(got, want) < REL_RMS and max_abs(got, want) < MAX_ABS, (rel_rms(got, want), max_abs(got, want))
    # The next, fed step reads the key and value the first one appended.
    batch.step(upto + 1, fed=True, tokens=1, logits=True)
    want, _ = orc.step(upto + 1, [tok], logits=True)
    got = batch.logits(0)
    assert batch.tokens()[0] == int(np.argmax(want))
    assert rel_rms(got, want) < REL_RMS and max_abs(got, want) < MAX_ABS, (rel_rms(got, want), max_abs(got, want))
    orc.close()
    batch.free()
    model.free()
    dev.close()


@pytest.mark.slow
def test_c4_gemma_sampled_steered_pair(gemma_model_path):
    """Config 4's draw on the Gemma-shaped model: sequence 0 steered at layer
    13 (8 neurons set in [-10, 10]), sequence 1 its unsteered twin, one batch,
    the same seed, temperature 1, top-k 64.  Each draw's uniform must be the
    oracle's bits (Philox is integer arithmetic) and its token the oracle's
    unless the uniform falls within float rounding of a cumulative boundary;
    the oracle follows the GPU's tokens."""
    s = synth.GEMMA3_1B
    n_prompt, steps, seed = 64, 8, (3, 5)
    rng = np.random.default_rng(21)
    idx = rng.choice(s.ffn, size=8, replace=False)
    vals = rng.uniform(-10, 10, size=8).astype(np.float32)
    edits = [Edit(13, int(i), SET, float(v), 0) for i, v in zip(idx, vals)]
    assert check(edits, s.layers, s.ffn).ok
    words = np.array(table(edits, s.layers, n_prompt - 1), dtype=np.uint32)
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, gemma_model_path)
    batch = engine.Batch(model, 2, 1024)
    batch.set_edits(0, words)
    batch.set_edits(1, None)
    samp = engine.Sampling(temperature=1.0, top_k=64, top_p=1.0, min_p=0.0, seed=seed)
    ids = prompt(s, n_prompt, seed=4)
    batch.step(0, np.stack([ids, ids]), tokens=n_prompt, logits=True, sampling=samp)
    orcs = [oracle.OracleModel(gemma_model_path, context=1024) for _ in range(2)]
    want = [orcs[0].step(0, ids, logits=True, edit_table=words)[0], orcs[1].step(0, ids, logits=True)[0]]
    drawn = [[], []]
    agree = total = 0
    for i in range(steps):
        recs = batch.wait()
        for q in range(2):
            tok, failed, u = int(recs[q][0]), int(recs[q][1]), float(recs[q][2])
            cand = oracle.topk64(want[q])
            w = oracle.draw(cand, 64, 1.0, 1.0, 0.0, seed, n_prompt + i)
            assert failed == 0
            assert np.float32(u).view(np.uint32) == w[2]
            agree += tok == int(w[0])
            total += 1
            drawn[q].append(tok)
        if i + 1 < steps:
            batch.step(n_prompt + i, fed=True, tokens=1, logits=True, sampling=samp)
            want = [orcs[0].step(n_prompt + i, [drawn[0][-1]], logits=True, edit_table=words)[0],
                    orcs[1].step(n_prompt + i, [drawn[1][-1]], logits=True)[0]]
    assert agree >= total - 1, (agree, total)
    for o in orcs:
        o.close()
    batch.free()
    model.free()
    dev.close()
