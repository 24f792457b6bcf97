"""The steering sweep's per-rank run on the GPU against the oracle: every steered sequence and its
unsteered twin, batched several to a step (the prompt prefilled in one tensor-core step, then one-token
steps through the persistent decode kernel), greedy, token for token."""
import numpy as np
import pytest

import oracle
from frizzle_b200 import edits as E
from frizzle_b200 import engine, sweep, synth

pytestmark = pytest.mark.gpu


def test_tiny_sweep_matches_oracle(tiny_model_path):
    s = synth.TINY
    pairs = sweep.make_pairs(5, s.ffn, seed=5)   # 10 sequences: groups of 4, 4 (batch reused) and 2
    prompt = np.random.default_rng([5, 20]).integers(2, s.vocab, size=20).astype(np.uint32)
    steps, layer = 5, 3
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, tiny_model_path)
    got = sweep.run(model, prompt, pairs, steps, layer, batch_seqs=4, context=256, temperature=0.0)
    model.free()
    dev.close()
    for p in pairs:
        for row, steered in ((0, True), (1, False)):
            words = np.array(E.table(p.edits(layer), s.layers, len(prompt) - 1), dtype=np.uint32) if steered else None
            orc = oracle.OracleModel(tiny_model_path, context=256)
            logits, _ = orc.step(0, prompt, logits=True, edit_table=words)
            want = []
            for i in range(steps):
                tok = int(np.argmax(logits))
                want.append(tok)
                if i + 1 < steps:
                    logits, _ = orc.step(len(prompt) + i, [tok], logits=True, edit_table=words)
            orc.close()
            assert got[p.index][row].tolist() == want, (p.index, steered, got[p.index][row].tolist(), want)
