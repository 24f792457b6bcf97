"""The model with the pinned file's format mix (docs/architecture/
logical-overview.md:63-64): the tied embedding and head Q8_0, ffn_down Q4_1
in layers 0-2, every other linear Q4_0.  On the GPU the Q8_0 table is read by
the embedding gather and by the head (the norm's rows in f32, the Q8_0
product, the argmax); a Q4_1 down projection is its Q4_0 part plus the
correction (8 d + m) x the activation's block sums, added by the persistent
decode kernel, by a correction launch after the skinny product, and folded
into the f16 copies the tensor-core prefill reads.

Greedy decode, steered decode and per-layer captures against the oracle
(which reads the same file's Q8_0 and Q4_1 blocks) at the north-star bars:
logits and captures within 1e-2 max-abs and 1e-3 relative RMS, identical
greedy tokens."""
import numpy as np
import pytest

from frizzle_b200 import capture as C
from frizzle_b200 import synth
from frizzle_b200.edits import Edit, SCALE, SET, ZERO

from test_gpu_model import assert_parity, run_both

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_pinned_path():
    return synth.model_path(synth.TINY_PINNED, 0)


@pytest.fixture(scope="module")
def gemma_pinned_path():
    return synth.model_path(synth.GEMMA3_1B_PINNED, 0)


def test_tiny_pinned_greedy(tiny_pinned_path):
    # 16-row prefill blocks (the skinny products and the correction launch), then the decode kernel.
    assert_parity(run_both(tiny_pinned_path, synth.TINY_PINNED, 21, 12))


def test_tiny_pinned_wide_prefill(tiny_pinned_path):
    # One 40-row step: the Q4_1 layers' f16 copies carry the correction.
    assert_parity(run_both(tiny_pinned_path, synth.TINY_PINNED, 40, 8, block=40))


def test_tiny_pinned_steered(tiny_pinned_path):
    s = synth.TINY_PINNED
    # Edits in a Q4_1 layer (1) and a Q4_0 one (5).
    edits = [Edit(1, 5, SET, 8.0, 0), Edit(1, 100, SCALE, -2.5, 1), Edit(5, 900, ZERO, 0.0, 0, 3)]
    out = run_both(tiny_pinned_path, s, 9, 8, edits=edits)
    assert_parity(out)
    cap, _ = out["cap_layers"]
    neurons = C.Capture(cap, C.layout(s), s.head_dim).neurons(1)
    assert neurons[5] == np.float32(8.0)


def test_gemma_pinned_config1_greedy(gemma_pinned_path):
    assert_parity(run_both(gemma_pinned_path, synth.GEMMA3_1B_PINNED, 32, 32, capture=True))


def test_gemma_pinned_config1_steered(gemma_pinned_path):
    s = synth.GEMMA3_1B_PINNED
    rng = np.random.default_rng(13)
    idx = rng.choice(s.ffn, size=8, replace=False)
    vals = rng.uniform(-10, 10, size=8).astype(np.float32)
    # Layer 2 (Q4_1 down) and layer 13 (Q4_0).
    edits = [Edit(2 if j < 4 else 13, int(i), SET, float(v), 0) for j, (i, v) in enumerate(zip(idx, vals))]
    assert_parity(run_both(gemma_pinned_path, s, 32, 32, edits=edits, capture=True))


def test_gemma_pinned_wide_prefill(gemma_pinned_path):
    # A 64-token prompt in one tensor-core step, then decode.
    assert_parity(run_both(gemma_pinned_path, synth.GEMMA3_1B_PINNED, 64, 4, block=64, capture=False))
