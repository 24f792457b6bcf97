"""Other head groupings than Gemma 3 1B's (4 query heads on 1 KV head): 8 on
1, 2 on 1, 2 on each of 2 KV heads, 1 on each of 4, on 3-layer models of the
tiny shape.  A 40-token prompt in one step runs the wide path (the tcgen05
attention with G = 128 / 8, 64 or 128 tokens a CTA and one CTA column a KV
head), then greedy decode (the persistent decode kernel for G = 1, 2, 4; the
per-operation launches for G = 8), against the oracle at the north-star
bars."""
from dataclasses import replace

import pytest

from frizzle_b200 import synth

from test_gpu_model import assert_parity, run_both

pytestmark = pytest.mark.gpu

BASE = replace(synth.TINY, layers=3, pattern=3)


@pytest.mark.parametrize("heads,kv_heads", [(8, 1), (2, 1), (4, 2), (4, 4)])
def test_head_groups_wide_prefill_and_decode(heads, kv_heads):
    shape = replace(BASE, heads=heads, kv_heads=kv_heads)
    path = synth.model_path(shape, 0)
    assert_parity(run_both(path, shape, 40, 6, block=40, capture=False))


@pytest.mark.parametrize("heads,kv_heads", [(4, 2), (8, 1)])
def test_head_groups_chunked_prompt(heads, kv_heads):
    # 70 tokens in 24-token steps: later steps read earlier keys from the cache
    # (the window layers over a sliding range, the global layer over all).
    shape = replace(BASE, heads=heads, kv_heads=kv_heads)
    path = synth.model_path(shape, 0)
    assert_parity(run_both(path, shape, 70, 4, block=24, capture=False))
