"""The residency plan against the device: a batch created at the plan's
sequences and context takes no more device memory than the plan counts for
its rings and scratch (plus the plan's slack), and a plan over the free
memory offers the trained context (src/core/residency/plan.cpp:373-383)."""
import ctypes as C

import pytest

from frizzle_b200 import _native, engine, synth

pytestmark = pytest.mark.gpu


def test_plan_matches_the_batch_it_sizes(gemma_model_path):
    import torch
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, gemma_model_path)
    lib = model.lib
    p = _native.Plan(sequences=8, context=0, rollback=4096, rows=8 * 16, budget=0)
    _native.check(lib.fz_model_plan(model.handle, C.byref(p)))
    assert p.sequences == 8 and p.context == synth.GEMMA3_1B.context   # 180 GB holds every context
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    batch = engine.Batch(model, p.sequences, p.context)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    used = free0 - free1
    counted = p.cache_bytes + p.scratch_bytes
    assert used <= counted + (64 << 20), (used, counted)
    assert used >= 0.9 * counted, (used, counted)
    # A 1 GiB budget cannot hold even the weights: refused.
    q = _native.Plan(sequences=1, context=0, rollback=4096, rows=0, budget=1 << 30)
    assert lib.fz_model_plan(model.handle, C.byref(q)) == 5
    batch.free()
    model.free()
    dev.close()
