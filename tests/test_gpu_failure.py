"""The decode step's failure path on the GPU, without a fault: a bounded wait
that runs out reports the step as failed, and the next step runs normally
(ProgramError::Step / TurnFailure, src/core/kernels/program.cpp:621-625 and
src/core/runtime/turn.h:108-113).

The wait is made to run out by the batch's test hook: the QKV products are
published under the previous step's epoch, so the attention polls for words
that never arrive.  With a 1 ms limit the attention gives up, every other CTA
sees the error word in its own bounded waits, and the kernel returns by
itself; nothing traps, faults or hangs."""
import numpy as np
import pytest

import oracle
from frizzle_b200 import _native, engine, synth

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_fails_the_step_and_the_next_step_recovers(tiny_model_path):
    dev = engine.Device(0)
    model = engine.Model.from_file(dev, tiny_model_path)
    batch = engine.Batch(model, 1, 256)
    orc = oracle.OracleModel(tiny_model_path, context=256)
    lib = batch.lib
    ids = np.random.default_rng(5).integers(2, synth.TINY.vocab, size=9).astype(np.uint32)
    batch.step(0, ids, tokens=9, logits=True)
    want, _ = orc.step(0, ids, logits=True)
    tok = batch.tokens()[0]
    assert tok == int(np.argmax(want))

    # A one-token step whose QKV words never carry its epoch: its waits give up after 1 ms.
    _native.check(lib.fz_batch_set_wait_limit(batch.handle, 1000))
    _native.check(lib.fz_batch_inject_stale_epoch(batch.handle, 1))
    batch.step(9, np.array([tok], dtype=np.uint32), tokens=1, logits=True)
    with pytest.raises(_native.FzError) as failed:
        batch.wait()
    assert failed.value.status == 2, failed.value
    message = lib.fz_last_error().decode()
    assert "gave up" in message and "phase's wait for another phase's output" in message, message

    # Out of range limits are refused; the default limit and epochs come back.
    assert lib.fz_batch_set_wait_limit(batch.handle, 50) == 1
    _native.check(lib.fz_batch_inject_stale_epoch(batch.handle, 0))
    _native.check(lib.fz_batch_set_wait_limit(batch.handle, 0))

    # The failed step's position again, from the cache's last good length: the oracle's token.
    assert batch.truncate(9) == 9
    batch.step(9, np.array([tok], dtype=np.uint32), tokens=1, logits=True)
    want, _ = orc.step(9, [tok], logits=True)
    got = batch.tokens()[0]
    logits = batch.logits(0).astype(np.float64)
    rel = float(np.sqrt(np.mean((logits - want) ** 2) / np.mean(want.astype(np.float64) ** 2)))
    assert got == int(np.argmax(want)) and rel < 1e-3, (got, int(np.argmax(want)), rel)
    # And one more ordinary fed step after it.
    batch.step(10, fed=True, tokens=1, logits=True)
    want, _ = orc.step(10, [got], logits=True)
    assert batch.tokens()[0] == int(np.argmax(want))
    orc.close()
    batch.free()
    model.free()
    dev.close()
