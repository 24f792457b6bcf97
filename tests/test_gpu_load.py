"""The streaming load (Upload::begin/write/finish with the PieceWriter's
repack, src/core/residency/upload.h:263-337 and piece_writer.h:165-245): the
file's bytes arrive in order in chunks of any size, each Q4_0 matrix is
repacked a 16-row group at a time from a bounded 32 MiB device stage as soon
as a group is whole, and no copy of the whole file is staged on the device."""
import os

import numpy as np
import pytest

from frizzle_b200 import _native, engine, synth

pytestmark = pytest.mark.gpu

STAGE = 32 << 20


def _load(dev, path, chunk):
    m = engine.Model(dev)
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        head = f.read(min(size, 8 << 20))
    m.begin_load(head, size)
    data = np.memmap(path, dtype=np.uint8, mode="r")
    for off in range(0, size, chunk):
        part = np.ascontiguousarray(data[off:off + chunk])
        _native.check(m.lib.fz_model_load_write(m.handle, off, part.ctypes.data, part.size))
    m.finish_load()
    return m


def _logits(model, ids):
    b = engine.Batch(model, 1, 256)
    b.step(0, ids, tokens=len(ids), logits=True)
    out = b.logits(0)
    b.wait()
    b.free()
    return out


def test_odd_chunks_give_the_same_model(tiny_model_path):
    dev = engine.Device(0)
    ids = np.random.default_rng(2).integers(2, synth.TINY.vocab, size=7).astype(np.uint32)
    ref = engine.Model.from_file(dev, tiny_model_path)
    want = _logits(ref, ids)
    ref.free()
    # 1,000,003 bytes: chunks end inside blocks, rows and row groups; 4099: many chunks a row group.
    for chunk in (1_000_003, 4099):
        m = _load(dev, tiny_model_path, chunk)
        got = _logits(m, ids)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), chunk
        m.free()
    dev.close()


def test_chunks_out_of_order_or_missing_are_refused(tiny_model_path):
    dev = engine.Device(0)
    size = os.path.getsize(tiny_model_path)
    data = np.memmap(tiny_model_path, dtype=np.uint8, mode="r")
    m = engine.Model(dev)
    m.begin_load(bytes(data[:8 << 20]), size)
    part = np.ascontiguousarray(data[:1 << 20])
    _native.check(m.lib.fz_model_load_write(m.handle, 0, part.ctypes.data, part.size))
    skip = np.ascontiguousarray(data[2 << 20:3 << 20])
    assert m.lib.fz_model_load_write(m.handle, 2 << 20, skip.ctypes.data, skip.size) == 6   # FZ_ERR_UPLOAD
    assert b"in order" in m.lib.fz_last_error()
    assert m.lib.fz_model_load_finish(m.handle) == 6
    assert b"was not written" in m.lib.fz_last_error()
    m.free()
    dev.close()


def test_load_holds_no_whole_file_copy(gemma_model_path):
    """Device memory at the end of begin_load is the final buffers and the
    stage; the chunks then add nothing: the peak is the loaded model's bytes
    plus the 32 MiB stage, not plus the file's 0.57 GB."""
    import torch
    dev = engine.Device(0)
    size = os.path.getsize(gemma_model_path)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    m = engine.Model(dev)
    with open(gemma_model_path, "rb") as f:
        head = f.read(8 << 20)
    m.begin_load(head, size)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    data = np.memmap(gemma_model_path, dtype=np.uint8, mode="r")
    low = free1
    for off in range(0, size, 64 << 20):
        part = np.ascontiguousarray(data[off:off + (64 << 20)])
        _native.check(m.lib.fz_model_load_write(m.handle, off, part.ctypes.data, part.size))
        low = min(low, torch.cuda.mem_get_info()[0])
    m.finish_load()
    torch.cuda.synchronize()
    free2, _ = torch.cuda.mem_get_info()
    placed = free0 - free1
    assert free1 - low < 64 << 20, (free1 - low)          # the chunks allocate nothing
    assert 0 <= (free0 - free2) <= placed                  # finish frees the stage
    assert placed - (free0 - free2) >= STAGE - (2 << 20)
    m.free()
    dev.close()
