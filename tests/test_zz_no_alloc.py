"""fz_attention_static, the attention entry point for callers that cannot
allocate device memory (hosts with no device allocator of their own, or work
that must stay free of allocation), against fz_attention with caller scratch.

Collected last on purpose: a run that stops at the first failure has run every
other test before this one.  It needs nothing from the other tests, so it
also passes alone in a fresh process."""
import numpy as np
import pytest

from frizzle_b200 import _native

pytestmark = pytest.mark.gpu

HEADS, KV, D = 4, 1, 256


def _torch():
    import torch
    assert torch.cuda.is_available(), "the GPU tests need a CUDA device"
    return torch


def _inputs(rows, position, slots, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((rows, HEADS, D)).astype(np.float32)
    kc = (rng.standard_normal((slots, KV, D)) * 0.5).astype(np.float16)
    vc = rng.standard_normal((slots, KV, D)).astype(np.float16)
    return q, kc, vc


def _both(rows, position, window, slots, seed):
    torch = _torch()
    lib = _native.load()
    stream = torch.cuda.current_stream().cuda_stream
    q, kc, vc = _inputs(rows, position, slots, seed)
    qd = torch.from_numpy(q).cuda()
    kd = torch.from_numpy(kc.view(np.int16)).cuda()
    vd = torch.from_numpy(vc.view(np.int16)).cuda()
    splits = lib.fz_attention_splits(window, position, rows)
    po = torch.empty(rows * HEADS * splits * D, dtype=torch.float32, device="cuda")
    pml = torch.empty(rows * HEADS * splits * 2, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(rows * KV, dtype=torch.int32, device="cuda")
    want = torch.empty((rows, HEADS, D), dtype=torch.float32, device="cuda")
    got = torch.full((rows, HEADS, D), float("nan"), dtype=torch.float32, device="cuda")
    _native.check(lib.fz_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), slots, HEADS, KV, D, window, position,
                                   rows, po.data_ptr(), pml.data_ptr(), cnt.data_ptr(), want.data_ptr(), stream))
    _native.check(lib.fz_attention_static(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), slots, HEADS, KV, D, window,
                                          position, rows, got.data_ptr(), stream))
    torch.cuda.synchronize()
    return got.cpu().numpy().astype(np.float64), want.cpu().numpy().astype(np.float64), splits


def _assert_close(got, want):
    # The parity bar the kernel tests use for f32 results.
    rel = np.sqrt(np.mean((got - want) ** 2)) / np.sqrt(np.mean(want ** 2))
    assert np.isfinite(got).all()
    assert rel < 1e-5, rel
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


def test_static_scratch_matches_caller_scratch_twice_in_a_row():
    """Two calls back to back, each spanning several 512-key splits, so the
    second reads scratch the first left behind and must not be affected by it.

    The entry point also clears the shared split counters before each launch.
    A finished launch leaves them at zero already (its last split resets
    them), and no call through the C ABI can leave them otherwise, so this
    test cannot show that the clear itself works: it guards only a launch
    that never finished."""
    got, want, splits = _both(rows=2, position=1500, window=32768, slots=4096, seed=1)
    assert splits == 3
    _assert_close(got, want)
    got, want, splits = _both(rows=4, position=2500, window=32768, slots=4096, seed=2)
    assert splits == 5
    _assert_close(got, want)


def test_static_scratch_single_split():
    # Every row's keys fit one 512-key split: no partials, no counters.
    got, want, splits = _both(rows=3, position=200, window=512, slots=1024, seed=3)
    assert splits == 1
    _assert_close(got, want)


def test_static_scratch_refuses_calls_past_its_limit():
    torch = _torch()
    lib = _native.load()
    q = torch.zeros((16, HEADS, D), dtype=torch.float32, device="cuda")
    cache = torch.zeros((32768, KV, D), dtype=torch.int16, device="cuda")
    out = torch.zeros_like(q)
    # 16 rows x 4 heads x 63 splits = 4032 partials, above the 2048 the array holds.
    st = lib.fz_attention_static(q.data_ptr(), cache.data_ptr(), cache.data_ptr(), 32768, HEADS, KV, D, 32768, 32000,
                                 16, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 1
    assert b"FZ_ATTENTION_STATIC_MAX_PARTIALS" in lib.fz_last_error()


def test_static_scratch_refuses_counters_and_group_sizes_past_its_limits():
    torch = _torch()
    lib = _native.load()
    stream = torch.cuda.current_stream().cuda_stream
    rows = 129   # 129 x 1 KV head split counters, above the 128 the array holds (partials: 129 x 4 x 1)
    q = torch.zeros((rows, HEADS, D), dtype=torch.float32, device="cuda")
    cache = torch.zeros((1024, KV, D), dtype=torch.int16, device="cuda")
    out = torch.zeros_like(q)
    st = lib.fz_attention_static(q.data_ptr(), cache.data_ptr(), cache.data_ptr(), 1024, HEADS, KV, D, 256, 0, rows,
                                 out.data_ptr(), stream)
    assert st == 1
    assert b"FZ_ATTENTION_STATIC_MAX_COUNTERS" in lib.fz_last_error()
    # Three query heads a KV head: no kernel takes that grouping, refused before any launch.
    q3 = torch.zeros((1, 3, D), dtype=torch.float32, device="cuda")
    st = lib.fz_attention_static(q3.data_ptr(), cache.data_ptr(), cache.data_ptr(), 1024, 3, 1, D, 256, 10, 1,
                                 q3.data_ptr(), stream)
    assert st == 1
    assert b"1, 2, 4 or 8" in lib.fz_last_error()
    torch.cuda.synchronize()
