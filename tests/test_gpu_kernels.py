"""Kernel-level parity through the C ABI on the GPU: each hot kernel against the
CPU oracle on the same seeded inputs (BASELINE config 2's Q4_0 sweep shapes).

Bars: the Q4_0 decode and repack bit-exact; products within 1e-5 relative RMS
and 1e-4 x max|y| of the oracle's f32 (the hi/lo split keeps them f32-exact
to ~2^-22; the sum order differs from the reference's 32 ranges); argmax
identical to the argmax of the kernel's own logits."""
import ctypes as C

import numpy as np
import pytest

import oracle
from frizzle_b200 import _native, synth
from frizzle_b200.edits import Edit, check, table, SET, SCALE, ZERO

pytestmark = pytest.mark.gpu

SHAPES = [(1152, 1024), (1152, 256), (1024, 1152), (1152, 6912), (6912, 1152)]  # (K, N)


def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "the GPU tests need a CUDA device"
    return torch


def dev(arr):
    torch = torch_cuda()
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def stream():
    return torch_cuda().cuda.current_stream().cuda_stream


def repacked(blocks, n, k):
    torch = torch_cuda()
    lib = _native.load()
    src = dev(blocks)
    codes = torch.empty(lib.fz_q4_0_codes_bytes(n, k), dtype=torch.uint8, device="cuda")
    scales = torch.empty(lib.fz_q4_0_scales_bytes(n, k), dtype=torch.uint8, device="cuda")
    _native.check(lib.fz_q4_0_repack(src.data_ptr(), n, k, codes.data_ptr(), scales.data_ptr(), stream()))
    return codes, scales


def test_repack_and_rows_bit_exact():
    torch = torch_cuda()
    lib = _native.load()
    n, k = 96, 1152
    blocks = synth.random_q4_0(n, k, seed=11)
    codes, scales = repacked(blocks, n, k)
    rows = dev(np.arange(n, dtype=np.uint32).astype(np.int32)).to(torch.int32)
    out = torch.empty(n * k, dtype=torch.float32, device="cuda")
    _native.check(lib.fz_q4_0_rows(codes.data_ptr(), scales.data_ptr(), n, k, rows.data_ptr(), n, 1.0,
                                   out.data_ptr(), stream()))
    got = out.cpu().numpy()
    want = oracle.dequant(blocks)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # And the gather's scaling: (code - 8) * d, then * sqrt(width), in f32.
    s = np.float32(np.sqrt(np.float32(k)))
    _native.check(lib.fz_q4_0_rows(codes.data_ptr(), scales.data_ptr(), n, k, rows.data_ptr(), n, float(s),
                                   out.data_ptr(), stream()))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), (want * s).view(np.uint32))


@pytest.mark.parametrize("k,n", SHAPES)
@pytest.mark.parametrize("m", [1, 4, 8, 16])
def test_matvec_sweep_shapes(k, n, m):
    torch = torch_cuda()
    lib = _native.load()
    blocks = synth.random_q4_0(n, k, seed=k * 7 + n)
    x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    codes, scales = repacked(blocks, n, k)
    xd = dev(x)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    _native.check(lib.fz_q4_0_matvec(codes.data_ptr(), scales.data_ptr(), n, k, xd.data_ptr(), m, y.data_ptr(),
                                     stream()))
    got = y.cpu().numpy()
    want = oracle.matmul(blocks, n, k, x)
    err = np.sqrt(np.mean((got.astype(np.float64) - want) ** 2)) / np.sqrt(np.mean(want.astype(np.float64) ** 2))
    assert err < 1e-5
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


def test_head_shape_and_argmax():
    torch = torch_cuda()
    lib = _native.load()
    n, k = 262144, 1152
    blocks = synth.random_q4_0(n, k, seed=5)
    codes, scales = repacked(blocks, n, k)
    x = np.random.default_rng(3).standard_normal((2, k)).astype(np.float32)
    xd = dev(x)
    logits = torch.empty((2, n), dtype=torch.float32, device="cuda")
    am = torch.zeros(2, dtype=torch.int64, device="cuda")
    _native.check(lib.fz_q4_0_head(codes.data_ptr(), scales.data_ptr(), n, k, xd.data_ptr(), 2, logits.data_ptr(),
                                   am.data_ptr(), stream()))
    got = logits.cpu().numpy()
    want = oracle.matmul(blocks, n, k, x)
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
    packed = am.cpu().numpy().view(np.uint64)
    for r in range(2):
        token = 0xFFFFFFFF - int(packed[r] & 0xFFFFFFFF)
        assert token == int(np.argmax(got[r]))


@pytest.mark.parametrize("m,position", [(5, 36), (5, 40), (1, 45), (1, 46), (16, 30)])
def test_gated_with_edits(m, position):
    torch = torch_cuda()
    lib = _native.load()
    f, k = 6912, 1152
    gate = synth.random_q4_0(f, k, seed=1)
    up = synth.random_q4_0(f, k, seed=2)
    x = np.random.default_rng(4).standard_normal((m, k)).astype(np.float32) * np.float32(0.05)
    gc, gs = repacked(gate, f, k)
    uc, us = repacked(up, f, k)
    edits = [Edit(1, n, [SET, SCALE, ZERO][n % 3], [n * 0.5, -1.75, 0.0][n % 3], 0, 6) for n in range(10, 160)]
    edits += [Edit(1, 7, SCALE, 1.0, 0, 6), Edit(1, 6911, SET, 10.0, 2, 4), Edit(0, 3, SET, 999.0, 0)]
    assert check(edits, 3, f).ok
    words = np.array(table(edits, 3, 40), dtype=np.uint32)
    td = dev(words.view(np.int32))
    xd = dev(x)
    act = torch.empty((m, f), dtype=torch.float32, device="cuda")
    _native.check(lib.fz_q4_0_gated(gc.data_ptr(), gs.data_ptr(), uc.data_ptr(), us.data_ptr(), f, k, xd.data_ptr(),
                                    m, td.data_ptr(), 1, position, act.data_ptr(), stream()))
    got = act.cpu().numpy()
    want = oracle.edit_apply(words, 1, position, oracle.gated(gate, up, f, k, x))
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
    # Set and Zero edits land exactly.
    for e in edits:
        if e.layer == 1 and e.kind in (SET, ZERO):
            for r in range(m):
                if 40 + e.start <= position + r < 40 + e.until:
                    assert got[r, e.neuron] == np.float32(e.value)


ATTN_CASES = [
    # (rows, position, window, slots): decode and prefill rows, one and several 512-key splits,
    # a sliding window, and a ring smaller than the positions (keys at slot j mod slots).
    (1, 35, 512, 5120),
    (1, 1500, 32768, 4096),
    (4, 1020, 32768, 2048),
    (16, 100, 16, 48),
    (1, 3000, 512, 1100),
    (2, 5000, 32768, 8192),
]


@pytest.mark.parametrize("rows,position,window,slots", ATTN_CASES)
def test_attention_vs_oracle(rows, position, window, slots):
    torch = torch_cuda()
    lib = _native.load()
    heads, kv, d = 4, 1, 256
    rng = np.random.default_rng([rows, position, window])
    q = rng.standard_normal((rows, heads, d)).astype(np.float32)
    kc = (rng.standard_normal((slots, kv, d)) * 0.5).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((slots, kv, d)).astype(np.float16).view(np.uint16)
    scale = float(np.float32(np.float64(np.float32(1.0) / np.sqrt(np.float32(d))) * 1.4426950408889634))
    want = oracle.attention(q, kc, vc, slots, kv, window, scale, position)
    splits = lib.fz_attention_splits(window, position, rows)
    qd, kd, vd = dev(q), dev(kc.view(np.int16)), dev(vc.view(np.int16))
    po = torch.empty(rows * heads * splits * d, dtype=torch.float32, device="cuda")
    pml = torch.empty(rows * heads * splits * 2, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(rows * kv, dtype=torch.int32, device="cuda")
    out = torch.empty((rows, heads, d), dtype=torch.float32, device="cuda")
    _native.check(lib.fz_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), slots, heads, kv, d, window, position,
                                   rows, po.data_ptr(), pml.data_ptr(), cnt.data_ptr(), out.data_ptr(), stream()))
    got = out.cpu().numpy()
    err = np.sqrt(np.mean((got.astype(np.float64) - want) ** 2)) / np.sqrt(np.mean(want.astype(np.float64) ** 2))
    assert err < 1e-5, err
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()
    assert int(cnt.abs().sum()) == 0  # the counters are left at zero for the next launch


WIDE_CASES = [
    # (heads, kv_heads, rows, position, window, slots)
    (4, 1, 1600, 0, 32768, 2048),    # 50 blocks of 32 tokens: those of more than 40 key tiles split
    (4, 1, 300, 1000, 32768, 2048),  # a later step: its blocks start past position 1000
    (8, 1, 1400, 0, 32768, 2048),    # 16-token blocks
    (4, 2, 1500, 0, 32768, 2048),    # two KV heads, 64-token blocks
    (4, 1, 700, 1900, 512, 1024),    # a window layer over a ring (key j at slot j mod 1024): never split
]
_WIDE_WANT = {}


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("heads,kv,rows,position,window,slots", WIDE_CASES)
def test_attention_wide_vs_oracle(heads, kv, rows, position, window, slots, split):
    """The tensor-core attention (fz_attention_wide) on every row against the
    oracle, whole blocks and, with split scratch, long blocks whose two halves
    of keys run on two CTAs and merge."""
    torch = torch_cuda()
    lib = _native.load()
    d = 256
    rng = np.random.default_rng([heads, kv, rows, position])
    q = rng.standard_normal((rows, heads, d)).astype(np.float32)
    kc = (rng.standard_normal((slots, kv, d)) * 0.5).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((slots, kv, d)).astype(np.float16).view(np.uint16)
    scale = float(np.float32(np.float64(np.float32(1.0) / np.sqrt(np.float32(d))) * 1.4426950408889634))
    key = (heads, kv, rows, position, window, slots)
    if key not in _WIDE_WANT:
        _WIDE_WANT[key] = oracle.attention(q, kc, vc, slots, kv, window, scale, position)
    want = _WIDE_WANT[key]
    qd, kd, vd = dev(q), dev(kc.view(np.int16)), dev(vc.view(np.int16))
    maps = torch.zeros(64, dtype=torch.int32, device="cuda")   # 256 bytes (torch aligns to 256)
    part = torch.empty(148 * 2 * 258 * 128, dtype=torch.float32, device="cuda") if split else None
    cnt = torch.zeros(148, dtype=torch.int32, device="cuda")
    err_word = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full((rows, heads, d), float("nan"), dtype=torch.float32, device="cuda")
    _native.check(lib.fz_attention_wide(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), slots, heads, kv, d, window,
                                        position, rows, maps.data_ptr(), part.data_ptr() if split else None,
                                        cnt.data_ptr(), out.data_ptr(), err_word.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert int(err_word.item()) == 0
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    err = np.sqrt(np.mean((got.astype(np.float64) - want) ** 2)) / np.sqrt(np.mean(want.astype(np.float64) ** 2))
    print(f"wide attention {key} split={split} rel_rms={err:.3e}")
    assert err < 1e-4, err
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()
    assert int(cnt.abs().sum()) == 0  # the split counters are left at zero for the next launch


def split_dev(x):
    torch = torch_cuda()
    lib = _native.load()
    xd = dev(x)
    hi = torch.empty(x.shape, dtype=torch.float16, device="cuda")
    lo = torch.empty(x.shape, dtype=torch.float16, device="cuda")
    _native.check(lib.fz_split_f16(xd.data_ptr(), x.size, hi.data_ptr(), lo.data_ptr(), stream()))
    return hi, lo


GEMM_SHAPES = [(1152, 1536), (1024, 1152), (6912, 1152), (1152, 6912)]  # (K, N)


@pytest.mark.parametrize("k,n", GEMM_SHAPES)
@pytest.mark.parametrize("m", [64, 200, 512])
@pytest.mark.parametrize("passes", [1, 2, 3])
def test_tensor_core_gemm(k, n, m, passes):
    """The tcgen05 product against the oracle's f32.  One pass: X and the
    weights each rounded once to f16.  Two: X as f16 hi + lo, the weights
    rounded once (two MMAs).  Three: the weights as hi + lo too (three MMAs):
    f32-level, within the tensor core's own f32 accumulation (about 4e-6
    relative at K = 1152, 2.3e-5 at K = 6912)."""
    torch = torch_cuda()
    lib = _native.load()
    blocks = synth.random_q4_0(n, k, seed=k + n)
    x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    codes, scales = repacked(blocks, n, k)
    hi, lo = split_dev(x)
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _native.check(lib.fz_q4_0_gemm(codes.data_ptr(), scales.data_ptr(), n, k, hi.data_ptr(),
                                   lo.data_ptr() if passes >= 2 else None, 1 if passes == 3 else 0, m, y.data_ptr(),
                                   err.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = y.cpu().numpy()
    want = oracle.matmul(blocks, n, k, x)
    rel = np.sqrt(np.mean((got.astype(np.float64) - want) ** 2)) / np.sqrt(np.mean(want.astype(np.float64) ** 2))
    print(f"gemm k={k} n={n} m={m} passes={passes} rel_rms={rel:.3e}")
    assert np.isfinite(got).all()
    assert rel < {1: 1e-3, 2: 5e-4, 3: 5e-5}[passes], rel


@pytest.mark.parametrize("m,position", [(128, 30), (300, 0)])
def test_tensor_core_gated_with_edits(m, position):
    torch = torch_cuda()
    lib = _native.load()
    f, k = 6912, 1152
    gate = synth.random_q4_0(f, k, seed=1)
    up = synth.random_q4_0(f, k, seed=2)
    x = np.random.default_rng(4).standard_normal((m, k)).astype(np.float32) * np.float32(0.05)
    gc, gs = repacked(gate, f, k)
    uc, us = repacked(up, f, k)
    edits = [Edit(1, nn, [SET, SCALE, ZERO][nn % 3], [nn * 0.5, -1.75, 0.0][nn % 3], 0, 6) for nn in range(10, 160)]
    edits += [Edit(1, 7, SCALE, 1.0, 0, 6), Edit(1, 6911, SET, 10.0, 2, 4), Edit(0, 3, SET, 999.0, 0)]
    words = np.array(table(edits, 3, 40), dtype=np.uint32)
    td = dev(words.view(np.int32))
    hi, lo = split_dev(x)
    act = torch.empty((m, f), dtype=torch.float32, device="cuda")
    ahi = torch.empty((m, f), dtype=torch.float16, device="cuda")
    alo = torch.empty((m, f), dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _native.check(lib.fz_q4_0_gemm_gated(gc.data_ptr(), gs.data_ptr(), uc.data_ptr(), us.data_ptr(), f, k,
                                         hi.data_ptr(), lo.data_ptr(), 1, m, td.data_ptr(), 1, position, act.data_ptr(),
                                         ahi.data_ptr(), alo.data_ptr(), err.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = act.cpu().numpy()
    want = oracle.edit_apply(words, 1, position, oracle.gated(gate, up, f, k, x))
    rel = np.sqrt(np.mean((got.astype(np.float64) - want) ** 2)) / np.sqrt(np.mean(want.astype(np.float64) ** 2))
    assert rel < 1e-5, rel
    split = ahi.float().cpu().numpy() + alo.float().cpu().numpy()
    assert np.abs(split - got).max() <= 1e-6 * max(1.0, np.abs(got).max())
    for e in edits:
        if e.layer == 1 and e.kind in (SET, ZERO):
            for r in range(m):
                if 40 + e.start <= position + r < 40 + e.until:
                    assert got[r, e.neuron] == np.float32(e.value)


@pytest.mark.parametrize("k,n", [(1152, 1536), (6912, 1152)])
def test_q4_0_to_f16_split_is_exact(k, n):
    """fz_q4_0_to_f16: hi = f16 of (code - 8) d, lo = the f16 remainder; hi + lo
    is the exact product (in f64) wherever the remainder is a normal f16."""
    torch = torch_cuda()
    lib = _native.load()
    blocks = synth.random_q4_0(n, k, seed=n + 3)
    codes, scales = repacked(blocks, n, k)
    hi = torch.empty((n, k), dtype=torch.float16, device="cuda")
    lo = torch.empty((n, k), dtype=torch.float16, device="cuda")
    _native.check(lib.fz_q4_0_to_f16(codes.data_ptr(), scales.data_ptr(), n, k, hi.data_ptr(), lo.data_ptr(),
                                     stream()))
    torch.cuda.synchronize()
    want = oracle.dequant(blocks).reshape(n, k).astype(np.float64)
    h = hi.cpu().numpy().astype(np.float64)
    lo_ = lo.cpu().numpy().astype(np.float64)
    assert np.array_equal(h, want.astype(np.float16).astype(np.float64))
    err = np.abs(h + lo_ - want)
    assert err.max() <= 2.0 ** -24 * max(1.0, np.abs(want).max()), err.max()


@pytest.mark.parametrize("passes", [1, 2, 3])
@pytest.mark.parametrize("m", [64, 300])
def test_f16_weight_gemm(m, passes):
    """The tensor-core product with the weight tiles by TMA from f16 copies:
    the same tolerances as the in-kernel dequant path."""
    torch = torch_cuda()
    lib = _native.load()
    k, n = 1152, 6912
    blocks = synth.random_q4_0(n, k, seed=77)
    codes, scales = repacked(blocks, n, k)
    whi = torch.empty((n, k), dtype=torch.float16, device="cuda")
    wlo = torch.empty((n, k), dtype=torch.float16, device="cuda")
    _native.check(lib.fz_q4_0_to_f16(codes.data_ptr(), scales.data_ptr(), n, k, whi.data_ptr(), wlo.data_ptr(),
                                     stream()))
    x = np.random.default_rng(m + 1).standard_normal((m, k)).astype(np.float32)
    hi, lo = split_dev(x)
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _native.check(lib.fz_f16_gemm(whi.data_ptr(), wlo.data_ptr() if passes == 3 else None, n, k, hi.data_ptr(),
                                  lo.data_ptr() if passes >= 2 else None, 1 if passes == 3 else 0, m, y.data_ptr(),
                                  err.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = y.cpu().numpy()
    want = oracle.matmul(blocks, n, k, x)
    rel = np.sqrt(np.mean((got.astype(np.float64) - want) ** 2)) / np.sqrt(np.mean(want.astype(np.float64) ** 2))
    assert np.isfinite(got).all()
    assert rel < {1: 1e-3, 2: 5e-4, 3: 5e-5}[passes], rel


def test_f16_weight_gated_with_edits():
    torch = torch_cuda()
    lib = _native.load()
    m, position, f, k = 200, 7, 6912, 1152
    gate = synth.random_q4_0(f, k, seed=1)
    up = synth.random_q4_0(f, k, seed=2)
    x = np.random.default_rng(5).standard_normal((m, k)).astype(np.float32) * np.float32(0.05)
    mats = []
    for b in (gate, up):
        c, s = repacked(b, f, k)
        whi = torch.empty((f, k), dtype=torch.float16, device="cuda")
        wlo = torch.empty((f, k), dtype=torch.float16, device="cuda")
        _native.check(lib.fz_q4_0_to_f16(c.data_ptr(), s.data_ptr(), f, k, whi.data_ptr(), wlo.data_ptr(), stream()))
        mats.append((whi, wlo))
    edits = [Edit(1, nn, [SET, SCALE, ZERO][nn % 3], [nn * 0.5, -1.75, 0.0][nn % 3], 0, 6) for nn in range(10, 90)]
    words = np.array(table(edits, 3, 40), dtype=np.uint32)
    td = dev(words.view(np.int32))
    hi, lo = split_dev(x)
    act = torch.empty((m, f), dtype=torch.float32, device="cuda")
    ahi = torch.empty((m, f), dtype=torch.float16, device="cuda")
    alo = torch.empty((m, f), dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    (ghi, glo), (uhi, ulo) = mats
    _native.check(lib.fz_f16_gemm_gated(ghi.data_ptr(), glo.data_ptr(), uhi.data_ptr(), ulo.data_ptr(), f, k,
                                        hi.data_ptr(), lo.data_ptr(), 1, m, td.data_ptr(), 1, position,
                                        act.data_ptr(), ahi.data_ptr(), alo.data_ptr(), err.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = act.cpu().numpy()
    want = oracle.edit_apply(words, 1, position, oracle.gated(gate, up, f, k, x))
    rel = np.sqrt(np.mean((got.astype(np.float64) - want) ** 2)) / np.sqrt(np.mean(want.astype(np.float64) ** 2))
    assert rel < 1e-5, rel
