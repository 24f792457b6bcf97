"""Q8_0 and Q4_1 on the CPU: the oracle's unpack pinned to each format's
definition, its product checked against f64, and the entry points' argument
refusals (which return before anything reaches a GPU).

The reference holds no Q8_0 or Q4_1 fixtures (its tests run those formats
only through the real pinned file, which is absent), so the unpack is pinned
to the definition the reference states: Q8_0 weight j = qs[j] * d
(formats/q8_0/q8_0.h:19-21); Q4_1 weight j = (qs[j] & 0xF) * d + m and
weight j + 16 = (qs[j] >> 4) * d + m (formats/q4_1/q4_1.h:20-23), here in
numpy, independently of the C restatement."""
import numpy as np
import pytest

import oracle
from frizzle_b200 import _native, synth


def numpy_q8_0(blocks):
    b = blocks.reshape(-1, 34)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(-1)


def numpy_q4_1(blocks):
    b = blocks.reshape(-1, 20)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    m = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    qs = b[:, 4:]
    q = np.concatenate([qs & 0xF, qs >> 4], axis=1).astype(np.float32)
    return (q * d + m).reshape(-1)


def special_scales(blocks, bytes_per_block, fields):
    """Plants subnormal, zero, negative-zero and extreme scales in the first blocks."""
    b = blocks.reshape(-1, bytes_per_block).copy()
    specials = np.array([0x0001, 0x03FF, 0x0000, 0x8000, 0x7BFF, 0xFBFF, 0x8123], dtype=np.uint16)
    for i, h in enumerate(specials):
        for f in range(fields):
            b[i, 2 * f:2 * f + 2] = np.frombuffer(np.uint16(h ^ (f * 0x8000)).tobytes(), dtype=np.uint8)
    return b.reshape(-1)


def test_q8_0_unpack_is_the_definition():
    blocks = special_scales(synth.random_q8_0(64, 1152, seed=3), 34, 1)
    got = oracle.dequant_fmt(oracle.TYPE_Q8_0, blocks)
    assert np.array_equal(got.view(np.uint32), numpy_q8_0(blocks).view(np.uint32))


def test_q4_1_unpack_is_the_definition():
    blocks = special_scales(synth.random_q4_1(64, 1152, seed=4), 20, 2)
    got = oracle.dequant_fmt(oracle.TYPE_Q4_1, blocks)
    assert np.array_equal(got.view(np.uint32), numpy_q4_1(blocks).view(np.uint32))


def test_q8_0_codes_cover_the_signed_range():
    blocks = synth.random_q8_0(8, 1024, seed=5).reshape(-1, 34).copy()
    blocks[:, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), dtype=np.uint8)
    blocks[0, 2:] = np.arange(-128, -96, dtype=np.int8).view(np.uint8)
    blocks[1, 2:] = np.arange(96, 128, dtype=np.int8).view(np.uint8)
    got = oracle.dequant_fmt(oracle.TYPE_Q8_0, blocks.reshape(-1))
    assert np.array_equal(got[:32], np.arange(-128, -96, dtype=np.float32))
    assert np.array_equal(got[32:64], np.arange(96, 128, dtype=np.float32))


@pytest.mark.parametrize("gguf_type,gen", [(oracle.TYPE_Q8_0, synth.random_q8_0), (oracle.TYPE_Q4_1, synth.random_q4_1),
                                          (oracle.TYPE_Q4_0, synth.random_q4_0)])
def test_format_product_against_f64(gguf_type, gen):
    n, k, m = 96, 1152, 3
    blocks = gen(n, k, seed=6)
    x = np.random.default_rng(7).standard_normal((m, k)).astype(np.float32)
    y = oracle.matmul_fmt(gguf_type, blocks, n, k, x)
    w = oracle.dequant_fmt(gguf_type, blocks).reshape(n, k).astype(np.float64)
    want = x.astype(np.float64) @ w.T
    rel = np.sqrt(np.mean((y - want) ** 2) / np.mean(want ** 2))
    assert rel < 1e-6
    if gguf_type == oracle.TYPE_Q4_0:
        assert np.array_equal(y, oracle.matmul(blocks, n, k, x))


def test_oracle_refuses_unrestated_types():
    with pytest.raises(ValueError):
        oracle.matmul_fmt(1, np.zeros(64, np.uint8), 1, 32, np.zeros(32, np.float32))


def test_format_entry_points_refuse_bad_arguments():
    """Refusals are host-side checks, made before any device work."""
    lib = _native.load()
    fake = 1 << 20  # 16-byte aligned, never dereferenced: every call below is refused first
    for matvec in (lib.fz_q8_0_matvec, lib.fz_q4_1_matvec):
        assert matvec(fake, fake, 64, 1000, fake, 1, fake, None) == 1          # k not a multiple of 32
        assert matvec(fake, fake, 0, 1024, fake, 1, fake, None) == 1           # no rows
        assert matvec(fake, fake, 64, 1024, fake, 9, fake, None) == 1          # m beyond 8
        assert matvec(fake, fake, 64, 1024, fake, 0, fake, None) == 1
        assert matvec(fake + 4, fake, 64, 1024, fake, 1, fake, None) == 1      # codes misaligned
        assert matvec(fake, fake, 64, 1024, fake + 4, 1, fake, None) == 1      # x misaligned
        assert matvec(fake, fake, 64, 8 * 6912, fake, 8, fake, None) == 1      # staged x past 200 KiB
        assert matvec(None, fake, 64, 1024, fake, 1, fake, None) == 1
    assert lib.fz_q8_0_repack(fake + 1, 16, 64, fake, fake, None) == 1
    assert lib.fz_q4_1_repack(fake + 2, 16, 64, fake, fake, None) == 1
    assert lib.fz_q4_1_rows(fake, fake + 2, 16, 64, fake, 1, 1.0, fake, None) == 1
    assert lib.fz_q8_0_rows(fake, fake, 16, 48, fake, 1, 1.0, fake, None) == 1
    assert b"multiple of 32" in lib.fz_last_error()
    assert lib.fz_q8_0_codes_bytes(262144, 1152) == 262144 * 1152
    assert lib.fz_q8_0_scales_bytes(262144, 1152) == 262144 * 36 * 2
    assert lib.fz_q4_1_codes_bytes(1152, 6912) == 1152 * 6912 // 2
    assert lib.fz_q4_1_scales_bytes(1152, 6912) == 1152 * 216 * 4
