"""The oracle's pins: known-answer vectors and independent implementations.

- Philox4x32-10 against the Random123 known-answer vectors (the published
  algorithm the draw restates, draw.wgsl:48-60).
- f16 decode and round-to-nearest-even encode against numpy's IEEE float16,
  over every half and edge values (unpack2x16float / pack2x16float).
- Q4_0 decode against an independent numpy decode, subnormal scales included.
- The GELU and e^x restatements against the closed forms.
- The Q4_0 matmul against float64.
"""
import math

import numpy as np
import pytest

import oracle
from frizzle_b200 import synth


def test_philox_random123_known_answers():
    assert list(oracle.philox([0, 0, 0, 0], [0, 0])) == [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]
    assert list(oracle.philox([0xffffffff] * 4, [0xffffffff] * 2)) == [0x408f276d, 0x41c83b0e, 0xa20bc7c6,
                                                                       0x6d5451fd]
    assert list(oracle.philox([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0])) == [
        0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]


def test_f16_decode_every_half():
    L = oracle.lib()
    halves = np.arange(65536, dtype=np.uint16)
    want = halves.view(np.float16).astype(np.float32)
    got = np.array([L.oracle_f16_to_f32(int(h)) for h in halves], dtype=np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(want)]))


def test_f16_encode_round_to_nearest_even():
    L = oracle.lib()
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(3.0),
        (rng.standard_normal(20000) * 1e-5).astype(np.float32),        # subnormal halves
        (rng.standard_normal(5000) * 3e4).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 5.960464477539063e-08, 2.9802322387695312e-08,
                  2.98023224e-08, 6.103515625e-05, 6.1e-05, 1.0009765625, 1.00048828125], dtype=np.float32),
    ])
    got = np.array([L.oracle_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_f16_pack_saturates():
    L = oracle.lib()
    assert L.oracle_f16_pack(1e6) == 0x7BFF
    assert L.oracle_f16_pack(-1e6) == 0xFBFF
    assert L.oracle_f16_pack(65519.0) == 0x7BFF


def test_q4_0_decode_matches_independent_numpy():
    blocks = synth.random_q4_0(64, 1152, seed=3)
    d = blocks.reshape(-1, 18)[:, :2].copy().view(np.float16)
    assert (np.abs(d.astype(np.float32)) < 6.1e-5).any(), "the sweep's scales include subnormal halves"
    got = oracle.dequant(blocks)
    want = synth.dequantize_q4_0(blocks)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q4_0_quantizer_round_trips_codes():
    rng = np.random.default_rng(5)
    x = rng.standard_normal(32 * 1000).astype(np.float32) * np.float32(0.02)
    blocks = synth.quantize_q4_0(x)
    w = synth.dequantize_q4_0(blocks).reshape(-1, 32)
    b = x.reshape(-1, 32)
    d = np.abs(blocks.reshape(-1, 18)[:, :2].copy().view(np.float16).astype(np.float32))
    # Each weight within one step of its value (codes clamped at 15 can be a step off).
    assert np.all(np.abs(w - b) <= d * 1.0 + 1e-6)


def test_gelu_and_exp_restatements():
    L = oracle.lib()
    for x in np.linspace(-30, 0, 301):
        assert L.oracle_exp_nonpositive(float(x)) == pytest.approx(math.exp(x), rel=1e-6, abs=1e-38)
    for g in np.linspace(-6, 6, 241):
        want = 0.5 * g * (1 + math.tanh(math.sqrt(2 / math.pi) * (g + 0.044715 * g ** 3)))
        assert L.oracle_gelu(float(g)) == pytest.approx(want, rel=1e-5, abs=2e-7)


@pytest.mark.parametrize("n,k", [(64, 1152), (32, 6912), (48, 1024)])
def test_matmul_against_float64(n, k):
    W = synth.random_q4_0(n, k, seed=7)
    x = np.random.default_rng(9).standard_normal((3, k)).astype(np.float32)
    y = oracle.matmul(W, n, k, x)
    ref = x.astype(np.float64) @ oracle.dequant(W).reshape(n, k).astype(np.float64).T
    assert np.abs(y - ref).max() <= 2e-6 * np.abs(ref).max()


def test_topk_order_and_ties():
    logits = np.zeros(300, dtype=np.float32)
    logits[[5, 9, 200]] = 3.0
    logits[7] = np.float32("nan")
    logits[8] = -0.0
    pairs = oracle.topk64(logits)
    ids = pairs[1::2]
    assert ids[0] == 7                       # NaN first
    assert list(ids[1:4]) == [5, 9, 200]     # ties to the lower id
    assert pairs[0] == 0x7FC00000
    assert 8 in list(ids)                    # -0 ties with +0 and is kept by id order
