"""Q8_0 and Q4_1 kernels through the C ABI on the GPU, against the CPU oracle
on the same seeded blocks: the repacked streams are the file's fields moved
whole, the gather is bit-exact, and the product is within 1e-5 relative RMS
and 1e-4 x max|y| of the oracle's f32 (the kernel takes x as three 8-bit
digit planes a 32-column block, exact integer products with the codes, and
one f32 combination a chunk: about 6e-8 of a block's largest |x| lost, and
another order of sums than the reference's 32 ranges)."""
import numpy as np
import pytest

import oracle
from frizzle_b200 import _native, synth

pytestmark = pytest.mark.gpu

FORMATS = {
    "q8_0": (oracle.TYPE_Q8_0, synth.random_q8_0, 34, "fz_q8_0"),
    "q4_1": (oracle.TYPE_Q4_1, synth.random_q4_1, 20, "fz_q4_1"),
}


def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "the GPU tests need a CUDA device"
    return torch


def stream():
    return torch_cuda().cuda.current_stream().cuda_stream


def fn(fmt, name):
    return getattr(_native.load(), f"{FORMATS[fmt][3]}_{name}")


def repacked(fmt, blocks, n, k):
    torch = torch_cuda()
    src = torch.from_numpy(np.ascontiguousarray(blocks)).cuda()
    codes = torch.empty(fn(fmt, "codes_bytes")(n, k), dtype=torch.uint8, device="cuda")
    scales = torch.empty(fn(fmt, "scales_bytes")(n, k), dtype=torch.uint8, device="cuda")
    _native.check(fn(fmt, "repack")(src.data_ptr(), n, k, codes.data_ptr(), scales.data_ptr(), stream()))
    return codes, scales


@pytest.mark.parametrize("fmt", sorted(FORMATS))
def test_repack_streams_are_the_file_fields(fmt):
    """device_layout.h:115-121: every block's codes, then every block's scale word."""
    _, gen, bb, _ = FORMATS[fmt]
    n, k = 48, 1152
    blocks = gen(n, k, seed=21)
    codes, scales = repacked(fmt, blocks, n, k)
    b = blocks.reshape(-1, bb)
    head = 2 if fmt == "q8_0" else 4
    assert np.array_equal(codes.cpu().numpy(), b[:, head:].reshape(-1))
    assert np.array_equal(scales.cpu().numpy(), b[:, :head].reshape(-1))


@pytest.mark.parametrize("fmt", sorted(FORMATS))
@pytest.mark.parametrize("scale", [1.0, float(np.float32(np.sqrt(np.float32(1152))))])
def test_rows_bit_exact(fmt, scale):
    torch = torch_cuda()
    gtype, gen, _, _ = FORMATS[fmt]
    n, k = 40, 1152
    blocks = gen(n, k, seed=22)
    codes, scales = repacked(fmt, blocks, n, k)
    rows = np.array([5, 0, 39, 17, 5], dtype=np.uint32)
    rd = torch.from_numpy(rows.astype(np.int32)).cuda()
    out = torch.empty(len(rows) * k, dtype=torch.float32, device="cuda")
    _native.check(fn(fmt, "rows")(codes.data_ptr(), scales.data_ptr(), n, k, rd.data_ptr(), len(rows),
                                  scale, out.data_ptr(), stream()))
    want = (oracle.dequant_fmt(gtype, blocks).reshape(n, k)[rows] * np.float32(scale)).astype(np.float32)
    assert np.array_equal(out.cpu().numpy().reshape(len(rows), k).view(np.uint32), want.view(np.uint32))


def matvec_case(fmt, n, k, m, seed, x=None):
    torch = torch_cuda()
    gtype, gen, _, _ = FORMATS[fmt]
    blocks = gen(n, k, seed=seed)
    codes, scales = repacked(fmt, blocks, n, k)
    if x is None:
        x = np.random.default_rng([seed, m]).standard_normal((m, k)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    _native.check(fn(fmt, "matvec")(codes.data_ptr(), scales.data_ptr(), n, k, xd.data_ptr(), m, y.data_ptr(),
                                    stream()))
    got = y.cpu().numpy()
    want = oracle.matmul_fmt(gtype, blocks, n, k, x)
    assert np.all(np.isfinite(got))
    rel = np.sqrt(np.mean((got.astype(np.float64) - want) ** 2) / np.mean(want.astype(np.float64) ** 2))
    assert rel < 1e-5, rel
    assert np.max(np.abs(got - want)) <= 1e-4 * np.max(np.abs(want))


# Gemma 3 1B's shapes (K, N) with the pinned file's formats, plus ragged row
# counts (not a multiple of the four rows a warp takes) and small K.
@pytest.mark.parametrize("fmt,k,n,m", [
    ("q8_0", 1152, 4096, 1), ("q8_0", 1152, 4096, 3), ("q8_0", 1152, 2048, 8), ("q8_0", 6912, 1152, 6),
    ("q8_0", 1152, 1001, 2), ("q8_0", 6912, 1152, 8), ("q8_0", 32, 37, 1), ("q8_0", 1024, 1152, 5),
    ("q4_1", 6912, 1152, 1), ("q4_1", 6912, 1152, 4), ("q4_1", 6912, 1152, 7), ("q4_1", 1152, 6912, 8),
    ("q4_1", 1152, 1001, 3), ("q4_1", 64, 19, 2), ("q4_1", 1152, 1024, 1),
])
def test_matvec_against_oracle(fmt, k, n, m):
    matvec_case(fmt, n, k, m, seed=23)


def test_q8_0_head_full_shape():
    """The tied head of the pinned file: 262144 x 1152 Q8_0, one row."""
    matvec_case("q8_0", 262144, 1152, 1, seed=24)


@pytest.mark.parametrize("fmt", sorted(FORMATS))
def test_matvec_block_ranges(fmt):
    """x blocks of very different magnitudes, an all-zero block and a block
    below 2^-100: each block's digits carry its own scale."""
    k, m = 1152, 2
    x = np.random.default_rng(25).standard_normal((m, k)).astype(np.float32)
    x[0, 0:32] = 0.0
    x[0, 32:64] *= np.float32(1e-35)
    x[0, 64:96] *= np.float32(1e20)
    x[1, 96:128] *= np.float32(1e-20)
    x[1, 128:160] = 0.0
    x[1, 128] = np.float32(3.0)
    matvec_case(fmt, 512, k, m, seed=26, x=x)


@pytest.mark.parametrize("fmt", sorted(FORMATS))
def test_matvec_non_finite_row(fmt):
    torch = torch_cuda()
    n, k = 64, 1152
    codes, scales = repacked(fmt, FORMATS[fmt][1](n, k, seed=27), n, k)
    x = np.random.default_rng(28).standard_normal((2, k)).astype(np.float32)
    x[1, 500] = np.inf
    xd = torch.from_numpy(x).cuda()
    y = torch.zeros((2, n), dtype=torch.float32, device="cuda")
    _native.check(fn(fmt, "matvec")(codes.data_ptr(), scales.data_ptr(), n, k, xd.data_ptr(), 2, y.data_ptr(),
                                    stream()))
    got = y.cpu().numpy()
    assert np.all(np.isfinite(got[0])) and np.all(np.isnan(got[1]))
