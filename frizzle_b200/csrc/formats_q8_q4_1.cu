// Q8_0 and Q4_1: the two block formats of Gemma 3 1B's pinned file besides
// Q4_0 (the Q8_0 token embedding the head is tied to, Q4_1 ffn_down in
// layers 0-2), as kernel-level entry points: repack from GGUF blocks, row
// gather, and the HBM-streaming product y[m][n] = sum_k W[n][k] x[m][k] for up
// to eight rows of x.
//
// Device layout: the reference's piece layout with the whole matrix as one
// piece (src/core/formats/device_layout.h:115-121).  First every block's code
// bytes, row-major (row r, block g at (r*K/32 + g) * code_bytes: 32 for Q8_0,
// 16 for Q4_1), then every block's scale word (Q8_0: d, 2 bytes; Q4_1: d and
// m, 4 bytes, d in the low half).  The codes keep the file's bits; a row's
// codes are contiguous, so a warp streams a row with 128-bit loads.
//
// The product: each warp takes four rows of W at a time, their 16-byte code
// chunks as one stream shared over the lanes; every lane holds two batches of
// up to three chunks in registers, the next batch's loads in flight while the
// current one's arithmetic runs.  x is staged once per CTA as three signed
// 8-bit digit planes and an f32 scale per 32-column block (x = s (d0 + d1/254
// + d2/254^2) to about 6e-8 of the block's largest |x|), so the codes, as they
// come from memory (Q8_0) or masked to nibbles (Q4_1), meet x in dp4a integer
// dot products, exact in i32, with one f32 combination a chunk.  Q4_1's
// minimum enters as m * (f32 sum of x over the block).  The lanes' sums meet
// in a reduce-scatter over the warp (4*M values, one per lane group).  The
// result agrees with the reference's f32 sums (matmul.wgsl:154-185) within
// rounding, not bit for bit; a row of x with a non-finite value gives NaN
// sums.  The gather is bit-exact.
#include <algorithm>
#include <string>

#include "frizzle_b200.h"
#include "fz_common.cuh"
#include "last_error.h"

namespace {

enum Format : int { kQ8_0 = 0, kQ4_1 = 1 };

template <int F>
struct Fmt;
template <>
struct Fmt<kQ8_0> {
  static constexpr uint32_t file_bytes = 34, code_bytes = 32, scale_bytes = 2;
  static constexpr uint32_t chunk_cols = 16;  // columns a 16-byte code chunk covers
};
template <>
struct Fmt<kQ4_1> {
  static constexpr uint32_t file_bytes = 20, code_bytes = 16, scale_bytes = 4;
  static constexpr uint32_t chunk_cols = 32;
};

constexpr int kWarps = 8;       // warps a CTA
constexpr int kRows = 4;        // rows of W a warp takes at a time
constexpr int kMaxRows = 8;     // rows of x
constexpr size_t kMaxShared = 200 * 1024;

FZ_DEV uint4 load_stream(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int NV>
struct Log2 {
  static constexpr int value = NV <= 1 ? 0 : 1 + Log2<(NV > 1 ? NV / 2 : 1)>::value;
};
template <>
struct Log2<1> {
  static constexpr int value = 0;
};

// After the call, lane L holds the warp total of v[L >> (5 - log2 NV)]; NV - 1
// shuffles for the halving steps, then plain butterflies.
template <int NV>
FZ_DEV float reduce_scatter(float (&v)[NV], uint32_t lane) {
  constexpr int LOG = Log2<NV>::value;
#pragma unroll
  for (int s = 0; s < LOG; s++) {
    const int half = NV >> (s + 1);
    const int off = 16 >> s;
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int j = 0; j < half; j++) {
      const float send = upper ? v[j] : v[j + half];
      const float keep = upper ? v[j + half] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (int off = 16 >> LOG; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
  return v[0];
}

template <int F>
__global__ void repack_blocks_kernel(const uint8_t* file, size_t blocks, uint8_t* codes, uint8_t* scales) {
  for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < blocks; b += (size_t)gridDim.x * blockDim.x) {
    const uint8_t* src = file + b * Fmt<F>::file_bytes;
    if (F == kQ8_0) {
      // 34-byte blocks: the codes start 2-byte aligned.
      const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; i++) w[i] = (uint32_t)s16[1 + 2 * i] | ((uint32_t)s16[2 + 2 * i] << 16);
      uint4* dst = reinterpret_cast<uint4*>(codes + b * 32);
      dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      reinterpret_cast<uint16_t*>(scales)[b] = s16[0];
    } else {
      const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src);
      reinterpret_cast<uint4*>(codes)[b] = make_uint4(s32[1], s32[2], s32[3], s32[4]);
      reinterpret_cast<uint32_t*>(scales)[b] = s32[0];
    }
  }
}

// out[i][j] = unpack(row rows[i])[j] * scale, in f32 as the gather forms it
// (gather.wgsl:25-48 over q8_0.wgsl / q4_1.wgsl's unpack).
template <int F>
__global__ void rows_kernel(const uint8_t* codes, const uint8_t* scales, uint32_t n, uint32_t k, const uint32_t* rows,
                            uint32_t count, float scale, float* out) {
  const uint32_t i = blockIdx.x;
  if (i >= count) return;
  const uint32_t r = rows[i];
  if (r >= n) return;
  const size_t kb = k / 32;
  for (uint32_t j = threadIdx.x; j < k; j += blockDim.x) {
    const size_t g = (size_t)r * kb + j / 32;
    float w;
    if (F == kQ8_0) {
      const int8_t q = static_cast<int8_t>(codes[(size_t)r * k + j]);
      const float d = fz::f16_unpack(reinterpret_cast<const uint16_t*>(scales)[g]);
      w = fz::mul((float)q, d);
    } else {
      const uint8_t byte = codes[g * 16 + (j % 16)];
      const uint32_t q = (j % 32) < 16 ? byte & 0xFu : byte >> 4;
      const uint32_t dm = reinterpret_cast<const uint32_t*>(scales)[g];
      w = fz::add(fz::mul((float)q, fz::f16_unpack((uint16_t)(dm & 0xffffu))), fz::f16_unpack((uint16_t)(dm >> 16)));
    }
    out[(size_t)i * k + j] = fz::mul(w, scale);
  }
}

// One batch of a lane's code chunks: their words, scale words and places
// ((row in quad << 16) | chunk, ~0u for an empty slot), and the quad they
// belong to, `last` when the batch completes it.
template <int B>
struct Batch {
  uint4 w[B];
  uint32_t sw[B], at[B];
  uint32_t task;
  bool last;
};

template <int F, int MT>
__global__ void __launch_bounds__(kWarps * 32, MT == 1 ? 4 : 2) matvec_kernel(const uint8_t* __restrict__ codes,
                                                             const uint8_t* __restrict__ scales, uint32_t n,
                                                             uint32_t k, const float* __restrict__ x,
                                                             float* __restrict__ y) {
  constexpr int MTP = MT == 1 ? 1 : MT == 2 ? 2 : MT <= 4 ? 4 : 8;
  constexpr int NV = kRows * MTP;
  constexpr int B = MT <= 2 ? 3 : 2;  // chunks a lane loads a batch (3: a 1152- or 6912-wide Q8_0 quad in whole batches)
  extern __shared__ float4 smem[];
  const uint32_t chunks = k / Fmt<F>::chunk_cols, kb = k / 32;
  // x staged as digits: per row and 32-column block, s = max|x| / 127 and
  // three signed 8-bit digit planes with x = s (d0 + d1 / 254 + d2 / 254^2)
  // to within s / 2 / 254^2 (about 6e-8 of the block's largest |x|).
  int8_t* digits = reinterpret_cast<int8_t*>(smem);                  // [MT][3][k]
  float* xscale = reinterpret_cast<float*>(digits + (size_t)MT * 3 * k);  // [MT][kb]
  float* bsum = xscale + MT * kb;                                     // Q4_1: [MT][kb], sum of x
  {
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    for (uint32_t i = warp; i < MT * kb; i += kWarps) {
      const uint32_t mr = i / kb, g = i % kb;
      const float v = x[(size_t)mr * k + g * 32 + lane];
      float mx = fabsf(v);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      // Blocks below 2^-100 are scaled up by 2^64 first, so 127 / max stays
      // finite; a non-finite block gets a NaN scale (its rows' sums become NaN).
      const float pre = mx < 0x1p-100f ? 0x1p64f : 1.0f;
      const bool finite = mx <= 3.402823466e38f;
      const float inv = mx > 0.0f && finite ? 127.0f / (mx * pre) : 0.0f;
      const float t = finite ? v * pre * inv : 0.0f;
      const float d0 = fminf(fmaxf(rintf(t), -127.0f), 127.0f);
      const float r1 = (t - d0) * 254.0f;
      const float d1 = fminf(fmaxf(rintf(r1), -127.0f), 127.0f);
      const float r2 = (r1 - d1) * 254.0f;
      const float d2 = fminf(fmaxf(rintf(r2), -127.0f), 127.0f);
      int8_t* dg = digits + (size_t)mr * 3 * k + g * 32 + lane;
      dg[0] = (int8_t)d0;
      dg[k] = (int8_t)d1;
      dg[2 * k] = (int8_t)d2;
      if (lane == 0) xscale[i] = finite ? mx * pre / 127.0f / pre : __int_as_float(0x7fc00000);
      if (F == kQ4_1) {
        const float sum = fz::warp_sum(v);
        if (lane == 0) bsum[i] = sum;
      }
    }
  }
  __syncthreads();

  const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t quads = (n + kRows - 1) / kRows, stride = gridDim.x * kWarps;
  const size_t row_bytes = (size_t)kb * Fmt<F>::code_bytes;
  // A warp's quads' chunks as one stream: quad `task`'s kRows * chunks items,
  // item f being chunk f % chunks of row f / chunks, so every lane has work in
  // every batch whatever the row length; a lane's items advance by 32 a slot.
  // Two batches in registers: one batch's loads are in flight while the
  // other's arithmetic runs, across quad boundaries too.
  const uint32_t items = kRows * chunks;
  const uint32_t rl0 = lane / chunks, c0 = lane % chunks;
  uint32_t task = blockIdx.x * kWarps + warp, f0 = 0, rl = rl0, c = c0;

  float acc[kRows][MT];
#pragma unroll
  for (int r = 0; r < kRows; r++)
#pragma unroll
    for (int m = 0; m < MT; m++) acc[r][m] = 0.0f;

  Batch<B> bufA, bufB;
  auto fetch = [&](Batch<B>& bt) {
    bt.task = task;
    bt.last = false;
    if (task >= quads) return;
    const uint32_t r0 = task * kRows;
#pragma unroll
    for (int i = 0; i < B; i++) {
      const uint32_t row = r0 + rl;
      if (f0 + 32 * i + lane < items && row < n) {
        bt.w[i] = load_stream(codes + row * row_bytes + (size_t)c * 16);
        if (F == kQ8_0)
          bt.sw[i] = __ldg(reinterpret_cast<const uint16_t*>(scales) + (size_t)row * kb + c / 2);
        else
          bt.sw[i] = __ldg(reinterpret_cast<const uint32_t*>(scales) + (size_t)row * kb + c);
        bt.at[i] = (rl << 16) | c;
      } else {
        bt.at[i] = ~0u;
      }
      c += 32;
      while (c >= chunks) {
        c -= chunks;
        rl++;
      }
    }
    f0 += 32 * B;
    if (f0 >= items) {
      bt.last = true;
      task += stride;
      f0 = 0;
      rl = rl0;
      c = c0;
    }
  };
  auto consume = [&](const Batch<B>& bt) {
#pragma unroll
    for (int i = 0; i < B; i++) {
      if (bt.at[i] == ~0u) continue;
      const uint32_t cc = bt.at[i] & 0xffffu, rr = bt.at[i] >> 16;
      // Integer products of the codes with each digit plane (exact in i32),
      // then one f32 combination a chunk.
      float val[MT];
      if (F == kQ8_0) {
        const float d = fz::f16_unpack((uint16_t)bt.sw[i]);
#pragma unroll
        for (int m = 0; m < MT; m++) {
          const int8_t* dg = digits + (size_t)m * 3 * k + cc * 16;
          const uint4 p0 = *reinterpret_cast<const uint4*>(dg);
          const uint4 p1 = *reinterpret_cast<const uint4*>(dg + k);
          const uint4 p2 = *reinterpret_cast<const uint4*>(dg + 2 * k);
          const uint4 w = bt.w[i];
          const int s0 = __dp4a((int)w.w, (int)p0.w, __dp4a((int)w.z, (int)p0.z,
                         __dp4a((int)w.y, (int)p0.y, __dp4a((int)w.x, (int)p0.x, 0))));
          const int s1 = __dp4a((int)w.w, (int)p1.w, __dp4a((int)w.z, (int)p1.z,
                         __dp4a((int)w.y, (int)p1.y, __dp4a((int)w.x, (int)p1.x, 0))));
          const int s2 = __dp4a((int)w.w, (int)p2.w, __dp4a((int)w.z, (int)p2.z,
                         __dp4a((int)w.y, (int)p2.y, __dp4a((int)w.x, (int)p2.x, 0))));
          const float sum = fmaf((float)s2, 1.0f / 64516.0f, fmaf((float)s1, 1.0f / 254.0f, (float)s0));
          val[m] = d * xscale[m * kb + cc / 2] * sum;
        }
      } else {
        const float d = fz::f16_unpack((uint16_t)(bt.sw[i] & 0xffffu));
        const float mn = fz::f16_unpack((uint16_t)(bt.sw[i] >> 16));
        // Byte j's low nibble is column j, its high nibble column j + 16;
        // nibbles are 0..15, the same bytes signed or unsigned.
        const uint32_t words[4] = {bt.w[i].x, bt.w[i].y, bt.w[i].z, bt.w[i].w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          lo[q] = words[q] & 0x0F0F0F0Fu;
          hi[q] = (words[q] >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
          int sp[3];
#pragma unroll
          for (int pl = 0; pl < 3; pl++) {
            const int8_t* dg = digits + ((size_t)m * 3 + pl) * k + cc * 32;
            const uint4 a0 = *reinterpret_cast<const uint4*>(dg);
            const uint4 a1 = *reinterpret_cast<const uint4*>(dg + 16);
            int t = __dp4a((int)lo[0], (int)a0.x, 0);
            t = __dp4a((int)lo[1], (int)a0.y, t);
            t = __dp4a((int)lo[2], (int)a0.z, t);
            t = __dp4a((int)lo[3], (int)a0.w, t);
            t = __dp4a((int)hi[0], (int)a1.x, t);
            t = __dp4a((int)hi[1], (int)a1.y, t);
            t = __dp4a((int)hi[2], (int)a1.z, t);
            sp[pl] = __dp4a((int)hi[3], (int)a1.w, t);
          }
          const float sum = fmaf((float)sp[2], 1.0f / 64516.0f, fmaf((float)sp[1], 1.0f / 254.0f, (float)sp[0]));
          val[m] = fmaf(mn, bsum[m * kb + cc], d * xscale[m * kb + cc] * sum);
        }
      }
#pragma unroll
      for (int r = 0; r < kRows; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) acc[r][m] += rr == (uint32_t)r ? val[m] : 0.0f;
    }
    if (!bt.last) return;
    // The quad is complete: its kRows x MT sums meet across the warp.
    float v[NV];
#pragma unroll
    for (int r = 0; r < kRows; r++)
#pragma unroll
      for (int m = 0; m < MTP; m++) v[r * MTP + m] = m < MT ? acc[r][m < MT ? m : 0] : 0.0f;
    const float sum = reduce_scatter<NV>(v, lane);
    constexpr int SHIFT = 5 - Log2<NV>::value;
    if ((lane & ((1u << SHIFT) - 1)) == 0) {
      const uint32_t idx = lane >> SHIFT, r = idx / MTP, m = idx % MTP;
      const uint32_t row = bt.task * kRows + r;
      if (m < MT && row < n) y[(size_t)m * n + row] = sum;
    }
#pragma unroll
    for (int r = 0; r < kRows; r++)
#pragma unroll
      for (int m = 0; m < MT; m++) acc[r][m] = 0.0f;
  };

  // task, and so every branch below, is uniform over the warp.
  fetch(bufA);
  while (bufA.task < quads) {
    fetch(bufB);
    consume(bufA);
    if (bufB.task >= quads) break;
    fetch(bufA);
    consume(bufB);
  }
}

fz_status refuse(fz_status s, const std::string& why) {
  fz::set_last_error(why.c_str());
  return s;
}

fz_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FZ_OK;
  return refuse(e == cudaErrorIllegalAddress || e == cudaErrorLaunchFailure ? FZ_ERR_DEVICE_LOST : FZ_ERR_CUDA,
                std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

fz_status check_matrix(uint32_t n, uint32_t k) {
  if (n == 0 || k == 0 || k % 32) return refuse(FZ_ERR_ARGUMENT, "n must be at least 1 and k a multiple of 32");
  return FZ_OK;
}

template <int F>
fz_status repack(const void* file_blocks, uint32_t n, uint32_t k, void* codes, void* scales, void* stream) {
  fz_status st;
  if ((st = check_matrix(n, k))) return st;
  if (!file_blocks || !codes || !scales) return refuse(FZ_ERR_ARGUMENT, "null pointer");
  if (!aligned(file_blocks, F == kQ8_0 ? 2 : 4) || !aligned(codes, 16) || !aligned(scales, Fmt<F>::scale_bytes))
    return refuse(FZ_ERR_ARGUMENT, "misaligned pointer (file blocks 2 or 4 bytes, codes 16, scales 2 or 4)");
  const size_t blocks = (size_t)n * (k / 32);
  const int grid = (int)std::min<size_t>((blocks + 255) / 256, 148 * 16);
  (void)cudaGetLastError();
  repack_blocks_kernel<F><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(file_blocks), blocks, static_cast<uint8_t*>(codes), static_cast<uint8_t*>(scales));
  return cuda_status(cudaGetLastError(), "repack");
}

template <int F>
fz_status rows(const void* codes, const void* scales, uint32_t n, uint32_t k, const uint32_t* row_ids, uint32_t count,
               float scale, float* out, void* stream) {
  fz_status st;
  if ((st = check_matrix(n, k))) return st;
  if (!codes || !scales || !row_ids || !out) return refuse(FZ_ERR_ARGUMENT, "null pointer");
  if (!aligned(scales, Fmt<F>::scale_bytes)) return refuse(FZ_ERR_ARGUMENT, "misaligned scales");
  if (count == 0) return FZ_OK;
  (void)cudaGetLastError();
  rows_kernel<F><<<count, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(codes), static_cast<const uint8_t*>(scales), n, k, row_ids, count, scale, out);
  return cuda_status(cudaGetLastError(), "rows");
}

template <int F, int MT>
fz_status launch_mt(const uint8_t* codes, const uint8_t* scales, uint32_t n, uint32_t k, const float* x, float* y,
                    size_t smem, cudaStream_t stream) {
  auto kernel = matvec_kernel<F, MT>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "matvec attribute");
  int dev = 0, sms = 0, per_sm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess || (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
      (e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kWarps * 32, smem)) != cudaSuccess)
    return cuda_status(e, "matvec occupancy");
  const size_t quads = ((size_t)n + kRows - 1) / kRows;
  const size_t want = (quads + kWarps - 1) / kWarps;
  const int grid = (int)std::max<size_t>(1, std::min<size_t>(want, (size_t)sms * std::max(per_sm, 1)));
  (void)cudaGetLastError();
  kernel<<<grid, kWarps * 32, smem, stream>>>(codes, scales, n, k, x, y);
  return cuda_status(cudaGetLastError(), "matvec");
}

template <int F>
fz_status matvec(const void* codes, const void* scales, uint32_t n, uint32_t k, const float* x, uint32_t m, float* y,
                 void* stream) {
  fz_status st;
  if ((st = check_matrix(n, k))) return st;
  if (!codes || !scales || !x || !y) return refuse(FZ_ERR_ARGUMENT, "null pointer");
  if (m < 1 || m > (uint32_t)kMaxRows) return refuse(FZ_ERR_ARGUMENT, "m outside 1 .. 8");
  if (!aligned(codes, 16) || !aligned(x, 16) || !aligned(scales, Fmt<F>::scale_bytes))
    return refuse(FZ_ERR_ARGUMENT, "misaligned pointer (codes and x 16 bytes, scales 2 or 4)");
  // Staged x: three digit bytes a value and a scale a block (Q4_1: and a block sum).
  const size_t smem = (size_t)m * k * 3 + (size_t)m * (k / 32) * 4 * (F == kQ4_1 ? 2 : 1);
  if (smem > kMaxShared)
    return refuse(FZ_ERR_ARGUMENT, "m x k too large: x is staged in 200 KiB of shared memory, 3.125 bytes a value "
                                   "(3.25 for Q4_1)");
  const auto* c = static_cast<const uint8_t*>(codes);
  const auto* s = static_cast<const uint8_t*>(scales);
  cudaStream_t st_ = static_cast<cudaStream_t>(stream);
  switch (m) {
    case 1: return launch_mt<F, 1>(c, s, n, k, x, y, smem, st_);
    case 2: return launch_mt<F, 2>(c, s, n, k, x, y, smem, st_);
    case 3: return launch_mt<F, 3>(c, s, n, k, x, y, smem, st_);
    case 4: return launch_mt<F, 4>(c, s, n, k, x, y, smem, st_);
    case 5: return launch_mt<F, 5>(c, s, n, k, x, y, smem, st_);
    case 6: return launch_mt<F, 6>(c, s, n, k, x, y, smem, st_);
    case 7: return launch_mt<F, 7>(c, s, n, k, x, y, smem, st_);
    default: return launch_mt<F, 8>(c, s, n, k, x, y, smem, st_);
  }
}

}  // namespace

extern "C" {

size_t fz_q8_0_codes_bytes(uint32_t n, uint32_t k) { return (size_t)n * k; }
size_t fz_q8_0_scales_bytes(uint32_t n, uint32_t k) { return (size_t)n * (k / 32) * 2; }
size_t fz_q4_1_codes_bytes(uint32_t n, uint32_t k) { return (size_t)n * k / 2; }
size_t fz_q4_1_scales_bytes(uint32_t n, uint32_t k) { return (size_t)n * (k / 32) * 4; }

fz_status fz_q8_0_repack(const void* file_blocks, uint32_t n, uint32_t k, void* codes, void* scales, void* stream) {
  return repack<kQ8_0>(file_blocks, n, k, codes, scales, stream);
}
fz_status fz_q4_1_repack(const void* file_blocks, uint32_t n, uint32_t k, void* codes, void* scales, void* stream) {
  return repack<kQ4_1>(file_blocks, n, k, codes, scales, stream);
}
fz_status fz_q8_0_rows(const void* codes, const void* scales, uint32_t n, uint32_t k, const uint32_t* row_ids,
                       uint32_t count, float scale, float* out, void* stream) {
  return rows<kQ8_0>(codes, scales, n, k, row_ids, count, scale, out, stream);
}
fz_status fz_q4_1_rows(const void* codes, const void* scales, uint32_t n, uint32_t k, const uint32_t* row_ids,
                       uint32_t count, float scale, float* out, void* stream) {
  return rows<kQ4_1>(codes, scales, n, k, row_ids, count, scale, out, stream);
}
fz_status fz_q8_0_matvec(const void* codes, const void* scales, uint32_t n, uint32_t k, const float* x, uint32_t m,
                         float* y, void* stream) {
  return matvec<kQ8_0>(codes, scales, n, k, x, m, y, stream);
}
fz_status fz_q4_1_matvec(const void* codes, const void* scales, uint32_t n, uint32_t k, const float* x, uint32_t m,
                         float* y, void* stream) {
  return matvec<kQ4_1>(codes, scales, n, k, x, m, y, stream);
}

}  // extern "C"
