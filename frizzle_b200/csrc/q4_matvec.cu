// The Q4_0 repack and the skinny tensor-core product over the fragment-native
// layout (q4_matvec.cuh), with the norm prologue and the QKV/RoPE, gated
// GELU/steering and head/argmax epilogues of Frizzle's matmul launches
// (kernels/matmul/matmul.wgsl, kernels/norm/norm.wgsl, kernels/rope/*.wgsl,
// edit/edit.wgsl fused where they follow one another).
//
// Arithmetic.  Each weight (code - 8) is exact in f16; each f32 input x is
// split x = hi + lo with hi = f16(x) and lo = f16(x - hi), the pair carried
// as two columns of the mma's B operand, so a block's products are f32-exact
// to about 2^-22 relative; the block's f16 scale is applied in f32 to the
// block's f32 partial.  The sum order differs from the reference's 32 fixed
// ranges (matmul.h:88-97), so results agree with the oracle to f32 rounding,
// not bit for bit.
#include <cooperative_groups.h>

#include <map>
#include <mutex>

#include "q4_device.cuh"
#include "q4_matvec.cuh"

namespace cg = cooperative_groups;

namespace fz {
namespace {

using namespace q4dev;

constexpr int kThreads = 256;   // every matvec CTA: 8 warps, the norm's 256 invocations
constexpr int kWarps = kThreads / 32;
constexpr int kU = 4;           // block pairs a warp loads at once
constexpr int kUW = 6;          // the same, when a warp streams whole row groups (K = 1152: 3 batches)

// A warp's registers for kU block pairs of one row group.
struct Batch {
  uint4 c[kU];
  uint2 s[kU];
};

FZ_DEV void load_batch(const uint4* codes, const uint2* scales, int bp, int bp1, int lane, Batch& b) {
  const int g = lane >> 2;
#pragma unroll
  for (int u = 0; u < kU; u++) {
    if (bp + u < bp1) {
      b.c[u] = ld_stream(codes + (size_t)(bp + u) * 32 + lane);
      b.s[u] = ld_stream2(scales + (size_t)(bp + u) * 8 + g);
    }
  }
}

// The batch's products into acc: lane (g, t) accumulates rows g (acc[q][0])
// and g + 8 (acc[q][1]) against X row 4q + t.
template <int MQ>
FZ_DEV void compute_batch(const Batch& b, int bp, int bp1, const uint2* xf, int kb_base, int lane, float acc[MQ][2]) {
  const int g = lane >> 2, t = lane & 3;
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int u = 0; u < kU; u++) {
    if (bp + u < bp1) {
#pragma unroll
      for (int kbi = 0; kbi < 2; kbi++) {
        const int kb_rel = 2 * (bp + u) + kbi - kb_base;
        uint32_t a0[4], a1[4];
        dequant_word(kbi ? b.c[u].z : b.c[u].x, a0);
        dequant_word(kbi ? b.c[u].w : b.c[u].y, a1);
        const uint32_t sw = kbi ? b.s[u].y : b.s[u].x;
        const float dg = __half2float(__ushort_as_half((unsigned short)(sw & 0xffffu)));
        const float dg8 = __half2float(__ushort_as_half((unsigned short)(sw >> 16)));
#pragma unroll
        for (int q = 0; q < MQ; q++) {
          const uint2 b0 = xf[xf_index(kb_rel, 0, q, MQ, t, g)];
          const uint2 b1 = xf[xf_index(kb_rel, 1, q, MQ, t, g)];
          float d[4];
          mma16816(d, a0, b0, zero);
          mma16816(d, a1, b1, d);
          acc[q][0] = __fmaf_rn(dg, d[0] + d[1], acc[q][0]);
          acc[q][1] = __fmaf_rn(dg8, d[2] + d[3], acc[q][1]);
        }
      }
    }
  }
}

// Whole batches of U block pairs, for the warp-streaming form: no bounds
// test (the row group's block pairs are a multiple of U).
template <int U>
struct BatchU {
  uint4 c[U];
  uint2 s[U];
};

template <int U>
FZ_DEV void load_u(const uint4* codes, const uint2* scales, int bp, int lane, BatchU<U>& b) {
  const int g = lane >> 2;
#pragma unroll
  for (int u = 0; u < U; u++) {
    b.c[u] = ld_stream(codes + (size_t)(bp + u) * 32 + lane);
    b.s[u] = ld_stream2(scales + (size_t)(bp + u) * 8 + g);
  }
}

template <int U, int MQ>
FZ_DEV void compute_u(const BatchU<U>& b, int bp, const uint2* xf, int lane, float acc[MQ][2]) {
  const int g = lane >> 2, t = lane & 3;
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int u = 0; u < U; u++) {
#pragma unroll
    for (int kbi = 0; kbi < 2; kbi++) {
      const int kb = 2 * (bp + u) + kbi;
      uint32_t a0[4], a1[4];
      dequant_word(kbi ? b.c[u].z : b.c[u].x, a0);
      dequant_word(kbi ? b.c[u].w : b.c[u].y, a1);
      const uint32_t sw = kbi ? b.s[u].y : b.s[u].x;
      const float dg = __half2float(__ushort_as_half((unsigned short)(sw & 0xffffu)));
      const float dg8 = __half2float(__ushort_as_half((unsigned short)(sw >> 16)));
#pragma unroll
      for (int q = 0; q < MQ; q++) {
        const uint2 b0 = xf[xf_index(kb, 0, q, MQ, t, g)];
        const uint2 b1 = xf[xf_index(kb, 1, q, MQ, t, g)];
        float d[4];
        mma16816(d, a0, b0, zero);
        mma16816(d, a1, b1, d);
        acc[q][0] = __fmaf_rn(dg, d[0] + d[1], acc[q][0]);
        acc[q][1] = __fmaf_rn(dg8, d[2] + d[3], acc[q][1]);
      }
    }
  }
}

// One warp's sums for its row group over block pairs [bp0, bp1), two register
// batches in flight: `first` already holds the batch at bp0.
template <int MQ>
FZ_DEV void rowgroup_dot(const uint4* codes, const uint2* scales, int bp0, int bp1, const uint2* xf, int kb_base,
                         int lane, Batch& first, float acc[MQ][2]) {
  Batch second;
  for (int bp = bp0; bp < bp1; bp += 2 * kU) {
    if (bp + kU < bp1) load_batch(codes, scales, bp + kU, bp1, lane, second);
    compute_batch<MQ>(first, bp, bp1, xf, kb_base, lane, acc);
    if (bp + kU < bp1) {
      if (bp + 2 * kU < bp1) load_batch(codes, scales, bp + 2 * kU, bp1, lane, first);
      compute_batch<MQ>(second, bp + kU, bp1, xf, kb_base, lane, acc);
    }
  }
}

// The reference norm's fixed-order tree over the CTA's 256 invocations, for
// `rows` rows at once (norm.wgsl:75-85): part[r][i] holds invocation i's sum;
// halving levels 128, 64, 32 in shared memory, the last five inside a warp.
// Leaves each row's total in total[r].
FZ_DEV void tree_reduce(float* part, int rows, float* total) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __syncthreads();
  for (int stride = 128; stride >= 32; stride >>= 1) {
    for (int idx = tid; idx < rows * stride; idx += kThreads) {
      const int r = idx / stride, i = idx % stride;
      part[r * kThreads + i] = add(part[r * kThreads + i], part[r * kThreads + i + stride]);
    }
    __syncthreads();
  }
  for (int r = warp; r < rows; r += kWarps) {
    float s = part[r * kThreads + lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float other = __shfl_down_sync(0xffffffffu, s, o);
      if (lane < o) s = add(s, other);
    }
    if (lane == 0) total[r] = s;
  }
  __syncthreads();
}

// vec4 v of the block output y for one row: y itself, or the sum of its
// n.y_parts K-slice partials (n.y_part_stride floats apart), in slice order.
FZ_DEV float4 y_sum(const NormArgs& n, const float* yr, int v) {
  float4 y = __ldcg(reinterpret_cast<const float4*>(yr) + v);
  for (uint32_t k = 1; k < n.y_parts; k++) {
    const float4 z = __ldcg(reinterpret_cast<const float4*>(yr + k * n.y_part_stride) + v);
    y = make_float4(add(y.x, z.x), add(y.y, z.y), add(y.z, z.z), add(y.w, z.w));
  }
  return y;
}

// The norm launch over the step's rows, by the whole CTA (norm.wgsl:97-198):
// invocation i of the reference is thread i, holding vec4s i, i + 256, ...
// Leaves the normed rows in `rowbuf` [rows][width]; CTA 0 writes X after the
// add to hidden_out and the captures of each sequence's last row.  With
// `ystage` ([rows][width] of shared memory) and several rows, every row's X
// and y are first staged by 16-byte cp.async with all the loads in flight,
// so the passes read shared memory instead of waiting on one row at a time.
FZ_DEV void norm_rows_cta(const MatvecArgs& a, const NormArgs& n, int rows, float* rowbuf, float* part, float* stat,
                          bool writer, float* ystage = nullptr) {
  const int tid = threadIdx.x, W = (int)n.width, V = W / 4;
  const float wf = (float)W;
  float* ry = stat;
  float* rx = stat + kMaxTokens;
  auto hrow_of = [&](int r) { return r * (int)n.row_of_token_stride + (int)n.row_of_token_offset; };
  const bool staged = ystage != nullptr && n.y_parts <= 1 && rows > 1;
  if (staged) {
    for (int i = tid; i < rows * V; i += kThreads) {
      const int r = i / V, v = i % V;
      const size_t off = (size_t)hrow_of(r) * W + 4 * v;
      stage16(rowbuf + (size_t)r * W + 4 * v, n.hidden_in + off);
      if (n.y) stage16(ystage + (size_t)r * W + 4 * v, n.y + off);
    }
    stage_wait();
    __syncthreads();
  }
  // Row r's y at vec4 v: staged, or the sum of its K-slice partials.
  auto y_at = [&](int r, const float* yr, int v) -> float4 {
    return staged ? reinterpret_cast<const float4*>(ystage + (size_t)r * W)[v] : y_sum(n, yr, v);
  };
  if (n.y && n.post_gain) {
    for (int r = 0; r < rows; r++) {
      const float* yr = n.y + (size_t)hrow_of(r) * W;
      float p = 0.f;
      for (int v = tid; v < V; v += kThreads) p = add(p, dot_self(y_at(r, yr, v)));
      part[r * kThreads + tid] = p;
    }
    tree_reduce(part, rows, ry);
    if (tid < rows) ry[tid] = inverse_sqrt(add(__fdiv_rn(ry[tid], wf), n.eps));
    __syncthreads();
  }
  for (int r = 0; r < rows; r++) {
    const int hrow = hrow_of(r);
    const uint32_t seq = (uint32_t)hrow / a.seq_tokens;
    const bool last = (uint32_t)hrow % a.seq_tokens == a.seq_tokens - 1;
    float4* buf = reinterpret_cast<float4*>(rowbuf + (size_t)r * W);
    const float4* x4 = staged ? buf : reinterpret_cast<const float4*>(n.hidden_in + (size_t)hrow * W);
    const float* yr = n.y ? n.y + (size_t)hrow * W : nullptr;
    const float4* pg4 = reinterpret_cast<const float4*>(n.post_gain);
    float4* out4 = writer && n.hidden_out ? reinterpret_cast<float4*>(n.hidden_out + (size_t)hrow * W) : nullptr;
    float4* xcap = writer && last && n.capture_residual
                       ? reinterpret_cast<float4*>(n.capture_residual + seq * a.capture_stride) : nullptr;
    float4* ycap = writer && last && n.capture_added
                       ? reinterpret_cast<float4*>(n.capture_added + seq * a.capture_stride) : nullptr;
    float p = 0.f;
    for (int v = tid; v < V; v += kThreads) {
      float4 x = x4[v];
      if (yr) {
        float4 y = y_at(r, yr, v);
        if (n.post_gain) {
          const float s = ry[r];
          const float4 g = pg4[v];
          y = make_float4(mul(mul(y.x, s), g.x), mul(mul(y.y, s), g.y), mul(mul(y.z, s), g.z), mul(mul(y.w, s), g.w));
        }
        if (ycap) ycap[v] = y;
        x = make_float4(add(x.x, y.x), add(x.y, y.y), add(x.z, y.z), add(x.w, y.w));
      }
      if (out4) out4[v] = x;
      if (xcap) xcap[v] = x;
      buf[v] = x;
      p = add(p, dot_self(x));
    }
    part[r * kThreads + tid] = p;
  }
  tree_reduce(part, rows, rx);
  if (tid < rows) rx[tid] = inverse_sqrt(add(__fdiv_rn(rx[tid], wf), n.eps));
  __syncthreads();
  const float4* g4 = reinterpret_cast<const float4*>(n.gain);
  for (int r = 0; r < rows; r++) {
    float4* buf = reinterpret_cast<float4*>(rowbuf + (size_t)r * W);
    const float s = rx[r];
    for (int v = tid; v < V; v += kThreads) {
      const float4 x = buf[v], g = g4[v];
      buf[v] = make_float4(mul(mul(x.x, s), g.x), mul(mul(x.y, s), g.y), mul(mul(x.z, s), g.z), mul(mul(x.w, s), g.w));
    }
  }
  __syncthreads();
}


// Shared memory of one CTA, carved from the dynamic allocation.
struct Smem {
  uint2* xf;       // X fragments of the CTA's K range
  float* red;      // [RG][KS][16 rows][16 tokens] K-split partials
  float* rowbuf;   // [m][width] normed rows (norm prologue)
  float* part;     // [m][256] the norm tree's partials
  float* stat;     // 2 x kMaxTokens reciprocal RMS values
  float* cred;     // [C][outs] cluster partials (rank 0's is the one read)
};

struct Geometry {
  uint32_t C, KS, RG, rank, NBP, nrowsets;
  int kb_base, nkb, nkb_max;
};

template <int MQ, int PRO>
FZ_DEV Smem carve(unsigned char* raw, const MatvecArgs& a, const Geometry& geo) {
  Smem s;
  s.xf = reinterpret_cast<uint2*>(raw);
  s.red = reinterpret_cast<float*>(s.xf + (size_t)geo.nkb_max * 2 * MQ * 32);
  s.rowbuf = s.red + geo.RG * geo.KS * 256;
  s.part = s.rowbuf + (PRO == kPrologueNorm ? (size_t)a.m * a.norm.width : 0);
  s.stat = s.part + (PRO == kPrologueNorm ? (size_t)a.m * kThreads : 0);
  s.cred = s.stat + 2 * kMaxTokens;
  return s;
}

// X rows as B fragments for the CTA's blocks [kb_base, kb_base + nkb): from
// the input rows, or through the norm.
template <int MQ, int PRO>
FZ_DEV void prologue(const MatvecArgs& a, const Smem& sm, const Geometry& geo) {
  const int M = (int)a.m, K = (int)a.mat[0].k;
  const float* rows = a.x;
  if (PRO == kPrologueNorm) {
    // The fragments' region holds the staged y rows until the fragments are built.
    const size_t xf_bytes = (size_t)geo.nkb_max * 2 * MQ * 32 * sizeof(uint2);
    float* ystage = geo.C == 1 && (size_t)M * a.norm.width * 4 <= xf_bytes ? reinterpret_cast<float*>(sm.xf) : nullptr;
    norm_rows_cta(a, a.norm, M, sm.rowbuf, sm.part, sm.stat, blockIdx.x == 0, ystage);
    rows = sm.rowbuf;
  }
  build_fragments_rows<MQ>(sm.xf, M, rows, K, geo.kb_base, geo.nkb, threadIdx.x, kThreads);
  __syncthreads();
}

// Writes one finished output (row n of the product, X row `tok`).
template <int EPI>
FZ_DEV void write_out(const MatvecArgs& a, uint32_t n, int tok, float v) {
  a.out[(size_t)tok * a.out_stride + n] = v;
}


template <int MQ, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads) matvec_kernel(const MatvecArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint32_t s_last;
  __shared__ unsigned long long s_best[kMaxTokens];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int M = (int)a.m;
  Geometry geo;
  geo.C = a.cluster;
  geo.KS = a.k_split;
  geo.RG = a.rg_per_cta;
  geo.rank = 0;
  if (geo.C > 1) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(geo.rank));
  geo.NBP = a.mat[0].k / 64;
  geo.nrowsets = EPI == kEpilogueGated ? a.mat[0].n / 16 : (a.mat[0].n / 16 + geo.RG - 1) / geo.RG;
  const int cta_bp0 = (int)(geo.rank * geo.NBP / geo.C), cta_bp1 = (int)((geo.rank + 1) * geo.NBP / geo.C);
  geo.kb_base = 2 * cta_bp0;
  geo.nkb = 2 * (cta_bp1 - cta_bp0);
  geo.nkb_max = 2 * (int)((geo.NBP + geo.C - 1) / geo.C);
  const Smem sm = carve<MQ, PRO>(smem_raw, a, geo);
  if (threadIdx.x < kMaxTokens) s_best[threadIdx.x] = 0ull;

  const bool warp_mode = geo.KS == 1 && geo.C == 1 && EPI != kEpilogueGated;
  Batch first;
  float acc[MQ][2];

  if (warp_mode && geo.NBP % kUW == 0) {
    // Each warp streams its row groups rg, rg + total, ... as one sequence of
    // kUW-block-pair batches: the next batch's loads (the next row group's
    // first, at a row group's end) are in flight while one is computed.
    const uint32_t nrg = a.mat[0].n / 16, NBP = geo.NBP, nb = NBP / kUW;
    const uint32_t total = gridDim.x * kWarps;
    const Q4Matrix& mat = a.mat[0];
    auto codes_of = [&](uint32_t r) { return mat.codes + (size_t)r * NBP * 32; };
    auto scales_of = [&](uint32_t r) { return mat.scales + (size_t)r * NBP * 8; };
    uint32_t rg = blockIdx.x * kWarps + warp, j = 0;
    BatchU<kUW> b0, b1;
    if (rg < nrg) load_u<kUW>(codes_of(rg), scales_of(rg), 0, lane, b0);
    pdl_wait();
    prologue<MQ, PRO>(a, sm, geo);
    unsigned long long best[MQ];
#pragma unroll
    for (int q = 0; q < MQ; q++) {
      best[q] = 0ull;
      acc[q][0] = acc[q][1] = 0.f;
    }
    auto finish = [&](uint32_t r) {
#pragma unroll
      for (int q = 0; q < MQ; q++) {
        const int tok = 4 * q + t;
        if (tok < M) {
          const uint32_t n0 = r * 16 + g, n8 = n0 + 8;
          a.out[(size_t)tok * a.out_stride + n0] = acc[q][0];
          a.out[(size_t)tok * a.out_stride + n8] = acc[q][1];
          if (EPI == kEpilogueHead) best[q] = max(best[q], max(head_key(acc[q][0], n0), head_key(acc[q][1], n8)));
        }
        acc[q][0] = acc[q][1] = 0.f;
      }
    };
    auto next = [&](uint32_t& r, uint32_t& k) {
      if (++k == nb) {
        k = 0;
        r += total;
      }
    };
    while (rg < nrg) {
      uint32_t rg1 = rg, j1 = j;
      next(rg1, j1);
      if (rg1 < nrg) load_u<kUW>(codes_of(rg1), scales_of(rg1), (int)(j1 * kUW), lane, b1);
      compute_u<kUW, MQ>(b0, (int)(j * kUW), sm.xf, lane, acc);
      if (j == nb - 1) finish(rg);
      if (rg1 >= nrg) break;
      uint32_t rg2 = rg1, j2 = j1;
      next(rg2, j2);
      if (rg2 < nrg) load_u<kUW>(codes_of(rg2), scales_of(rg2), (int)(j2 * kUW), lane, b0);
      compute_u<kUW, MQ>(b1, (int)(j1 * kUW), sm.xf, lane, acc);
      if (j1 == nb - 1) finish(rg1);
      rg = rg2;
      j = j2;
    }
    pdl_launch_dependents();
    if (EPI == kEpilogueHead) {
#pragma unroll
      for (int q = 0; q < MQ; q++) {
        unsigned long long b = best[q];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
        const int tok = 4 * q + t;
        if (g == 0 && tok < M && b) atomicMax(a.head.argmax + tok, b);
      }
    }
  } else if (warp_mode) {
    // Each warp streams whole row groups on its own; no CTA barrier in the loop.
    const uint32_t nrg = a.mat[0].n / 16, NBP = geo.NBP;
    const uint32_t total = gridDim.x * kWarps;
    uint32_t rg = blockIdx.x * kWarps + warp;
    const Q4Matrix& mat = a.mat[0];
    if (rg < nrg) {
      const uint4* codes = mat.codes + (size_t)rg * NBP * 32;
      const uint2* scales = mat.scales + (size_t)rg * NBP * 8;
      load_batch(codes, scales, 0, (int)NBP, lane, first);
    }
    pdl_wait();
    prologue<MQ, PRO>(a, sm, geo);
    unsigned long long best[MQ];
#pragma unroll
    for (int q = 0; q < MQ; q++) best[q] = 0ull;
    for (; rg < nrg; rg += total) {
      const uint4* codes = mat.codes + (size_t)rg * NBP * 32;
      const uint2* scales = mat.scales + (size_t)rg * NBP * 8;
#pragma unroll
      for (int q = 0; q < MQ; q++) acc[q][0] = acc[q][1] = 0.f;
      rowgroup_dot<MQ>(codes, scales, 0, (int)NBP, sm.xf, 0, lane, first, acc);
      if (rg + total < nrg)
        load_batch(mat.codes + (size_t)(rg + total) * NBP * 32, mat.scales + (size_t)(rg + total) * NBP * 8, 0,
                   (int)NBP, lane, first);
#pragma unroll
      for (int q = 0; q < MQ; q++) {
        const int tok = 4 * q + t;
        if (tok < M) {
          const uint32_t n0 = rg * 16 + g, n8 = n0 + 8;
          a.out[(size_t)tok * a.out_stride + n0] = acc[q][0];
          a.out[(size_t)tok * a.out_stride + n8] = acc[q][1];
          if (EPI == kEpilogueHead) {
            const unsigned long long k0 = head_key(acc[q][0], n0), k8 = head_key(acc[q][1], n8);
            best[q] = max(best[q], max(k0, k8));
          }
        }
      }
    }
    pdl_launch_dependents();
    if (EPI == kEpilogueHead) {
#pragma unroll
      for (int q = 0; q < MQ; q++) {
        unsigned long long b = best[q];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
        const int tok = 4 * q + t;
        if (g == 0 && tok < M && b) atomicMax(a.head.argmax + tok, b);
      }
    }
  } else {
    // CTA mode: the CTA's warps split K (and, with a cluster, so do its CTAs);
    // partials meet in shared memory, in a fixed order.
    const uint32_t rgl = warp / geo.KS, ks = warp % geo.KS;
    const uint32_t S = geo.KS * geo.C, slice = geo.rank * geo.KS + ks;
    const int bp0 = (int)(slice * geo.NBP / S), bp1 = (int)((slice + 1) * geo.NBP / S);
    const Q4Matrix& mat = EPI == kEpilogueGated ? a.mat[rgl & 1] : a.mat[0];
    const uint32_t stride = gridDim.x / geo.C;
    uint32_t rowset = blockIdx.x / geo.C;
    auto rg_of = [&](uint32_t rs) { return EPI == kEpilogueGated ? rs : rs * geo.RG + rgl; };
    auto live_of = [&](uint32_t rs) { return rgl < geo.RG && rs < geo.nrowsets && rg_of(rs) < mat.n / 16 && bp0 < bp1; };
    if (live_of(rowset)) {
      const uint32_t rg = rg_of(rowset);
      load_batch(mat.codes + (size_t)rg * geo.NBP * 32, mat.scales + (size_t)rg * geo.NBP * 8, bp0, bp1, lane, first);
    }
    pdl_wait();
    prologue<MQ, PRO>(a, sm, geo);
    const int rows_padded = 4 * MQ;
    const int outs = (int)geo.RG * 16 * rows_padded;
    for (; rowset < geo.nrowsets; rowset += stride) {
#pragma unroll
      for (int q = 0; q < MQ; q++) acc[q][0] = acc[q][1] = 0.f;
      if (live_of(rowset)) {
        const uint32_t rg = rg_of(rowset);
        rowgroup_dot<MQ>(mat.codes + (size_t)rg * geo.NBP * 32, mat.scales + (size_t)rg * geo.NBP * 8, bp0, bp1, sm.xf,
                         geo.kb_base, lane, first, acc);
      }
      if (live_of(rowset + stride)) {
        const uint32_t rg = rg_of(rowset + stride);
        load_batch(mat.codes + (size_t)rg * geo.NBP * 32, mat.scales + (size_t)rg * geo.NBP * 8, bp0, bp1, lane, first);
      }
      if (rgl < geo.RG) {
        float* red = sm.red + (rgl * geo.KS + ks) * 256;
#pragma unroll
        for (int q = 0; q < MQ; q++) {
          red[g * 16 + 4 * q + t] = acc[q][0];
          red[(g + 8) * 16 + 4 * q + t] = acc[q][1];
        }
      }
      __syncthreads();
      if (geo.C > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        float* dst = cluster.map_shared_rank(sm.cred, 0);
        for (int i = threadIdx.x; i < outs; i += kThreads) {
          const int rr = i / (16 * rows_padded), rest = i % (16 * rows_padded);
          const int row = rest / rows_padded, tok = rest % rows_padded;
          float v = 0.f;
          for (uint32_t k2 = 0; k2 < geo.KS; k2++) v = add(v, sm.red[(rr * geo.KS + k2) * 256 + row * 16 + tok]);
          dst[geo.rank * outs + i] = v;
        }
        cluster.sync();
      }
      auto final_value = [&](int rr, int row, int tok) -> float {
        float v = 0.f;
        if (geo.C > 1) {
          const int i = (rr * 16 + row) * rows_padded + tok;
          for (uint32_t c2 = 0; c2 < geo.C; c2++) v = add(v, sm.cred[c2 * outs + i]);
        } else {
          for (uint32_t k2 = 0; k2 < geo.KS; k2++) v = add(v, sm.red[(rr * geo.KS + k2) * 256 + row * 16 + tok]);
        }
        return v;
      };
      if (geo.rank == 0) {
        if (EPI == kEpilogueWrite || EPI == kEpilogueQkv) {
          for (int i = threadIdx.x; i < (int)geo.RG * 16 * M; i += kThreads) {
            const int rr = i / (16 * M), rest = i % (16 * M), tok = rest / 16, row = rest % 16;
            const uint32_t rgi = rowset * geo.RG + rr;
            if (rgi < mat.n / 16) a.out[(size_t)tok * a.out_stride + rgi * 16 + row] = final_value(rr, row, tok);
          }
        } else if (EPI == kEpilogueGated) {
          for (int i = threadIdx.x; i < 16 * M; i += kThreads) {
            const int tok = i / 16, row = i % 16;
            const uint32_t neuron = rowset * 16 + row;
            const float gate = final_value(0, row, tok), up = final_value(1, row, tok);
            float v = mul(gelu_tanh(gate), up);
            const uint32_t seq = (uint32_t)tok / a.seq_tokens;
            const uint32_t pos = (a.step ? a.step->position : a.position) + (uint32_t)tok % a.seq_tokens;
            if (a.edit.table) v = apply_edits(a.edit.table + seq * a.edit.table_stride, a.edit.layer, neuron, pos, v);
            a.out[(size_t)tok * a.out_stride + neuron] = v;
            if (a.edit.capture_neurons && (uint32_t)tok % a.seq_tokens == a.seq_tokens - 1)
              a.edit.capture_neurons[seq * a.capture_stride + neuron] = v;
          }
        } else if (EPI == kEpilogueHead) {
          for (int i = threadIdx.x; i < (int)geo.RG * 16 * M; i += kThreads) {
            const int tok = i / (geo.RG * 16), rest = i % (geo.RG * 16), rr = rest / 16, row = rest % 16;
            const uint32_t n = (rowset * geo.RG + rr) * 16 + row;
            if (n < mat.n) {
              const float v = final_value(rr, row, tok);
              a.out[(size_t)tok * a.out_stride + n] = v;
              atomicMax(&s_best[tok], head_key(v, n));
            }
          }
        }
      }
      // The partials are rewritten by the next rowset.
      if (geo.C > 1) cg::this_cluster().sync();
      else __syncthreads();
    }
    pdl_launch_dependents();
    if (EPI == kEpilogueHead) {
      __syncthreads();
      if (geo.rank == 0 && threadIdx.x < M && s_best[threadIdx.x]) atomicMax(a.head.argmax + threadIdx.x, s_best[threadIdx.x]);
    }
    if (geo.C > 1 && geo.rank != 0) return;
  }

  if (EPI == kEpilogueQkv) {
    // The last CTA to finish runs QK-norm, RoPE and the KV append over every
    // row and head (rope_cache.wgsl:16-91).
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const uint32_t writers = gridDim.x / geo.C;
      s_last = atomicAdd(a.counter, 1u) == writers - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const RopeArgs& r = a.rope;
    const int heads = (int)(r.heads + 2 * r.kv_heads);
    for (int item = warp; item < M * heads; item += kWarps) {
      const int row = item / heads, head = item % heads;
      const uint32_t seq = (uint32_t)row / a.seq_tokens;
      const uint32_t pos = (a.step ? a.step->position : a.position) + (uint32_t)row % a.seq_tokens;
      float* cq = (r.capture_query && (uint32_t)row % a.seq_tokens == a.seq_tokens - 1)
                      ? r.capture_query + seq * a.capture_stride
                      : nullptr;
      rope_head_warp(r, a.out, a.out_stride, row, head, seq, pos, cq, lane);
    }
    if (threadIdx.x == 0) *a.counter = 0u;
  }
}

// ---------------------------------------------------------------- wide steps

// The norm launch for many rows, one CTA a row (norm.wgsl:97-198): X after
// the add to hidden_out, the normed row as f16 hi (and lo) for the tensor-core
// products, the captures of each sequence's last row.
__global__ void __launch_bounds__(kThreads) norm_f16_kernel(const MatvecArgs a, __half* out_hi, __half* out_lo) {
  __shared__ __align__(16) float rowbuf[8192];
  __shared__ float part[kThreads];
  __shared__ float stat[2 * kMaxTokens];
  pdl_wait();
  NormArgs n = a.norm;
  n.row_of_token_stride = 1;
  n.row_of_token_offset = blockIdx.x;
  norm_rows_cta(a, n, 1, rowbuf, part, stat, true);
  const int W = (int)n.width;
  __half* hi = out_hi + (size_t)blockIdx.x * W;
  __half* lo = out_lo ? out_lo + (size_t)blockIdx.x * W : nullptr;
  for (int i = threadIdx.x; i < W; i += kThreads) {
    const float v = rowbuf[i];
    const __half h = __float2half_rn(v);
    hi[i] = h;
    if (lo) lo[i] = __float2half_rn(__fsub_rn(v, __half2float(h)));
  }
  pdl_launch_dependents();
}

// The same for rows of a width that is a multiple of 128 (up to 2048): a warp
// a row, the row's NV float4s a lane in registers, every load of the row in
// flight at once and each sum of squares a warp shuffle reduction, so no CTA
// barrier sits between the loads and the stores (the one-CTA-a-row form
// above runs two 256-invocation trees with a barrier a level).  The
// per-element formulas are the norm's; only the order of the two sums of
// squares differs (a few f32 roundings of the statistics).
template <int NV>
__global__ void __launch_bounds__(kThreads) norm_rows_warp_kernel(const MatvecArgs a, __half* out_hi,
                                                                  __half* out_lo) {
  // The gains are weights, not the previous launch's output: staged in
  // shared memory before waiting for it.
  __shared__ float4 gsm[2][NV * 32];
  {
    const float4* g4 = reinterpret_cast<const float4*>(a.norm.gain);
    const float4* p4 = reinterpret_cast<const float4*>(a.norm.post_gain);
    for (int i = threadIdx.x; i < NV * 32; i += kThreads) {
      gsm[0][i] = g4[i];
      if (p4) gsm[1][i] = p4[i];
    }
  }
  pdl_wait();
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t row = blockIdx.x * kWarps + warp;
  if (row < a.m) {
    const NormArgs& n = a.norm;
    const uint32_t W = n.width;
    // (1 / width, rounded once: each reciprocal RMS is one multiply-add and
    // the hardware reciprocal square root, within 2e-7 of a division and an
    // IEEE square root)
    const float inv_w = __frcp_rn((float)W);
    const float4* x4 = reinterpret_cast<const float4*>(n.hidden_in + (size_t)row * W);
    float4 x[NV], y[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) x[i] = x4[lane + 32 * i];
    if (n.y) {
      const float* yr = n.y + (size_t)row * W;
#pragma unroll
      for (int i = 0; i < NV; i++) y[i] = y_sum(n, yr, lane + 32 * i);
    }
    const uint32_t seq = row / a.seq_tokens;
    const bool last = row % a.seq_tokens == a.seq_tokens - 1;
    if (n.y) {
      if (n.post_gain) {
        float p = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) p = add(p, dot_self(y[i]));
        const float s = rsqrtf(__fmaf_rn(warp_sum(p), inv_w, n.eps));
#pragma unroll
        for (int i = 0; i < NV; i++) {
          const float4 g = gsm[1][lane + 32 * i];
          y[i] = make_float4(mul(mul(y[i].x, s), g.x), mul(mul(y[i].y, s), g.y), mul(mul(y[i].z, s), g.z),
                             mul(mul(y[i].w, s), g.w));
        }
      }
      float4* ycap = last && n.capture_added ? reinterpret_cast<float4*>(n.capture_added + seq * a.capture_stride)
                                             : nullptr;
#pragma unroll
      for (int i = 0; i < NV; i++) {
        if (ycap) ycap[lane + 32 * i] = y[i];
        x[i] = make_float4(add(x[i].x, y[i].x), add(x[i].y, y[i].y), add(x[i].z, y[i].z), add(x[i].w, y[i].w));
      }
    }
    float4* out4 = n.hidden_out ? reinterpret_cast<float4*>(n.hidden_out + (size_t)row * W) : nullptr;
    float4* xcap = last && n.capture_residual
                       ? reinterpret_cast<float4*>(n.capture_residual + seq * a.capture_stride) : nullptr;
    float p = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      if (out4) out4[lane + 32 * i] = x[i];
      if (xcap) xcap[lane + 32 * i] = x[i];
      p = add(p, dot_self(x[i]));
    }
    const float s = rsqrtf(__fmaf_rn(warp_sum(p), inv_w, n.eps));
    uint2* hi = reinterpret_cast<uint2*>(out_hi + (size_t)row * W);
    uint2* lo = out_lo ? reinterpret_cast<uint2*>(out_lo + (size_t)row * W) : nullptr;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const float4 g = gsm[0][lane + 32 * i];
      const float v[4] = {mul(mul(x[i].x, s), g.x), mul(mul(x[i].y, s), g.y), mul(mul(x[i].z, s), g.z),
                          mul(mul(x[i].w, s), g.w)};
      uint2 h, l;
      split2(v[0], v[1], h.x, l.x);
      split2(v[2], v[3], h.y, l.y);
      hi[lane + 32 * i] = h;
      if (lo) lo[lane + 32 * i] = l;
    }
  }
  pdl_launch_dependents();
}

// The norm prologue's rows as f32 (CTA i: the row the prologue would read for
// slot i), for a product that takes f32 x (the Q8_0 head).
__global__ void __launch_bounds__(kThreads) norm_f32_kernel(const MatvecArgs a, float* out) {
  __shared__ __align__(16) float rowbuf[8192];
  __shared__ float part[kThreads];
  __shared__ float stat[2 * kMaxTokens];
  pdl_wait();
  NormArgs n = a.norm;
  n.row_of_token_offset = a.norm.row_of_token_offset + blockIdx.x * a.norm.row_of_token_stride;
  n.row_of_token_stride = 1;
  norm_rows_cta(a, n, 1, rowbuf, part, stat, true);
  const int W = (int)n.width;
  for (int i = threadIdx.x; i < W; i += kThreads) out[(size_t)blockIdx.x * W + i] = rowbuf[i];
  pdl_launch_dependents();
}

// QK-norm, RoPE and the KV append for many rows: one warp a (row, head).
__global__ void __launch_bounds__(kThreads) rope_rows_kernel(const MatvecArgs a) {
  pdl_wait();
  const RopeArgs& r = a.rope;
  const int heads = (int)(r.heads + 2 * r.kv_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int item = blockIdx.x * kWarps + warp;
  if (item < (int)a.m * heads) {
    const int row = item / heads, head = item % heads;
    const uint32_t seq = (uint32_t)row / a.seq_tokens;
    const uint32_t pos = (a.step ? a.step->position : a.position) + (uint32_t)row % a.seq_tokens;
    float* cq = (r.capture_query && (uint32_t)row % a.seq_tokens == a.seq_tokens - 1)
                    ? r.capture_query + seq * a.capture_stride
                    : nullptr;
    rope_head_warp(r, a.out, a.out_stride, row, head, seq, pos, cq, lane);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------- repack

__global__ void repack_kernel(const uint8_t* __restrict__ file, uint32_t n, uint32_t k, uint4* codes,
                              uint2* scales) {
  const uint32_t NBP = k / 64, KB = k / 32;
  const size_t total = (size_t)(n / 16) * NBP * 32;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t lane = (uint32_t)(i % 32), bp = (uint32_t)((i / 32) % NBP), rg = (uint32_t)(i / 32 / NBP);
    const uint32_t g = lane >> 2, t = lane & 3;
    const size_t row0 = (size_t)rg * 16 + g, row8 = row0 + 8;
    uint32_t w[4];
#pragma unroll
    for (int kbi = 0; kbi < 2; kbi++) {
      const uint32_t kb = 2 * bp + kbi;
      const uint8_t* b0 = file + (row0 * KB + kb) * 18 + 2;
      const uint8_t* b8 = file + (row8 * KB + kb) * 18 + 2;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int j = 8 * h + 2 * t;
        w[kbi * 2 + h] = (uint32_t)b0[j] | ((uint32_t)b8[j] << 8) | ((uint32_t)b0[j + 1] << 16) |
                         ((uint32_t)b8[j + 1] << 24);
      }
    }
    codes[i] = make_uint4(w[0], w[1], w[2], w[3]);
    if (t == 0) {
      auto scale = [&](size_t row, uint32_t kb) -> uint32_t {
        const uint8_t* p = file + (row * KB + kb) * 18;
        return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
      };
      const uint32_t kb = 2 * bp;
      scales[((size_t)rg * NBP + bp) * 8 + g] =
          make_uint2(scale(row0, kb) | (scale(row8, kb) << 16), scale(row0, kb + 1) | (scale(row8, kb + 1) << 16));
    }
  }
}

// Rows of a fragment-layout matrix back to f32 weights times `scale`
// (gather.wgsl:25-48 over the layout; the embedding's row is (code - 8) * d,
// exact, times sqrt(width) in f32).
__global__ void dequant_rows_kernel(Q4Matrix mat, const uint32_t* rows, uint32_t count, float scale, float* out) {
  const uint32_t NBP = mat.k / 64, KB = mat.k / 32;
  const uint32_t i = blockIdx.x;
  if (i >= count) return;
  const uint32_t r = rows[i];
  if (r >= mat.n) return;
  const uint32_t rg = r / 16, rr = r % 16, g = rr % 8, hsel = rr / 8;
  for (uint32_t j = threadIdx.x; j < KB * 8; j += blockDim.x) {
    const uint32_t kb = j / 8, h = (j / 4) % 2, t = j % 4;
    const uint32_t bp = kb / 2, kbi = kb % 2;
    const uint4 c = mat.codes[((size_t)rg * NBP + bp) * 32 + g * 4 + t];
    const uint32_t w = (kbi * 2 + h == 0) ? c.x : (kbi * 2 + h == 1) ? c.y : (kbi * 2 + h == 2) ? c.z : c.w;
    const uint2 sc = mat.scales[((size_t)rg * NBP + bp) * 8 + g];
    const uint32_t sw = kbi ? sc.y : sc.x;
    const float d = __half2float(__ushort_as_half((unsigned short)(hsel ? sw >> 16 : sw & 0xffffu)));
    const uint32_t q0 = (w >> (8 * hsel)) & 0xffu, q1 = (w >> (16 + 8 * hsel)) & 0xffu;
    const uint32_t k0 = 32 * kb + 8 * h + 2 * t;
    float* o = out + (size_t)i * mat.k;
    o[k0] = mul(mul((float)(q0 & 0xF) - 8.0f, d), scale);
    o[k0 + 1] = mul(mul((float)(q1 & 0xF) - 8.0f, d), scale);
    o[k0 + 16] = mul(mul((float)(q0 >> 4) - 8.0f, d), scale);
    o[k0 + 17] = mul(mul((float)(q1 >> 4) - 8.0f, d), scale);
  }
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int MQ, int PRO, int EPI>
int blocks_per_sm(size_t smem) {
  static std::mutex mu;
  static std::map<size_t, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(smem);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, matvec_kernel<MQ, PRO, EPI>, kThreads, smem) != cudaSuccess ||
      n < 1) {
    (void)cudaGetLastError();
    n = 1;
  }
  cache[smem] = n;
  return n;
}

template <int MQ, int PRO, int EPI>
cudaError_t launch_one(const MatvecArgs& a, cudaStream_t stream, bool pdl) {
  const uint32_t NBP = a.mat[0].k / 64;
  const uint32_t C = a.cluster, RG = a.rg_per_cta, KS = a.k_split;
  if (RG * KS != (uint32_t)kWarps || (EPI == kEpilogueGated && RG != 2) || C < 1 || C > 8) return cudaErrorInvalidValue;
  const size_t nkb_max = 2 * ((NBP + C - 1) / C);
  const size_t outs = (size_t)RG * 16 * 4 * MQ;
  const size_t smem = nkb_max * 2 * MQ * 32 * sizeof(uint2) + (size_t)RG * KS * 256 * 4 +
                      (PRO == kPrologueNorm ? (size_t)a.m * a.norm.width * 4 + (size_t)a.m * kThreads * 4 : 0) +
                      2 * kMaxTokens * 4 + (C > 1 ? C * outs * 4 : 0);
  const bool warp_mode = KS == 1 && C == 1 && EPI != kEpilogueGated;
  const uint32_t cap = (uint32_t)(sm_count() * blocks_per_sm<MQ, PRO, EPI>(smem));
  uint32_t grid;
  if (warp_mode) {
    grid = std::min<uint32_t>((a.mat[0].n / 16 + kWarps - 1) / kWarps, cap);
  } else {
    const uint32_t rowsets = EPI == kEpilogueGated ? a.mat[0].n / 16 : (a.mat[0].n / 16 + RG - 1) / RG;
    grid = std::min<uint32_t>(rowsets, std::max<uint32_t>(1, cap / C)) * C;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (C > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = C;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    na++;
  }
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, matvec_kernel<MQ, PRO, EPI>, a);
  if (e != cudaSuccess) (void)cudaGetLastError();  // the error is returned, not left behind
  return e;
}

template <int MQ, int PRO, int EPI>
cudaError_t configure_one() {
  return cudaFuncSetAttribute(matvec_kernel<MQ, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

template <int PRO, int EPI>
cudaError_t configure_mq() {
  cudaError_t e;
  if ((e = configure_one<1, PRO, EPI>()) != cudaSuccess) return e;
  if ((e = configure_one<2, PRO, EPI>()) != cudaSuccess) return e;
  if ((e = configure_one<3, PRO, EPI>()) != cudaSuccess) return e;
  return configure_one<4, PRO, EPI>();
}

template <int PRO, int EPI>
cudaError_t launch_mq(const MatvecArgs& a, cudaStream_t s, bool pdl) {
  switch ((a.m + 3) / 4) {
    case 1: return launch_one<1, PRO, EPI>(a, s, pdl);
    case 2: return launch_one<2, PRO, EPI>(a, s, pdl);
    case 3: return launch_one<3, PRO, EPI>(a, s, pdl);
    case 4: return launch_one<4, PRO, EPI>(a, s, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t configure_kernels() {
  cudaError_t e;
  if ((e = configure_mq<kPrologueInput, kEpilogueWrite>()) != cudaSuccess) return e;
  if ((e = configure_mq<kPrologueInput, kEpilogueQkv>()) != cudaSuccess) return e;
  if ((e = configure_mq<kPrologueInput, kEpilogueGated>()) != cudaSuccess) return e;
  if ((e = configure_mq<kPrologueInput, kEpilogueHead>()) != cudaSuccess) return e;
  if ((e = configure_mq<kPrologueNorm, kEpilogueWrite>()) != cudaSuccess) return e;
  if ((e = configure_mq<kPrologueNorm, kEpilogueQkv>()) != cudaSuccess) return e;
  if ((e = configure_mq<kPrologueNorm, kEpilogueGated>()) != cudaSuccess) return e;
  return configure_mq<kPrologueNorm, kEpilogueHead>();
}

// Raises the shared-memory limits once per device, on first use there.
cudaError_t ensure_configured() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return cudaSuccess;
  e = configure_kernels();
  if (e == cudaSuccess) done[dev] = true;
  return e;
}

cudaError_t launch_matvec(const MatvecArgs& a, int prologue, int epilogue, cudaStream_t stream, bool pdl) {
  if (a.m < 1 || a.m > (uint32_t)kMaxTokens) return cudaErrorInvalidValue;
  cudaError_t ce = ensure_configured();
  if (ce != cudaSuccess) return ce;
  if (prologue == kPrologueInput) {
    switch (epilogue) {
      case kEpilogueWrite: return launch_mq<kPrologueInput, kEpilogueWrite>(a, stream, pdl);
      case kEpilogueQkv: return launch_mq<kPrologueInput, kEpilogueQkv>(a, stream, pdl);
      case kEpilogueGated: return launch_mq<kPrologueInput, kEpilogueGated>(a, stream, pdl);
      case kEpilogueHead: return launch_mq<kPrologueInput, kEpilogueHead>(a, stream, pdl);
    }
  } else {
    switch (epilogue) {
      case kEpilogueWrite: return launch_mq<kPrologueNorm, kEpilogueWrite>(a, stream, pdl);
      case kEpilogueQkv: return launch_mq<kPrologueNorm, kEpilogueQkv>(a, stream, pdl);
      case kEpilogueGated: return launch_mq<kPrologueNorm, kEpilogueGated>(a, stream, pdl);
      case kEpilogueHead: return launch_mq<kPrologueNorm, kEpilogueHead>(a, stream, pdl);
    }
  }
  return cudaErrorInvalidValue;
}

namespace {
cudaError_t launch_plain(const void* fn, dim3 grid, dim3 block, cudaStream_t stream, bool pdl, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  if (e != cudaSuccess) (void)cudaGetLastError();
  return e;
}
}  // namespace

template <int NV>
const void* norm_warp_fn() {
  return (const void*)norm_rows_warp_kernel<NV>;
}

cudaError_t launch_norm_f16(const MatvecArgs& a, __half* out_hi, __half* out_lo, cudaStream_t stream, bool pdl) {
  if (a.norm.width > 8192 || a.norm.width % 4 || a.m == 0) return cudaErrorInvalidValue;
  MatvecArgs copy = a;
  void* args[] = {&copy, &out_hi, &out_lo};
  // A warp a row for widths of 128 .. 2048 in 128s (both forms take rows 0 .. m - 1).
  const void* warp_fn = nullptr;
  if (a.norm.width % 128 == 0) {
    switch (a.norm.width / 128) {
      case 1: warp_fn = norm_warp_fn<1>(); break;
      case 2: warp_fn = norm_warp_fn<2>(); break;
      case 3: warp_fn = norm_warp_fn<3>(); break;
      case 4: warp_fn = norm_warp_fn<4>(); break;
      case 5: warp_fn = norm_warp_fn<5>(); break;
      case 6: warp_fn = norm_warp_fn<6>(); break;
      case 7: warp_fn = norm_warp_fn<7>(); break;
      case 8: warp_fn = norm_warp_fn<8>(); break;
      case 9: warp_fn = norm_warp_fn<9>(); break;
      case 10: warp_fn = norm_warp_fn<10>(); break;
      case 11: warp_fn = norm_warp_fn<11>(); break;
      case 12: warp_fn = norm_warp_fn<12>(); break;
      case 13: warp_fn = norm_warp_fn<13>(); break;
      case 14: warp_fn = norm_warp_fn<14>(); break;
      case 15: warp_fn = norm_warp_fn<15>(); break;
      case 16: warp_fn = norm_warp_fn<16>(); break;
      default: break;
    }
  }
  if (warp_fn) return launch_plain(warp_fn, dim3((a.m + kWarps - 1) / kWarps), dim3(kThreads), stream, pdl, args);
  return launch_plain((const void*)norm_f16_kernel, dim3(a.m), dim3(kThreads), stream, pdl, args);
}

cudaError_t launch_norm_f32(const MatvecArgs& a, float* out, cudaStream_t stream, bool pdl) {
  if (a.norm.width > 8192 || a.norm.width % 4 || a.m == 0) return cudaErrorInvalidValue;
  MatvecArgs copy = a;
  void* args[] = {&copy, &out};
  return launch_plain((const void*)norm_f32_kernel, dim3(a.m), dim3(kThreads), stream, pdl, args);
}

cudaError_t launch_rope_rows(const MatvecArgs& a, cudaStream_t stream, bool pdl) {
  if (a.rope.head_dim != 256 || a.m == 0) return cudaErrorInvalidValue;
  const uint32_t items = a.m * (a.rope.heads + 2 * a.rope.kv_heads);
  MatvecArgs copy = a;
  void* args[] = {&copy};
  return launch_plain((const void*)rope_rows_kernel, dim3((items + kWarps - 1) / kWarps), dim3(kThreads), stream, pdl,
                      args);
}

cudaError_t launch_repack(const uint8_t* file_blocks, uint32_t n, uint32_t k, uint4* codes, uint2* scales,
                          cudaStream_t stream) {
  if (n % 16 || k % 64) return cudaErrorInvalidValue;
  const size_t total = (size_t)(n / 16) * (k / 64) * 32;
  const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  (void)cudaGetLastError();
  repack_kernel<<<blocks, 256, 0, stream>>>(file_blocks, n, k, codes, scales);
  return cudaGetLastError();
}

cudaError_t launch_dequant_rows(const Q4Matrix& mat, const uint32_t* rows, uint32_t count, float scale, float* out,
                                cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  (void)cudaGetLastError();
  dequant_rows_kernel<<<count, 256, 0, stream>>>(mat, rows, count, scale, out);
  return cudaGetLastError();
}

}  // namespace fz
