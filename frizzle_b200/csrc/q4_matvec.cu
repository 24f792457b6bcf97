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

#include <mutex>

#include "q4_matvec.cuh"

namespace cg = cooperative_groups;

namespace fz {
namespace {

FZ_DEV uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
FZ_DEV __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Four A registers (rows g, g+8 x the permuted columns) from one code word:
// 0x6400 | n is the half 1024 + n, less 1032 gives n - 8 exactly.
FZ_DEV void dequant_word(uint32_t w, uint32_t a[4]) {
  const uint32_t kMask = 0x000F000Fu, kMagic = 0x64006400u;
  const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6408u));
  a[0] = h2_bits(__hsub2(bits_h2((w & kMask) | kMagic), bias));
  a[1] = h2_bits(__hsub2(bits_h2(((w >> 8) & kMask) | kMagic), bias));
  a[2] = h2_bits(__hsub2(bits_h2(((w >> 4) & kMask) | kMagic), bias));
  a[3] = h2_bits(__hsub2(bits_h2(((w >> 12) & kMask) | kMagic), bias));
}

FZ_DEV void mma16816(float d[4], const uint32_t a[4], uint2 b, const float c[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

FZ_DEV uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
FZ_DEV uint2 ld_stream2(const uint2* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
FZ_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  if (bytes) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// hi/lo f16 pair of an f32 value.
FZ_DEV void split_hi_lo(float v, __half& hi, __half& lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
}

FZ_DEV uint2 pack4(__half a, __half b, __half c, __half d) {
  return make_uint2(h2_bits(__halves2half2(a, b)), h2_bits(__halves2half2(c, d)));
}

// B fragments of 4 rows of X (one "quad") for block kb, half h: lane (g, t)
// reads slot t*8 + g; column g is row 4q + g/2 of X, its hi part for even g and
// its lo part for odd g; its four values are X at columns 32kb + 8h + 2t + {0, 1}
// and 32kb + 16 + 8h + 2t + {0, 1} (the layout's column permutation).
FZ_DEV int xf_index(int kb_rel, int h, int q, int MQ, int t, int g) {
  return ((kb_rel * 2 + h) * MQ + q) * 32 + t * 8 + g;
}

// Writes the fragments of X row `row` (values in `src`, K floats) for blocks
// [kb_base, kb_base + nkb), or zeros when src is null.  Threads of the CTA
// share the work from index `first` with stride `step`.
FZ_DEV void build_fragments(uint2* xf, int MQ, int row, const float* src, int kb_base, int nkb, int first,
                            int step) {
  const int q = row >> 2, gp = row & 3;
  for (int i = first; i < nkb * 8; i += step) {
    const int kb_rel = i >> 3, h = (i >> 2) & 1, t = i & 3;
    uint2 hi = make_uint2(0, 0), lo = make_uint2(0, 0);
    if (src) {
      const int k0 = 32 * (kb_base + kb_rel) + 8 * h + 2 * t;
      const float2 v01 = *reinterpret_cast<const float2*>(src + k0);
      const float2 v23 = *reinterpret_cast<const float2*>(src + k0 + 16);
      __half h0, h1, h2, h3, l0, l1, l2, l3;
      split_hi_lo(v01.x, h0, l0);
      split_hi_lo(v01.y, h1, l1);
      split_hi_lo(v23.x, h2, l2);
      split_hi_lo(v23.y, h3, l3);
      hi = pack4(h0, h1, h2, h3);
      lo = pack4(l0, l1, l2, l3);
    }
    xf[xf_index(kb_rel, h, q, MQ, t, 2 * gp)] = hi;
    xf[xf_index(kb_rel, h, q, MQ, t, 2 * gp + 1)] = lo;
  }
}

// One warp's sums for its row group over block pairs [bp0, bp1): lane (g, t)
// ends with acc[q][0] = row g and acc[q][1] = row g + 8 against X row 4q + t.
template <int MQ>
FZ_DEV void rowgroup_dot(const uint4* codes, const uint2* scales, int bp0, int bp1, const uint2* xf,
                         int kb_base, int lane, float acc[MQ][2]) {
  const int g = lane >> 2, t = lane & 3;
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
  constexpr int U = 4;
  for (int bp = bp0; bp < bp1; bp += U) {
    uint4 c[U];
    uint2 s[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (bp + u < bp1) {
        c[u] = ld_stream(codes + (size_t)(bp + u) * 32 + lane);
        s[u] = ld_stream2(scales + (size_t)(bp + u) * 8 + g);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (bp + u < bp1) {
#pragma unroll
        for (int kbi = 0; kbi < 2; kbi++) {
          const int kb_rel = 2 * (bp + u) + kbi - kb_base;
          uint32_t a0[4], a1[4];
          dequant_word(kbi ? c[u].z : c[u].x, a0);
          dequant_word(kbi ? c[u].w : c[u].y, a1);
          const uint32_t sw = kbi ? s[u].y : s[u].x;
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
}

// The norm of one row by one warp into `buf` (norm.wgsl:97-198): y through
// its post-norm added into x, then (x * r) * gain.  `buf` ends holding the
// normed row; `xout` and `xcap` (if non-null) receive x after the add, `yadd`
// y as added.
FZ_DEV void norm_row_warp(const NormArgs& n, int row, float* buf, float* xout, float* xcap, float* yadd,
                          int lane) {
  const int W = n.width, V = W / 4;
  float4* b4 = reinterpret_cast<float4*>(buf);
  const float inv_n = (float)W;
  if (n.y) {
    const float4* y4 = reinterpret_cast<const float4*>(n.y + (size_t)row * W);
    for (int v = lane; v < V; v += 32) b4[v] = y4[v];
    __syncwarp();
    if (n.post_gain) {
      const float r = inverse_sqrt(add(__fdiv_rn(norm_sum_squares_warp(b4, V, lane), inv_n), n.eps));
      const float4* pg = reinterpret_cast<const float4*>(n.post_gain);
      __syncwarp();
      for (int v = lane; v < V; v += 32) {
        float4 y = b4[v], p = pg[v];
        b4[v] = make_float4(mul(mul(y.x, r), p.x), mul(mul(y.y, r), p.y), mul(mul(y.z, r), p.z),
                            mul(mul(y.w, r), p.w));
      }
    }
    const float4* x4 = reinterpret_cast<const float4*>(n.hidden_in + (size_t)row * W);
    for (int v = lane; v < V; v += 32) {
      float4 y = b4[v], x = x4[v];
      if (yadd) reinterpret_cast<float4*>(yadd)[v] = y;
      b4[v] = make_float4(add(x.x, y.x), add(x.y, y.y), add(x.z, y.z), add(x.w, y.w));
    }
  } else {
    const float4* x4 = reinterpret_cast<const float4*>(n.hidden_in + (size_t)row * W);
    for (int v = lane; v < V; v += 32) b4[v] = x4[v];
  }
  __syncwarp();
  if (xout)
    for (int v = lane; v < V; v += 32) reinterpret_cast<float4*>(xout)[v] = b4[v];
  if (xcap)
    for (int v = lane; v < V; v += 32) reinterpret_cast<float4*>(xcap)[v] = b4[v];
  const float r = inverse_sqrt(add(__fdiv_rn(norm_sum_squares_warp(b4, V, lane), inv_n), n.eps));
  __syncwarp();
  const float4* g4 = reinterpret_cast<const float4*>(n.gain);
  for (int v = lane; v < V; v += 32) {
    float4 x = b4[v], gg = g4[v];
    b4[v] = make_float4(mul(mul(x.x, r), gg.x), mul(mul(x.y, r), gg.y), mul(mul(x.z, r), gg.z),
                        mul(mul(x.w, r), gg.w));
  }
  __syncwarp();
}

// QK-norm, RoPE and the f16 KV append for one (row, head) by one warp
// (rope.wgsl:40-138, rope_cache.wgsl:16-91, d = 256: lane l holds the head's
// elements 4l..4l+3 and 128+4l..128+4l+3).
FZ_DEV void rope_head_warp(const RopeArgs& r, const float* raw, uint32_t raw_stride, int row, int head,
                           uint32_t seq, uint32_t pos, float* capture_query, int lane) {
  const int d = (int)r.head_dim, H = (int)r.heads, KV = (int)r.kv_heads;
  const bool is_query = head < H, is_value = head >= H + KV;
  const int kvh = is_query ? 0 : (is_value ? head - H - KV : head - H);
  const int col = is_query ? head * d : (is_value ? H * d + KV * d + kvh * d : H * d + kvh * d);
  const float* src = raw + (size_t)row * raw_stride + col;
  float4 a = __ldcg(reinterpret_cast<const float4*>(src) + lane);
  float4 b = __ldcg(reinterpret_cast<const float4*>(src + d / 2) + lane);
  if (!is_value) {
    float s = add(dot_self(a), dot_self(b));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float other = __shfl_down_sync(0xffffffffu, s, o);
      if (lane < o) s = add(s, other);
    }
    s = __shfl_sync(0xffffffffu, s, 0);
    const float rr = inverse_sqrt(add(__fdiv_rn(s, (float)d), r.eps));
    const float* gain = is_query ? r.q_gain : r.k_gain;
    const float4 ga = reinterpret_cast<const float4*>(gain)[lane];
    const float4 gb = reinterpret_cast<const float4*>(gain + d / 2)[lane];
    a = make_float4(mul(mul(a.x, rr), ga.x), mul(mul(a.y, rr), ga.y), mul(mul(a.z, rr), ga.z),
                    mul(mul(a.w, rr), ga.w));
    b = make_float4(mul(mul(b.x, rr), gb.x), mul(mul(b.y, rr), gb.y), mul(mul(b.z, rr), gb.z),
                    mul(mul(b.w, rr), gb.w));
    const float tau = (float)6.283185307179586;
    float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const float tt = mul((float)pos, r.turns[4 * lane + c]);
      const float angle = mul(tau, sub(tt, rintf(tt)));
      float sn, cs;
      sincosf(angle, &sn, &cs);
      const float x = av[c], y = bv[c];
      av[c] = sub(mul(x, cs), mul(y, sn));
      bv[c] = add(mul(x, sn), mul(y, cs));
    }
    a = make_float4(av[0], av[1], av[2], av[3]);
    b = make_float4(bv[0], bv[1], bv[2], bv[3]);
  }
  if (is_query) {
    float* q = r.query_out + (size_t)row * H * d + head * d;
    reinterpret_cast<float4*>(q)[lane] = a;
    reinterpret_cast<float4*>(q + d / 2)[lane] = b;
    if (capture_query) {
      reinterpret_cast<float4*>(capture_query + head * d)[lane] = a;
      reinterpret_cast<float4*>(capture_query + head * d + d / 2)[lane] = b;
    }
  } else {
    uint16_t* cache = (is_value ? r.value_cache : r.key_cache) + seq * r.seq_stride +
                      ((size_t)(pos % r.slots) * KV + kvh) * d;
    ushort4 pa = make_ushort4(f16_pack(a.x), f16_pack(a.y), f16_pack(a.z), f16_pack(a.w));
    ushort4 pb = make_ushort4(f16_pack(b.x), f16_pack(b.y), f16_pack(b.z), f16_pack(b.w));
    reinterpret_cast<ushort4*>(cache)[lane] = pa;
    reinterpret_cast<ushort4*>(cache + d / 2)[lane] = pb;
  }
}

// The edit kernel's rewrite of one neuron of one row (edit.wgsl:55-76): the
// layer's edits are sorted by neuron, so a binary search finds the neuron's.
FZ_DEV float apply_edits(const uint32_t* table, uint32_t layer, uint32_t neuron, uint32_t pos, float v) {
  const uint32_t first = table[2 * layer], count = table[2 * layer + 1];
  uint32_t lo = 0, hi = count;
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (table[first + 5 * mid] < neuron) lo = mid + 1; else hi = mid;
  }
  for (uint32_t i = lo; i < count; i++) {
    const uint32_t* e = table + first + 5 * i;
    if (e[0] != neuron) break;
    if (pos < e[3] || pos >= e[4]) continue;
    const float value = __uint_as_float(e[2]);
    float edited = value;  // Set, and Zero whose value is 0
    if (e[1] == 1u) edited = value == 1.0f ? v : mul(v, value);
    v = edited;
  }
  return v;
}

struct Smem {
  uint2* xf;
  float* red;
  float* rowbuf;
  float* cred;
};

template <int MQ, int PRO, int EPI>
__global__ void __launch_bounds__(256) matvec_kernel(const MatvecArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint32_t s_last;
  __shared__ unsigned long long s_best[kMaxTokens];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const uint32_t C = a.cluster, KS = a.k_split, RG = a.rg_per_cta;
  uint32_t rank = 0;
  if (C > 1) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const uint32_t rowset = blockIdx.x / C;
  const uint32_t K = a.mat[0].k, NBP = K / 64;
  const uint32_t rgl = warp / KS, ks = warp % KS;
  const uint32_t S = KS * C, slice = rank * KS + ks;
  const int bp0 = (int)(slice * NBP / S), bp1 = (int)((slice + 1) * NBP / S);
  const int cta_bp0 = (int)(rank * NBP / C), cta_bp1 = (int)((rank + 1) * NBP / C);
  const int kb_base = 2 * cta_bp0, nkb = 2 * (cta_bp1 - cta_bp0);
  const int M = (int)a.m;

  const Q4Matrix& mat = (EPI == kEpilogueGated) ? a.mat[rgl & 1] : a.mat[0];
  const uint32_t rg = (EPI == kEpilogueGated) ? rowset : rowset * RG + rgl;
  const bool live = rgl < RG && rg < mat.n / 16;
  const uint4* codes = mat.codes + (size_t)rg * NBP * 32;
  const uint2* scales = mat.scales + (size_t)rg * NBP * 8;

  // Smem carve-up.
  const int nkb_max = 2 * (int)((NBP + C - 1) / C);
  Smem sm;
  sm.xf = reinterpret_cast<uint2*>(smem_raw);
  sm.red = reinterpret_cast<float*>(sm.xf + nkb_max * 2 * MQ * 32);
  sm.rowbuf = sm.red + RG * KS * 256;
  const int norm_warps = PRO == kPrologueNorm ? min(nwarps, M) : 0;
  sm.cred = sm.rowbuf + norm_warps * (int)a.norm.width;

  // Weights do not depend on the previous kernel: start them toward L2 now.
  if (live && lane == 0) {
    prefetch_l2(codes + (size_t)bp0 * 32, (uint32_t)(bp1 - bp0) * 512u);
    prefetch_l2(scales + (size_t)bp0 * 8, (uint32_t)(bp1 - bp0) * 64u);
  }
  pdl_wait();

  // X rows as B fragments.
  const int rows_padded = 4 * MQ;
  if (PRO == kPrologueInput) {
    for (int r = 0; r < rows_padded; r++)
      build_fragments(sm.xf, MQ, r, r < M ? a.x + (size_t)r * K : nullptr, kb_base, nkb, threadIdx.x,
                      blockDim.x);
  } else {
    const NormArgs& n = a.norm;
    const bool writer = blockIdx.x == 0;
    for (int r0 = 0; r0 < rows_padded; r0 += norm_warps) {
      if (warp < norm_warps && r0 + warp < M) {
        const int r = r0 + warp;
        const int hrow = r * (int)n.row_of_token_stride + (int)n.row_of_token_offset;
        const uint32_t seq = (uint32_t)hrow / a.seq_tokens;
        const bool last_row = (uint32_t)hrow % a.seq_tokens == a.seq_tokens - 1;
        float* xout = writer && n.hidden_out ? n.hidden_out + (size_t)hrow * K : nullptr;
        float* yadd = writer && last_row && n.capture_added ? n.capture_added + seq * a.capture_stride : nullptr;
        float* xcap =
            writer && last_row && n.capture_residual ? n.capture_residual + seq * a.capture_stride : nullptr;
        norm_row_warp(n, hrow, sm.rowbuf + warp * K, xout, xcap, yadd, lane);
      }
      __syncthreads();
      for (int w = 0; w < norm_warps && r0 + w < rows_padded; w++) {
        const int r = r0 + w;
        build_fragments(sm.xf, MQ, r, r < M ? sm.rowbuf + w * K : nullptr, kb_base, nkb, threadIdx.x,
                        blockDim.x);
      }
      __syncthreads();
    }
    if (norm_warps == 0) {
      for (int r = 0; r < rows_padded; r++)
        build_fragments(sm.xf, MQ, r, nullptr, kb_base, nkb, threadIdx.x, blockDim.x);
    }
  }
  __syncthreads();

  float acc[MQ][2];
#pragma unroll
  for (int q = 0; q < MQ; q++) acc[q][0] = acc[q][1] = 0.f;
  if (live) rowgroup_dot<MQ>(codes, scales, bp0, bp1, sm.xf, kb_base, lane, acc);
  pdl_launch_dependents();

  // Reduce the K split inside the CTA: red[rgl][ks][row][token].
  if (rgl < RG) {
    const int g = lane >> 2, t = lane & 3;
    float* red = sm.red + (rgl * KS + ks) * 256;
#pragma unroll
    for (int q = 0; q < MQ; q++) {
      red[g * 16 + 4 * q + t] = acc[q][0];
      red[(g + 8) * 16 + 4 * q + t] = acc[q][1];
    }
  }
  __syncthreads();
  const int outs = (int)RG * 16 * rows_padded;
  if (C > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    float* dst = cluster.map_shared_rank(sm.cred, 0);
    for (int i = threadIdx.x; i < outs; i += blockDim.x) {
      const int rr = i / (16 * rows_padded), rest = i % (16 * rows_padded);
      const int row = rest / rows_padded, tok = rest % rows_padded;
      float v = 0.f;
      for (uint32_t k2 = 0; k2 < KS; k2++) v = add(v, sm.red[(rr * KS + k2) * 256 + row * 16 + tok]);
      dst[rank * outs + i] = v;
    }
    cluster.sync();
    if (rank != 0) return;
  }
  // Final values: vals[rr][row][tok] in red's first slots (re-used after a sync).
  auto final_value = [&](int rr, int row, int tok) -> float {
    float v = 0.f;
    if (C > 1) {
      const int i = (rr * 16 + row) * rows_padded + tok;
      for (uint32_t c2 = 0; c2 < C; c2++) v = add(v, sm.cred[c2 * outs + i]);
    } else {
      for (uint32_t k2 = 0; k2 < KS; k2++) v = add(v, sm.red[(rr * KS + k2) * 256 + row * 16 + tok]);
    }
    return v;
  };

  if (EPI == kEpilogueWrite || EPI == kEpilogueQkv) {
    for (int i = threadIdx.x; i < (int)RG * 16 * M; i += blockDim.x) {
      const int rr = i / (16 * M), rest = i % (16 * M), tok = rest / 16, row = rest % 16;
      const uint32_t rgi = rowset * RG + rr;
      if (rgi < mat.n / 16) a.out[(size_t)tok * a.out_stride + rgi * 16 + row] = final_value(rr, row, tok);
    }
  } else if (EPI == kEpilogueGated) {
    const uint32_t F = a.mat[0].n;
    for (int i = threadIdx.x; i < 16 * M; i += blockDim.x) {
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
    (void)F;
  } else if (EPI == kEpilogueHead) {
    if (threadIdx.x < kMaxTokens) s_best[threadIdx.x] = 0ull;
    __syncthreads();
    for (int i = threadIdx.x; i < (int)RG * 16 * M; i += blockDim.x) {
      const int tok = i / (RG * 16), rest = i % (RG * 16), rr = rest / 16, row = rest % 16;
      const uint32_t n = (rowset * RG + rr) * 16 + row;
      if (n < mat.n) {
        const float v = final_value(rr, row, tok);
        a.out[(size_t)tok * a.out_stride + n] = v;
        const unsigned long long key =
            ((unsigned long long)topk_key(__float_as_uint(v)) << 32) | (0xFFFFFFFFu - n);
        atomicMax(&s_best[tok], key);
      }
    }
    __syncthreads();
    if (threadIdx.x < M) atomicMax(a.head.argmax + threadIdx.x, s_best[threadIdx.x]);
  }

  if (EPI == kEpilogueQkv) {
    // The last CTA to finish runs QK-norm, RoPE and the KV append over every
    // row and head (rope_cache.wgsl:16-91).
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const uint32_t writers = gridDim.x / C;
      s_last = atomicAdd(a.counter, 1u) == writers - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const RopeArgs& r = a.rope;
    const int heads = (int)(r.heads + 2 * r.kv_heads);
    for (int item = warp; item < M * heads; item += nwarps) {
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

template <int MQ, int PRO, int EPI>
cudaError_t launch_one(const MatvecArgs& a, cudaStream_t stream, bool pdl) {
  const uint32_t NBP = a.mat[0].k / 64;
  const uint32_t C = a.cluster, RG = a.rg_per_cta, KS = a.k_split;
  const int threads = (int)(RG * KS * 32);
  const int norm_warps = PRO == kPrologueNorm ? (int)std::min<uint32_t>(RG * KS, a.m) : 0;
  const size_t nkb_max = 2 * ((NBP + C - 1) / C);
  size_t smem = nkb_max * 2 * MQ * 32 * sizeof(uint2) + (size_t)RG * KS * 256 * 4 +
                (size_t)norm_warps * a.norm.width * 4 + (C > 1 ? (size_t)C * RG * 16 * 4 * MQ * 4 : 0);
  uint32_t rowsets;
  if (EPI == kEpilogueGated) rowsets = a.mat[0].n / 16;
  else rowsets = (a.mat[0].n / 16 + RG - 1) / RG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rowsets * C);
  cfg.blockDim = dim3(threads);
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
