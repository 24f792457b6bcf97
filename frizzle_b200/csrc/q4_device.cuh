// Device helpers shared by the skinny Q4_0 products (q4_matvec.cu) and the
// persistent decode step (decode_step.cu): dequantisation into mma fragments,
// the f16 hi/lo split of X, QK-norm/RoPE for one head, the steering rewrite.
#pragma once

#include "q4_matvec.cuh"

namespace fz {
namespace q4dev {

FZ_DEV uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
FZ_DEV __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Four A registers (rows g, g+8 x the permuted columns) from one code word.
// A nibble n at bits 0-3 of a half: (n | 0x6400) is the half 1024 + n, less
// 1032 gives n - 8 exactly.  A nibble at bits 4-7: (16 n | 0x6400) is
// 1024 + 16 n, and 1/16 of it less 72 (one fused multiply-add) is n - 8,
// exactly; so one shift serves the word's upper two nibbles of each half.
FZ_DEV void dequant_word(uint32_t w, uint32_t a[4]) {
  const uint32_t kLow = 0x000F000Fu, kHigh = 0x00F000F0u, kMagic = 0x64006400u;
  const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6408u));       // 1032
  const __half2 sixteenth = __half2half2(__ushort_as_half((unsigned short)0x2C00u));  // 1/16
  const __half2 bias16 = __half2half2(__ushort_as_half((unsigned short)0xD480u));     // -72
  const uint32_t w8 = w >> 8;
  a[0] = h2_bits(__hsub2(bits_h2((w & kLow) | kMagic), bias));
  a[1] = h2_bits(__hsub2(bits_h2((w8 & kLow) | kMagic), bias));
  a[2] = h2_bits(__hfma2(bits_h2((w & kHigh) | kMagic), sixteenth, bias16));
  a[3] = h2_bits(__hfma2(bits_h2((w8 & kHigh) | kMagic), sixteenth, bias16));
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
// hi/lo f16 pair of an f32 value.
FZ_DEV void split_hi_lo(float v, __half& hi, __half& lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
}

// split_hi_lo of two values at once, as packed half2 words (a the low half):
// one paired conversion (cvt.rn.f16x2.f32) for the parts and one for the
// remainders, the same bits as two split_hi_lo calls.
FZ_DEV void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 back = __half22float2(h);
  const __half2 l = __floats2half2_rn(__fsub_rn(a, back.x), __fsub_rn(b, back.y));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
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
      split2(v01.x, v01.y, hi.x, lo.x);
      split2(v23.x, v23.y, hi.y, lo.y);
    }
    xf[xf_index(kb_rel, h, q, MQ, t, 2 * gp)] = hi;
    xf[xf_index(kb_rel, h, q, MQ, t, 2 * gp + 1)] = lo;
  }
}

// As build_fragments, for rows 0 .. 4 MQ - 1 of X at once (row r at src + r
// ld; rows from M on are zeros): each item's loads for every row are in
// flight together instead of one row's at a time.
template <int MQ>
FZ_DEV void build_fragments_rows(uint2* xf, int M, const float* src, int ld, int kb_base, int nkb, int first,
                                 int step) {
  for (int i = first; i < nkb * 8; i += step) {
    const int kb_rel = i >> 3, h = (i >> 2) & 1, t = i & 3;
    const int k0 = 32 * (kb_base + kb_rel) + 8 * h + 2 * t;
    float2 v01[4 * MQ], v23[4 * MQ];
#pragma unroll
    for (int r = 0; r < 4 * MQ; r++) {
      v01[r] = v23[r] = make_float2(0.f, 0.f);
      if (r < M) {
        v01[r] = *reinterpret_cast<const float2*>(src + (size_t)r * ld + k0);
        v23[r] = *reinterpret_cast<const float2*>(src + (size_t)r * ld + k0 + 16);
      }
    }
#pragma unroll
    for (int r = 0; r < 4 * MQ; r++) {
      __half h0, h1, h2, h3, l0, l1, l2, l3;
      split_hi_lo(v01[r].x, h0, l0);
      split_hi_lo(v01[r].y, h1, l1);
      split_hi_lo(v23[r].x, h2, l2);
      split_hi_lo(v23[r].y, h3, l3);
      xf[xf_index(kb_rel, h, r >> 2, MQ, t, 2 * (r & 3))] = pack4(h0, h1, h2, h3);
      xf[xf_index(kb_rel, h, r >> 2, MQ, t, 2 * (r & 3) + 1)] = pack4(l0, l1, l2, l3);
    }
  }
}

// 16 bytes global -> shared by cp.async (L2 only), waited for by stage_wait.
FZ_DEV void stage16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
FZ_DEV void stage_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// QK-norm and RoPE of one head held by a warp (rope.wgsl:40-138, d = 256:
// lane l holds elements 4l..4l+3 in a and 128+4l..128+4l+3 in b), given the
// lane's gains ga, gb and its four theta/2pi turns.
FZ_DEV void rope_apply(float4& a, float4& b, float4 ga, float4 gb, float4 turns, float eps, int d, uint32_t pos,
                       int lane) {
  float s = add(dot_self(a), dot_self(b));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float other = __shfl_down_sync(0xffffffffu, s, o);
    if (lane < o) s = add(s, other);
  }
  s = __shfl_sync(0xffffffffu, s, 0);
  // (s / d + eps with 1 / d exact for d = 256, then the hardware reciprocal
  // square root: within 2e-7 of the reference's inverseSqrt)
  const float rr = rsqrtf(__fmaf_rn(s, __frcp_rn((float)d), eps));
  a = make_float4(mul(mul(a.x, rr), ga.x), mul(mul(a.y, rr), ga.y), mul(mul(a.z, rr), ga.z), mul(mul(a.w, rr), ga.w));
  b = make_float4(mul(mul(b.x, rr), gb.x), mul(mul(b.y, rr), gb.y), mul(mul(b.z, rr), gb.z), mul(mul(b.w, rr), gb.w));
  // The angle is 2 pi times the turns' fraction (rope.wgsl:120-127 reduces the
  // same way); sincospi of twice the fraction has no large-argument path.
  const float tv[4] = {turns.x, turns.y, turns.z, turns.w};
  float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const float tt = mul((float)pos, tv[c]);
    float sn, cs;
    sincospif(mul(2.0f, sub(tt, rintf(tt))), &sn, &cs);
    const float x = av[c], y = bv[c];
    av[c] = sub(mul(x, cs), mul(y, sn));
    bv[c] = add(mul(x, sn), mul(y, cs));
  }
  a = make_float4(av[0], av[1], av[2], av[3]);
  b = make_float4(bv[0], bv[1], bv[2], bv[3]);
}

// The raw q, k or v of one (row, head), with QK-norm and RoPE applied to q
// and k (rope_cache.wgsl:16-91 reads the same columns).
FZ_DEV void rope_values(const RopeArgs& r, const float* raw, uint32_t raw_stride, int row, int head, uint32_t pos,
                       int lane, float4& a, float4& b) {
  const int d = (int)r.head_dim, H = (int)r.heads, KV = (int)r.kv_heads;
  const bool is_query = head < H, is_value = head >= H + KV;
  const int kvh = is_query ? 0 : (is_value ? head - H - KV : head - H);
  const int col = is_query ? head * d : (is_value ? H * d + KV * d + kvh * d : H * d + kvh * d);
  const float* src = raw + (size_t)row * raw_stride + col;
  a = __ldcg(reinterpret_cast<const float4*>(src) + lane);
  b = __ldcg(reinterpret_cast<const float4*>(src + d / 2) + lane);
  if (!is_value) {
    const float* gain = is_query ? r.q_gain : r.k_gain;
    rope_apply(a, b, reinterpret_cast<const float4*>(gain)[lane], reinterpret_cast<const float4*>(gain + d / 2)[lane],
               reinterpret_cast<const float4*>(r.turns)[lane], r.eps, d, pos, lane);
  }
}

// QK-norm, RoPE and the f16 KV append for one (row, head) by one warp, stored:
// the query to r.query_out (and its capture), keys and values to the cache.
FZ_DEV void rope_head_warp(const RopeArgs& r, const float* raw, uint32_t raw_stride, int row, int head,
                           uint32_t seq, uint32_t pos, float* capture_query, int lane) {
  const int d = (int)r.head_dim, H = (int)r.heads, KV = (int)r.kv_heads;
  const bool is_query = head < H, is_value = head >= H + KV;
  const int kvh = is_query ? 0 : (is_value ? head - H - KV : head - H);
  float4 a, b;
  rope_values(r, raw, raw_stride, row, head, pos, lane, a, b);
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
FZ_DEV unsigned long long head_key(float v, uint32_t n) {
  return ((unsigned long long)topk_key(__float_as_uint(v)) << 32) | (0xFFFFFFFFu - n);
}

}  // namespace q4dev
}  // namespace fz
