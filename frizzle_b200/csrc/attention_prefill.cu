// Attention for many query rows (prefill steps of more than 16 rows), on the
// tensor cores (attention.wgsl:166-438 computes the same softmax(q.k / 16) . v
// over keys j in [p - W + 1, p]; here it is the flash form).
//
// A CTA takes 16 tokens of one sequence and one KV head; warp h takes query
// head h of the group (GH warps).  Keys go in 64-key tiles, double-buffered in
// shared memory by cp.async (16-byte pieces of each row XOR-swizzled by the
// row, so ldmatrix reads of eight rows hit all banks).  Scores S = Q K^T and
// the output O = P V run on mma.m16n8k16 (f16 in, f32 accumulate) with Q and
// P each split into an f16 part and its f16 remainder (two MMAs), so every
// product is exact and the sums are f32: the same bar as the f32 scalar form.
// Each lane keeps rows g and g + 8 of its warp's 16: an online softmax in
// registers (max and sum across the four lanes of a row by shuffles), the
// output's 256 columns in 128 accumulators.
#include <cuda_fp16.h>

#include "kernels.cuh"
#include "q4_device.cuh"

namespace fz {
namespace {

using namespace q4dev;

constexpr int kD = 256;       // head dimension
constexpr int kQT = 16;       // tokens a CTA
constexpr int kKT = 64;       // keys a tile

FZ_DEV uint32_t su32p(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

FZ_DEV void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32p(dst)), "l"(src) : "memory");
}

// Byte offset of (row, 16-byte piece) in a [rows][256] f16 tile with swizzled pieces.
FZ_DEV uint32_t spiece(uint32_t row, uint32_t piece) { return row * 512u + ((piece ^ (row & 7u)) << 4); }

FZ_DEV void ldsm_x4(uint32_t addr, uint32_t r[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
FZ_DEV void ldsm_x4_t(uint32_t addr, uint32_t r[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}


template <int GH>
__global__ void __launch_bounds__(32 * GH, 1) attention_prefill_kernel(const AttentionArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* qhi = smem;                                   // [GH][16][256] f16, swizzled
  unsigned char* qlo = qhi + GH * kQT * 512;
  unsigned char* kbuf = qlo + GH * kQT * 512;                  // [2][64][256] f16, swizzled
  unsigned char* vbuf = kbuf + 2 * kKT * 512;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nthreads = 32 * GH;
  const uint32_t kvh = blockIdx.y, seq = blockIdx.z;
  const uint32_t T = a.seq_tokens;
  const uint32_t t0 = blockIdx.x * kQT;
  pdl_wait();
  const uint32_t p0 = (a.step ? a.step->position : a.position) + t0;   // position of token t0
  const uint32_t ntok = min((uint32_t)kQT, T - t0);
  const uint32_t p_last = p0 + ntok - 1;
  const uint32_t k_lo = p0 + 1 > a.window ? p0 + 1 - a.window : 0;      // earliest key any row needs
  const uint32_t KV = a.kv_heads;
  const uint16_t* kc = a.key_cache + seq * a.seq_stride;
  const uint16_t* vc = a.value_cache + seq * a.seq_stride;

  // Copies keys [kb, kb + 64) into buffer `buf`; keys past p_last are zero rows.
  auto stage = [&](uint32_t kb, int buf) {
    unsigned char* kd = kbuf + buf * kKT * 512;
    unsigned char* vd = vbuf + buf * kKT * 512;
    for (int i = threadIdx.x; i < kKT * 32; i += nthreads) {
      const uint32_t r = (uint32_t)i >> 5, c = (uint32_t)i & 31u, j = kb + r;
      const uint32_t off = spiece(r, c);
      if (j <= p_last) {
        const size_t at = ((size_t)(j % a.slots) * KV + kvh) * kD + c * 8;
        cp16(kd + off, kc + at);
        cp16(vd + off, vc + at);
      } else {
        *reinterpret_cast<uint4*>(kd + off) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vd + off) = make_uint4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  stage(k_lo, 0);

  // This warp's queries (head kvh * GH + warp, tokens t0..t0+15) times scale * log2(e), split in f16.
  {
    const uint32_t head = kvh * GH + warp;
    for (int i = lane; i < kQT * 64; i += 32) {
      const uint32_t r = (uint32_t)i >> 6, c4 = (uint32_t)i & 63u;   // row, float4 column
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < ntok) {
        const size_t row = (size_t)seq * T + t0 + r;
        v = __ldcg(reinterpret_cast<const float4*>(a.q + (row * a.heads + head) * kD) + c4);
      }
      const float s = a.scale_log2e;
      const float x[4] = {__fmul_rn(v.x, s), __fmul_rn(v.y, s), __fmul_rn(v.z, s), __fmul_rn(v.w, s)};
      __half hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; e++) split_hi_lo(x[e], hi[e], lo[e]);
      // element 4 c4 .. 4 c4 + 3: piece c4 / 2, half (c4 & 1)
      const uint32_t off = (uint32_t)warp * kQT * 512 + spiece(r, c4 >> 1) + (c4 & 1u) * 8;
      *reinterpret_cast<uint2*>(qhi + off) = pack4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint2*>(qlo + off) = pack4(lo[0], lo[1], lo[2], lo[3]);
    }
  }

  // Rows g and g + 8 of the warp: tokens t0 + g, t0 + g + 8.
  const uint32_t pg = p0 + g, pg8 = p0 + g + 8;
  float m0 = -INFINITY, m8 = -INFINITY, l0 = 0.f, l8 = 0.f;
  float o[32][4];
#pragma unroll
  for (int i = 0; i < 32; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  const uint32_t qbase_hi = su32p(qhi) + (uint32_t)warp * kQT * 512;
  const uint32_t qbase_lo = su32p(qlo) + (uint32_t)warp * kQT * 512;
  int buf = 0;
#pragma unroll 1
  for (uint32_t kb = k_lo; kb <= p_last; kb += kKT, buf ^= 1) {
    if (kb + kKT <= p_last) {
      stage(kb + kKT, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint32_t kbase = su32p(kbuf + buf * kKT * 512), vbase = su32p(vbuf + buf * kKT * 512);
    // S = Q K^T for 64 keys: 8 n-tiles x 16 k-steps, Q's part and remainder.
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll 2
    for (int ks = 0; ks < 16; ks++) {
      uint32_t ah[4], al[4];
      {
        const uint32_t m = (uint32_t)lane >> 3, row = ((uint32_t)lane & 7u) + 8u * (m & 1u), piece = 2u * ks + (m >> 1);
        ldsm_x4(qbase_hi + spiece(row, piece), ah);
        ldsm_x4(qbase_lo + spiece(row, piece), al);
      }
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b[4];
        const uint32_t m = (uint32_t)lane >> 3, key = 8u * (nt + (m >> 1)) + ((uint32_t)lane & 7u);
        ldsm_x4(kbase + spiece(key, 2u * ks + (m & 1u)), b);
        const uint2 b0 = make_uint2(b[0], b[1]), b1 = make_uint2(b[2], b[3]);
        mma16816(s[nt], ah, b0, s[nt]);
        mma16816(s[nt], al, b0, s[nt]);
        mma16816(s[nt + 1], ah, b1, s[nt + 1]);
        mma16816(s[nt + 1], al, b1, s[nt + 1]);
      }
    }
    // Mask (causal, window, keys past the step) and the online softmax of rows g and g + 8.
    float mx0 = -INFINITY, mx8 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const uint32_t j = kb + 8u * nt + 2u * t + e;
        const bool ok0 = j <= pg && pg - j < a.window && g < (int)ntok;
        const bool ok8 = j <= pg8 && pg8 - j < a.window && g + 8 < (int)ntok;
        s[nt][e] = ok0 ? s[nt][e] : -INFINITY;
        s[nt][2 + e] = ok8 ? s[nt][2 + e] : -INFINITY;
        mx0 = fmaxf(mx0, s[nt][e]);
        mx8 = fmaxf(mx8, s[nt][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx8 = fmaxf(mx8, __shfl_xor_sync(0xffffffffu, mx8, 1));
    mx8 = fmaxf(mx8, __shfl_xor_sync(0xffffffffu, mx8, 2));
    const float n0 = fmaxf(m0, mx0), n8 = fmaxf(m8, mx8);
    // A row with nothing unmasked yet keeps max -inf: no rescale, weights 0.
    const float c0 = n0 == -INFINITY ? 1.f : exp2f(m0 - n0), c8 = n8 == -INFINITY ? 1.f : exp2f(m8 - n8);
    float sum0 = 0.f, sum8 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
#pragma unroll
      for (int e = 0; e < 2; e++) {
        s[nt][e] = n0 == -INFINITY ? 0.f : exp2f(s[nt][e] - n0);
        s[nt][2 + e] = n8 == -INFINITY ? 0.f : exp2f(s[nt][2 + e] - n8);
        sum0 += s[nt][e];
        sum8 += s[nt][2 + e];
      }
    }
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
    sum8 += __shfl_xor_sync(0xffffffffu, sum8, 1);
    sum8 += __shfl_xor_sync(0xffffffffu, sum8, 2);
    l0 = __fmaf_rn(l0, c0, sum0);
    l8 = __fmaf_rn(l8, c8, sum8);
    m0 = n0;
    m8 = n8;
#pragma unroll
    for (int i = 0; i < 32; i++) {
      o[i][0] *= c0;
      o[i][1] *= c0;
      o[i][2] *= c8;
      o[i][3] *= c8;
    }
    // O += P V: 4 k-steps of 16 keys x 32 n-tiles of 8 columns; P's part and remainder.
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      uint32_t ph[4], pl[4];
      {
        const float* p0v = s[2 * kk];
        const float* p1v = s[2 * kk + 1];
        const float w[8] = {p0v[0], p0v[1], p0v[2], p0v[3], p1v[0], p1v[1], p1v[2], p1v[3]};
        __half hh[8], ll[8];
#pragma unroll
        for (int e = 0; e < 8; e++) split_hi_lo(w[e], hh[e], ll[e]);
        ph[0] = h2_bits(__halves2half2(hh[0], hh[1]));
        ph[1] = h2_bits(__halves2half2(hh[2], hh[3]));
        ph[2] = h2_bits(__halves2half2(hh[4], hh[5]));
        ph[3] = h2_bits(__halves2half2(hh[6], hh[7]));
        pl[0] = h2_bits(__halves2half2(ll[0], ll[1]));
        pl[1] = h2_bits(__halves2half2(ll[2], ll[3]));
        pl[2] = h2_bits(__halves2half2(ll[4], ll[5]));
        pl[3] = h2_bits(__halves2half2(ll[6], ll[7]));
      }
#pragma unroll
      for (int dn = 0; dn < 32; dn += 2) {
        uint32_t b[4];
        const uint32_t m = (uint32_t)lane >> 3;
        const uint32_t key = 16u * kk + ((uint32_t)lane & 7u) + 8u * (m & 1u);
        ldsm_x4_t(vbase + spiece(key, (uint32_t)dn + (m >> 1)), b);
        const uint2 b0 = make_uint2(b[0], b[1]), b1 = make_uint2(b[2], b[3]);
        mma16816(o[dn], ph, b0, o[dn]);
        mma16816(o[dn], pl, b0, o[dn]);
        mma16816(o[dn + 1], ph, b1, o[dn + 1]);
        mma16816(o[dn + 1], pl, b1, o[dn + 1]);
      }
    }
    __syncthreads();
  }
  pdl_launch_dependents();
  // out = O / l; rows g and g + 8 (tokens t0 + g, t0 + g + 8), columns 8 dn + 2 t (+1).
  const uint32_t head = kvh * GH + warp;
#pragma unroll
  for (int half = 0; half < 2; half++) {
    const uint32_t r = (uint32_t)g + 8u * half;
    if (r >= ntok) continue;
    const float lsum = half ? l8 : l0;
    const size_t row = (size_t)seq * T + t0 + r;
    const size_t base = (row * a.heads + head) * kD;
#pragma unroll
    for (int dn = 0; dn < 32; dn++) {
      const uint32_t col = 8u * dn + 2u * t;
      const float v0 = __fdiv_rn(o[dn][2 * half], lsum), v1 = __fdiv_rn(o[dn][2 * half + 1], lsum);
      *reinterpret_cast<float2*>(a.out + base + col) = make_float2(v0, v1);
      if (a.out_hi) {
        __half h0, h1, e0, e1;
        split_hi_lo(v0, h0, e0);
        split_hi_lo(v1, h1, e1);
        *reinterpret_cast<__half2*>(a.out_hi + base + col) = __halves2half2(h0, h1);
        if (a.out_lo) *reinterpret_cast<__half2*>(a.out_lo + base + col) = __halves2half2(e0, e1);
      }
    }
  }
}

template <int GH>
cudaError_t launch_gh(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
  // (configure_attention_prefill raised the shared-memory limit on this device.)
  const size_t smem = (size_t)2 * GH * kQT * 512 + (size_t)4 * kKT * 512;
  const uint32_t seqs = a.m / a.seq_tokens;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.seq_tokens + kQT - 1) / kQT, a.kv_heads, seqs);
  cfg.blockDim = dim3(32 * GH);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  (void)cudaGetLastError();
  return cudaLaunchKernelEx(&cfg, attention_prefill_kernel<GH>, a);
}

}  // namespace

cudaError_t configure_attention_prefill() {
  size_t smem4 = (size_t)2 * 4 * kQT * 512 + (size_t)4 * kKT * 512;
  size_t smem2 = (size_t)2 * 2 * kQT * 512 + (size_t)4 * kKT * 512;
  size_t smem1 = (size_t)2 * 1 * kQT * 512 + (size_t)4 * kKT * 512;
  cudaError_t e = cudaFuncSetAttribute(attention_prefill_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem4);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_prefill_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_prefill_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
  return e;
}

bool attention_prefill_supported(uint32_t heads, uint32_t kv_heads, uint32_t head_dim) {
  if (head_dim != kD || kv_heads == 0 || heads % kv_heads) return false;
  const uint32_t gh = heads / kv_heads;
  return gh == 1 || gh == 2 || gh == 4;
}

cudaError_t launch_attention_prefill(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
  if (!attention_prefill_supported(a.heads, a.kv_heads, a.head_dim) || a.seq_tokens == 0 || a.m % a.seq_tokens)
    return cudaErrorInvalidValue;
  switch (a.heads / a.kv_heads) {
    case 4: return launch_gh<4>(a, stream, pdl);
    case 2: return launch_gh<2>(a, stream, pdl);
    case 1: return launch_gh<1>(a, stream, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fz
