// Shared device helpers for the frizzle_b200 kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define FZ_DEV __device__ __forceinline__

namespace fz {

// The step's parameters as the device reads them: kernels::Step's head
// (kernels/interface.h:163-185) with a capture switch in its padding.
// Kernels read the position and the sampling settings from here, so one CUDA
// graph serves every position.
struct DeviceStep {
  uint32_t position, tokens, logits, fed;
  uint32_t seed[2];
  uint32_t top_k;
  float temperature, top_p, min_p, log_min_p;
  uint32_t capture;
  uint32_t padding[4];   // [0]: the engine's step serial on the device copy (flag-in-data epochs)
};
static_assert(sizeof(DeviceStep) == 64, "the step head is 64 bytes");

FZ_DEV uint32_t f32_bits(float f) { return __float_as_uint(f); }
FZ_DEV float bits_f32(uint32_t u) { return __uint_as_float(u); }

// f32 sums and products kept as separate roundings where the restated shader
// does not fuse them (nvcc would otherwise contract a*b+c into an fma).
FZ_DEV float mul(float a, float b) { return __fmul_rn(a, b); }
FZ_DEV float add(float a, float b) { return __fadd_rn(a, b); }
FZ_DEV float sub(float a, float b) { return __fsub_rn(a, b); }

// x*x + y*y + z*z + w*w, left to right, no fusion: a vec4's dot with itself
// as the norm and QK-norm shaders form it (norm.wgsl:180-186).
FZ_DEV float dot_self(float4 v) {
  return add(add(add(mul(v.x, v.x), mul(v.y, v.y)), mul(v.z, v.z)), mul(v.w, v.w));
}

FZ_DEV float inverse_sqrt(float v) { return __fdiv_rn(1.0f, __fsqrt_rn(v)); }

// The KV cache's pack: saturate to +-65,504, round to nearest even
// (formats/f16/f16_pack.wgsl:16-19).
FZ_DEV uint16_t f16_pack(float v) {
  v = fminf(fmaxf(v, -65504.0f), 65504.0f);
  return __half_as_ushort(__float2half_rn(v));
}
FZ_DEV float f16_unpack(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous one's results before reading them.
FZ_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
FZ_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

FZ_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
FZ_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The reference norm's fixed-order sum of squares over a row of `vec4s`
// vec4s, evaluated by one warp: lane l stands in for the 256 invocations
// l, l + 32, ..., l + 224 of norm.wgsl; invocation i sums the squares of its
// vec4s i, i + 256, ... in order; the 256 partials are halved level by level
// (norm.wgsl:75-85), the first three levels inside each lane, the last five
// across lanes.  Every lane returns the total.
FZ_DEV float norm_sum_squares_warp(const float4* row, int vec4s, int lane) {
  float part[8];
#pragma unroll
  for (int a = 0; a < 8; a++) {
    float s = 0.0f;
    for (int v = lane + 32 * a; v < vec4s; v += 256) s = add(s, dot_self(row[v]));
    part[a] = s;
  }
#pragma unroll
  for (int a = 0; a < 4; a++) part[a] = add(part[a], part[a + 4]);  // stride 128
#pragma unroll
  for (int a = 0; a < 2; a++) part[a] = add(part[a], part[a + 2]);  // stride 64
  float s = add(part[0], part[1]);                                    // stride 32
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float other = __shfl_down_sync(0xffffffffu, s, o);
    if (lane < o) s = add(s, other);
  }
  return __shfl_sync(0xffffffffu, s, 0);
}

// Order-preserving key of a logit's bits: -0 as +0, every NaN above +inf
// (topk.wgsl:32-44).
FZ_DEV uint32_t topk_key(uint32_t b) {
  if (b == 0x80000000u) b = 0;
  if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x007FFFFFu) != 0) return 0xFFFFFFFFu;
  if (b & 0x80000000u) return ~b;
  return b | 0x80000000u;
}
FZ_DEV uint32_t topk_bits(uint32_t key) {
  if (key == 0xFFFFFFFFu) return 0x7FC00000u;
  if (key & 0x80000000u) return key & 0x7FFFFFFFu;
  return ~key;
}

// p * 2^k for k in [-149, 0], rounded once, as ldexp: a normal result is an
// exact product with 2^k; below 2^-126 the product with 2^(k + 64) is exact and
// the one with 2^-64 rounds once.
FZ_DEV float scale_pow2(float p, int k) {
  if (k >= -126) return __fmul_rn(p, __int_as_float((127 + k) << 23));
  return __fmul_rn(__fmul_rn(p, __int_as_float((127 + k + 64) << 23)), 5.421010862427522e-20f);
}

// e^x for x <= 0 (matmul.wgsl:122-138) and GELU's tanh form from it
// (matmul.wgsl:140-152): the same fma chain, so the same bits as the shader
// on an IEEE target.
FZ_DEV float exp_nonpositive(float x) {
  float xc = fmaxf(x, -100.0f);
  float k = floorf(__fmaf_rn(xc, 1.4426950408889634f, 0.5f));
  float r = __fmaf_rn(k, -0.693145751953125f, xc);
  r = __fmaf_rn(k, -1.4286068203094172e-06f, r);
  float p = (float)(1.0 / 720.0);
  p = __fmaf_rn(p, r, (float)(1.0 / 120.0));
  p = __fmaf_rn(p, r, (float)(1.0 / 24.0));
  p = __fmaf_rn(p, r, (float)(1.0 / 6.0));
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  return scale_pow2(p, (int)k);
}
FZ_DEV float gelu_tanh(float g) {
  float z = mul(0.7978845608028654f, __fmaf_rn(mul(mul(0.044715f, g), g), g, g));
  float e = exp_nonpositive(mul(-2.0f, fabsf(z)));
  float s = z > 0.0f ? 1.0f : (z < 0.0f ? -1.0f : 0.0f);
  float t = mul(s, mul(sub(1.0f, e), __frcp_rn(add(1.0f, e))));  // 1 / (1 + e), rounded once
  float half_g = mul(0.5f, g);
  return __fmaf_rn(half_g, t, half_g);
}

// Philox4x32-10 (draw.wgsl:48-60).
FZ_DEV uint4 philox(uint4 c, uint2 key) {
#pragma unroll
  for (int r = 0; r < 10; r++) {
    uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = make_uint4(hi1 ^ c.y ^ key.x, lo1, hi0 ^ c.w ^ key.y, lo0);
    key.x += 0x9E3779B9u;
    key.y += 0xBB67AE85u;
  }
  return c;
}

}  // namespace fz
