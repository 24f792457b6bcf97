// The persistent decode step (decode_step.cuh).
//
// Grid: one CTA per SM, launched cooperatively so every CTA is resident.
// Block: 8 consumer warps (the norm's 256 invocations, the products, the
// attention) and one producer warp whose lane 0 streams weight tiles.
//
// Every CTA walks the same sequence of phases:
//   for each layer: QKV (norm prologue) -> attention (QK-norm, RoPE, KV
//   append, split-K flash decode) -> O (2 K slices) -> gate/up (norm
//   prologue, GELU, steering) -> down (4 K slices);
//   then the final norm and the head (argmax for greedy selection).
// A phase's work is a list of tasks (one row group of 16 weight rows over one
// K slice); CTA c takes tasks c, c + P, ... of its slice.  A product's output
// is complete when every CTA that had tasks raised the phase's counter; the
// next phase's CTAs wait for that count (acquire) before reading it.  Partial
// sums over K slices meet in the consumer, in slice order, so results do not
// depend on timing.
//
// Weight tiles (a row group's block pairs, codes then scales) move from HBM to
// a ring of shared-memory slots by cp.async.bulk, completing on the slot's
// full mbarrier; the consumers release a slot on its empty mbarrier.  The
// producer walks the same phase sequence without waiting on counters, so it
// runs up to a ring ahead of the consumers, across phase and layer bounds.
//
// Every wait is bounded (2 s by the global timer, and an iteration cap); a
// wait that gives up records an error word for the host and the CTA abandons
// the step; other CTAs see the error word in their own waits.  Consumer
// barriers that follow a possible give-up are barrier reductions, so all
// consumer warps leave together.
#include <algorithm>
#include <mutex>

#include "decode_step.cuh"
#include "q4_device.cuh"

namespace fz {
namespace {

using namespace q4dev;

constexpr int kCW = 8;                  // consumer warps
constexpr int kCT = 32 * kCW;           // consumer threads
constexpr int kDT = kCT + 32;           // + the producer warp
constexpr uint32_t kSlotBp = 32;        // block pairs a ring slot holds
constexpr uint32_t kSlotCodes = kSlotBp * 512, kSlotScales = kSlotBp * 64;
constexpr uint32_t kHd = 256;           // head dimension
constexpr uint32_t kKeysPerSplit = 512;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr uint32_t kWaitIters = 1u << 30;

enum : uint32_t { kPhQkv = 0, kPhO = 1, kPhGate = 2, kPhDown = 3, kPhHead = 4 };
enum : uint32_t { kSyncQkv = 0, kSyncAttn = 1, kSyncO = 2, kSyncGate = 3, kSyncDown = 4 };
enum : uint32_t { kErrCounter = 0x100u, kErrFull = 0x200u, kErrEmpty = 0x400u, kErrDrain = 0x800u };

template <int MQ>
__host__ __device__ constexpr uint32_t ring_slots() {
  return MQ == 1 ? 8u : 6u;
}

__host__ __device__ inline uint32_t slice_kb(uint32_t k, uint32_t D) { return 2u * ((k / 64u + D - 1u) / D); }

__host__ __device__ inline uint32_t nkb_max(uint32_t hidden, uint32_t heads, uint32_t ffn) {
  uint32_t n = slice_kb(hidden, 1);
  n = n > slice_kb(heads * kHd, kDecodeOSlices) ? n : slice_kb(heads * kHd, kDecodeOSlices);
  n = n > slice_kb(ffn, kDecodeDownSlices) ? n : slice_kb(ffn, kDecodeDownSlices);
  return n;
}

// CTAs that hold tasks in a phase of nrg row groups over D slices.
__host__ __device__ inline uint32_t active_ctas(uint32_t nrg, uint32_t D, uint32_t G) {
  const uint32_t P = G / D;
  return D * (P < nrg ? P : nrg);
}

// Shared memory of one CTA (byte offsets).
struct DLayout {
  uint32_t codes, scales, full, empty, uni, xf, rowbuf, part, stat, red, best, flags, total;
};

__host__ __device__ inline DLayout layout_for(int MQ, uint32_t slots, uint32_t hidden, uint32_t group,
                                              uint32_t nkb) {
  DLayout L{};
  uint32_t o = 0;
  L.codes = o;
  o += slots * kSlotCodes;
  L.scales = o;
  o += slots * kSlotScales;
  L.full = o;
  o += slots * 8;
  L.empty = o;
  o += slots * 8;
  o = (o + 127u) & ~127u;
  L.uni = o;
  const uint32_t xf = nkb * 512u * (uint32_t)MQ;
  const uint32_t rows = 4u * (uint32_t)MQ * hidden * 4u;
  const uint32_t att = (group * kHd + 2u * kCW * group + kCW * group * kHd) * 4u + 2u * kHd * 2u;
  L.xf = o;
  L.rowbuf = o + xf;
  o += (xf + rows > att ? xf + rows : att);
  o = (o + 15u) & ~15u;
  L.part = o;
  o += 4u * MQ * kCT * 4u;
  L.stat = o;
  o += 2u * kDecodeMaxRows * 4u;
  L.red = o;
  o += kCW * 2u * 16u * 4u * MQ * 4u;
  L.best = o;
  o += kDecodeMaxRows * 8u;
  L.flags = o;
  o += 16u;
  L.total = o;
  return L;
}

// ------------------------------------------------------------ primitives

FZ_DEV uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

FZ_DEV void mb_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
FZ_DEV void mb_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
FZ_DEV void mb_arrive(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
FZ_DEV bool mb_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
FZ_DEV uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
FZ_DEV uint32_t error_word(const uint32_t* e) { return *reinterpret_cast<const volatile uint32_t*>(e); }

// Waits for the phase of parity `parity`; gives up after kWaitNs, or early
// once `abort` (shared) or the error word is set (either may be null).
FZ_DEV bool mb_wait(uint64_t* b, uint32_t parity, const uint32_t* err, const volatile uint32_t* abort) {
  if (mb_try(b, parity)) return true;
  const uint64_t t0 = now_ns();
  for (uint32_t i = 1; i < kWaitIters; i++) {
    if (mb_try(b, parity)) return true;
    if ((i & 63u) == 0) {
      if ((abort && *abort) || (err && error_word(err))) return false;
      if (now_ns() - t0 > kWaitNs) return false;
    }
  }
  return false;
}

// Bulk copy global -> this CTA's shared memory, completing on `bar`.
FZ_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   su32(dst)),
               "l"(src), "r"(bytes), "r"(su32(bar))
               : "memory");
}

// Consumer-warp barriers (named barrier 1; the producer warp never joins).
FZ_DEV void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
FZ_DEV bool cbar_or(bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred a, b;\n setp.ne.u32 a, %1, 0;\n bar.red.or.pred b, 1, 256, a;\n selp.u32 %0, 1, 0, b;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

// A phase counter: wait (thread 0) until it reaches `target`.
FZ_DEV bool wait_counter(const uint32_t* ctr, uint32_t target, uint32_t* err) {
  const uint64_t t0 = now_ns();
  for (uint32_t i = 0; i < kWaitIters; i++) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if ((i & 15u) == 15u) {
      if (error_word(err)) return false;
      if (now_ns() - t0 > kWaitNs) {
        atomicOr(err, kErrCounter);
        return false;
      }
    }
  }
  atomicOr(err, kErrCounter);
  return false;
}
FZ_DEV void raise_counter(uint32_t* ctr) {
  __threadfence();
  atomicAdd(ctr, 1u);
}

FZ_DEV float2 h2f2(uint32_t u) { return __half22float2(bits_h2(u)); }
FZ_DEV float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
FZ_DEV float4 add4(float4 a, float4 b) { return make_float4(add(a.x, b.x), add(a.y, b.y), add(a.z, b.z), add(a.w, b.w)); }
FZ_DEV float4 scale4(float4 v, float s, float4 g) {
  return make_float4(mul(mul(v.x, s), g.x), mul(mul(v.y, s), g.y), mul(mul(v.z, s), g.z), mul(mul(v.w, s), g.w));
}

// ------------------------------------------------------------ the walk

// Both roles walk this sequence; the producer issues each tile, the consumers
// wait for it, use it and release it.
template <class V>
FZ_DEV void matvec_phase(V& v, uint32_t kind, uint32_t l, const Q4Matrix& w, const Q4Matrix* w2, uint32_t D,
                         uint32_t c, uint32_t G) {
  const uint32_t P = G / D, d = c % D, i0 = c / D;
  const uint32_t nrg = w.n / 16, nbp = w.k / 64;
  const uint32_t bp0 = d * nbp / D, bp1 = (d + 1) * nbp / D;
  const bool has = i0 < P && i0 < nrg && bp0 < bp1;
  if (!v.phase_begin(kind, l, has, 2 * bp0, 2 * (bp1 - bp0))) return;
  if (has) {
    for (uint32_t rg = i0; rg < nrg; rg += P) {
      for (uint32_t b = bp0; b < bp1; b += kSlotBp) v.tile(w, rg, b, min(kSlotBp, bp1 - b), 0u);
      if (w2)
        for (uint32_t b = bp0; b < bp1; b += kSlotBp) v.tile(*w2, rg, b, min(kSlotBp, bp1 - b), 1u);
      v.task_end(kind, l, rg, d);
      if (v.aborted()) return;
    }
  }
  v.phase_end(kind, l, has);
}

template <class V>
FZ_DEV void walk(const DecodeArgs& a, V& v) {
  const uint32_t G = gridDim.x, c = blockIdx.x;
  for (uint32_t l = 0; l < a.n_layers; l++) {
    const DecodeLayer& L = a.layers[l];
    matvec_phase(v, kPhQkv, l, L.qkv, nullptr, 1, c, G);
    v.attention(l);
    matvec_phase(v, kPhO, l, L.o, nullptr, kDecodeOSlices, c, G);
    matvec_phase(v, kPhGate, l, L.gate, &L.up, 1, c, G);
    matvec_phase(v, kPhDown, l, L.down, nullptr, kDecodeDownSlices, c, G);
    if (v.aborted()) return;
  }
  if (!a.logits) return;
  // The head: a contiguous range of row groups a CTA, whole row groups a warp.
  const Q4Matrix& w = a.head;
  const uint32_t nrg = w.n / 16, nbp = w.k / 64;
  const uint32_t r0 = (uint32_t)((uint64_t)c * nrg / G), r1 = (uint32_t)((uint64_t)(c + 1) * nrg / G);
  if (!v.phase_begin(kPhHead, a.n_layers, r0 < r1, 0, 2 * nbp)) return;
  for (uint32_t rg = r0; rg < r1; rg++) {
    for (uint32_t b = 0; b < nbp; b += kSlotBp)
      v.head_tile(w, rg, b, min(kSlotBp, nbp - b), rg - r0, b == 0, b + kSlotBp >= nbp);
    if (v.aborted()) return;
  }
  v.phase_end(kPhHead, a.n_layers, r0 < r1);
}

// ------------------------------------------------------------ producer

template <int MQ>
struct Producer {
  static constexpr uint32_t S = ring_slots<MQ>();
  const DecodeArgs& a;
  unsigned char* codes;
  unsigned char* scales;
  uint64_t* full;
  uint64_t* empty;
  volatile uint32_t* flags;
  uint32_t idx;
  bool dead;

  FZ_DEV bool aborted() {
    if (!dead && flags[0]) dead = true;
    return dead;
  }
  FZ_DEV bool phase_begin(uint32_t, uint32_t, bool, uint32_t, uint32_t) { return !aborted(); }
  FZ_DEV void tile(const Q4Matrix& w, uint32_t rg, uint32_t b, uint32_t nb, uint32_t) {
    if (aborted()) return;
    const uint32_t slot = idx % S, use = idx / S;
    if (use > 0 && !mb_wait(empty + slot, (use - 1) & 1u, a.error, flags)) {
      if (!flags[0] && !error_word(a.error)) atomicOr(a.error, kErrEmpty);
      dead = true;
      return;
    }
    const size_t at = (size_t)rg * (w.k / 64) + b;
    mb_expect_tx(full + slot, nb * 576u);
    bulk_g2s(codes + (size_t)slot * kSlotCodes, reinterpret_cast<const unsigned char*>(w.codes) + at * 512, nb * 512u,
             full + slot);
    bulk_g2s(scales + (size_t)slot * kSlotScales, reinterpret_cast<const unsigned char*>(w.scales) + at * 64,
             nb * 64u, full + slot);
    idx++;
  }
  FZ_DEV void head_tile(const Q4Matrix& w, uint32_t rg, uint32_t b, uint32_t nb, uint32_t, bool, bool) {
    tile(w, rg, b, nb, 0);
  }
  FZ_DEV void task_end(uint32_t, uint32_t, uint32_t, uint32_t) {}
  FZ_DEV void phase_end(uint32_t, uint32_t, bool) {}
  FZ_DEV void attention(uint32_t) {}
  // Copies in flight must land before the CTA exits: every slot's last fill.
  FZ_DEV void drain() {
    const uint32_t n = idx < S ? idx : S;
    for (uint32_t k = idx - n; k < idx; k++)
      if (!mb_wait(full + k % S, (k / S) & 1u, nullptr, nullptr)) atomicOr(a.error, kErrDrain);
  }
};

// ------------------------------------------------------------ consumers

template <int MQ>
struct Consumer {
  static constexpr uint32_t S = ring_slots<MQ>();
  static constexpr int R = 4 * MQ;  // rows of X the fragments carry
  const DecodeArgs& a;
  unsigned char* sm;
  DLayout ly;
  const uint4* codes;
  const uint2* scales;
  uint64_t* full;
  uint64_t* empty;
  uint2* xf;
  float* rowbuf;
  float* part;
  float* stat;
  float* red;
  unsigned long long* best;
  volatile uint32_t* flags;
  uint32_t idx, kb_base, M, pos, W;
  int tid, warp, lane, g, t;
  bool fail, dead;
  float acc[2][MQ][2];
  unsigned long long hbest[MQ];

  FZ_DEV bool aborted() const { return dead; }
  // A barrier that also agrees on whether any consumer thread gave up.
  FZ_DEV bool sync_dead() {
    dead = cbar_or(fail);
    if (dead && tid == 0) flags[0] = 1u;
    return dead;
  }
  FZ_DEV uint32_t* sync_of(uint32_t l) { return a.sync + (size_t)l * W; }
  FZ_DEV void zero_acc() {
#pragma unroll
    for (int w = 0; w < 2; w++)
#pragma unroll
      for (int q = 0; q < MQ; q++) acc[w][q][0] = acc[w][q][1] = 0.f;
  }

  // The norm's fixed-order tree over the 256 invocations (norm.wgsl:75-85).
  FZ_DEV void tree(int rows, float* total) {
    cbar();
    for (int stride = 128; stride >= 32; stride >>= 1) {
      for (int i = tid; i < rows * stride; i += kCT) {
        const int r = i / stride, j = i % stride;
        part[r * kCT + j] = add(part[r * kCT + j], part[r * kCT + j + stride]);
      }
      cbar();
    }
    for (int r = warp; r < rows; r += kCW) {
      float s = part[r * kCT + lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float other = __shfl_down_sync(0xffffffffu, s, o);
        if (lane < o) s = add(s, other);
      }
      if (lane == 0) total[r] = s;
    }
    cbar();
  }

  // y of row r at vec4 v: the sum of its K-slice partials, in slice order.
  FZ_DEV float4 y_at(const float* y, uint32_t ny, int r, int v) {
    const int Wd = (int)a.hidden;
    float4 s = ldcg4(y + (size_t)r * Wd + 4 * v);
    for (uint32_t k = 1; k < ny; k++) s = add4(s, ldcg4(y + ((size_t)k * M + r) * Wd + 4 * v));
    return s;
  }

  // The norm launch (norm.wgsl:97-198) over the M rows into rowbuf: X plus
  // the post-normed block output, written back by CTA 0 with the captures;
  // then X's RMS norm times `gain`.
  FZ_DEV void norm(const float* xin, const float* y, uint32_t ny, const float* pg, const float* gain, float* xout,
                   uint64_t cap_x, uint64_t cap_y) {
    const int Wd = (int)a.hidden, V = Wd / 4;
    const float wf = (float)Wd;
    float* ry = stat;
    float* rx = stat + kDecodeMaxRows;
    const bool writer = blockIdx.x == 0;
    if (y) {
      for (int r = 0; r < (int)M; r++) {
        float p = 0.f;
        for (int v = tid; v < V; v += kCT) p = add(p, dot_self(y_at(y, ny, r, v)));
        part[r * kCT + tid] = p;
      }
      tree((int)M, ry);
      if (tid < (int)M) ry[tid] = inverse_sqrt(add(__fdiv_rn(ry[tid], wf), a.eps));
      cbar();
    }
    const float4* pg4 = reinterpret_cast<const float4*>(pg);
    for (int r = 0; r < (int)M; r++) {
      float* capbase = (writer && a.capture) ? a.capture + (size_t)r * a.capture_stride : nullptr;
      float4* xc = capbase && cap_x != ~0ull ? reinterpret_cast<float4*>(capbase + cap_x) : nullptr;
      float4* yc = capbase && cap_y != ~0ull ? reinterpret_cast<float4*>(capbase + cap_y) : nullptr;
      float4* out4 = writer && xout ? reinterpret_cast<float4*>(xout + (size_t)r * Wd) : nullptr;
      float4* buf = reinterpret_cast<float4*>(rowbuf + (size_t)r * Wd);
      float p = 0.f;
      for (int v = tid; v < V; v += kCT) {
        float4 x = ldcg4(xin + (size_t)r * Wd + 4 * v);
        if (y) {
          const float4 yy = scale4(y_at(y, ny, r, v), ry[r], pg4[v]);
          if (yc) yc[v] = yy;
          x = add4(x, yy);
        }
        if (out4) out4[v] = x;
        if (xc) xc[v] = x;
        buf[v] = x;
        p = add(p, dot_self(x));
      }
      part[r * kCT + tid] = p;
    }
    tree((int)M, rx);
    if (tid < (int)M) rx[tid] = inverse_sqrt(add(__fdiv_rn(rx[tid], wf), a.eps));
    cbar();
    const float4* g4 = reinterpret_cast<const float4*>(gain);
    for (int r = 0; r < (int)M; r++) {
      float4* buf = reinterpret_cast<float4*>(rowbuf + (size_t)r * Wd);
      for (int v = tid; v < V; v += kCT) buf[v] = scale4(buf[v], rx[r], g4[v]);
    }
    cbar();
  }

  // B fragments of the rows (src [M][K]) for blocks [kb0, kb0 + nkb); rows
  // past M are zero.  `global` rows were written by other CTAs this launch.
  template <bool kGlobal>
  FZ_DEV void fragments(const float* src, uint32_t K, uint32_t kb0, uint32_t nkb) {
    for (int r = 0; r < R; r++) {
      const int q = r >> 2, gp = r & 3;
      for (int i = tid; i < (int)nkb * 8; i += kCT) {
        const int kb_rel = i >> 3, h = (i >> 2) & 1, tq = i & 3;
        uint2 hi = make_uint2(0, 0), lo = make_uint2(0, 0);
        if (r < (int)M) {
          const float* row = src + (size_t)r * K + 32 * (kb0 + kb_rel) + 8 * h + 2 * tq;
          float2 v01, v23;
          if (kGlobal) {
            v01 = __ldcg(reinterpret_cast<const float2*>(row));
            v23 = __ldcg(reinterpret_cast<const float2*>(row + 16));
          } else {
            v01 = *reinterpret_cast<const float2*>(row);
            v23 = *reinterpret_cast<const float2*>(row + 16);
          }
          __half h0, h1, h2, h3, l0, l1, l2, l3;
          split_hi_lo(v01.x, h0, l0);
          split_hi_lo(v01.y, h1, l1);
          split_hi_lo(v23.x, h2, l2);
          split_hi_lo(v23.y, h3, l3);
          hi = pack4(h0, h1, h2, h3);
          lo = pack4(l0, l1, l2, l3);
        }
        xf[xf_index(kb_rel, h, q, MQ, tq, 2 * gp)] = hi;
        xf[xf_index(kb_rel, h, q, MQ, tq, 2 * gp + 1)] = lo;
      }
    }
  }

  FZ_DEV bool phase_begin(uint32_t kind, uint32_t l, bool has, uint32_t kb0, uint32_t nkb) {
    if (dead) return false;
    if (!has) return true;
    const uint32_t G = gridDim.x, Ln = a.n_layers;
    const uint32_t* ctr = nullptr;
    uint32_t target = 0;
    const DecodeLayer& L = a.layers[l < Ln ? l : Ln - 1];
    if (kind == kPhQkv && l > 0) {
      ctr = sync_of(l - 1) + kSyncDown;
      target = active_ctas(a.layers[l - 1].down.n / 16, kDecodeDownSlices, G);
    } else if (kind == kPhO) {
      ctr = sync_of(l) + kSyncAttn;
      target = M * a.kv_heads;
    } else if (kind == kPhGate) {
      ctr = sync_of(l) + kSyncO;
      target = active_ctas(L.o.n / 16, kDecodeOSlices, G);
    } else if (kind == kPhDown) {
      ctr = sync_of(l) + kSyncGate;
      target = active_ctas(L.gate.n / 16, 1, G);
    } else if (kind == kPhHead) {
      ctr = sync_of(Ln - 1) + kSyncDown;
      target = active_ctas(L.down.n / 16, kDecodeDownSlices, G);
    }
    if (tid == 0 && ctr && !wait_counter(ctr, target, a.error)) fail = true;
    if (sync_dead()) return false;
    kb_base = kb0;
    const uint64_t none = ~0ull, per = a.cap_per_layer;
    if (kind == kPhQkv) {
      norm(a.hidden_a, l > 0 ? a.y_mlp : nullptr, kDecodeDownSlices, l > 0 ? a.layers[l - 1].post_ffw_norm : nullptr,
           L.attn_norm, a.hidden_b, l * per + a.cap_residual, l > 0 ? (l - 1) * per + a.cap_mlp_added : none);
      fragments<false>(rowbuf, a.hidden, kb0, nkb);
    } else if (kind == kPhGate) {
      norm(a.hidden_b, a.y_attn, kDecodeOSlices, L.post_attn_norm, L.ffn_norm, a.hidden_a, none,
           l * per + a.cap_attn_added);
      fragments<false>(rowbuf, a.hidden, kb0, nkb);
    } else if (kind == kPhHead) {
      norm(a.hidden_a, a.y_mlp, kDecodeDownSlices, a.layers[Ln - 1].post_ffw_norm, a.output_norm, nullptr, none,
           (Ln - 1) * per + a.cap_mlp_added);
      fragments<false>(rowbuf, a.hidden, kb0, nkb);
#pragma unroll
      for (int q = 0; q < MQ; q++) hbest[q] = 0ull;
    } else if (kind == kPhO) {
      fragments<true>(a.attn, a.heads * kHd, kb0, nkb);
    } else {
      fragments<true>(a.act, a.ffn, kb0, nkb);
    }
    cbar();
    zero_acc();
    return true;
  }

  // One block pair's products into acc (rows g, g + 8 against X rows 4q + t).
  FZ_DEV void bp_dot(uint4 c, uint2 sc, int kb_rel0, float ac[MQ][2]) {
    const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kbi = 0; kbi < 2; kbi++) {
      uint32_t a0[4], a1[4];
      dequant_word(kbi ? c.z : c.x, a0);
      dequant_word(kbi ? c.w : c.y, a1);
      const uint32_t sw = kbi ? sc.y : sc.x;
      const float dg = __half2float(__ushort_as_half((unsigned short)(sw & 0xffffu)));
      const float dg8 = __half2float(__ushort_as_half((unsigned short)(sw >> 16)));
#pragma unroll
      for (int q = 0; q < MQ; q++) {
        const uint2 b0 = xf[xf_index(kb_rel0 + kbi, 0, q, MQ, t, g)];
        const uint2 b1 = xf[xf_index(kb_rel0 + kbi, 1, q, MQ, t, g)];
        float d[4];
        mma16816(d, a0, b0, zero);
        mma16816(d, a1, b1, d);
        ac[q][0] = __fmaf_rn(dg, d[0] + d[1], ac[q][0]);
        ac[q][1] = __fmaf_rn(dg8, d[2] + d[3], ac[q][1]);
      }
    }
  }

  // A tile shared by the 8 warps: warp w takes block pairs w, w + 8, ...
  FZ_DEV void tile(const Q4Matrix&, uint32_t, uint32_t b, uint32_t nb, uint32_t which) {
    if (dead) return;
    const uint32_t slot = idx % S, use = idx / S;
    idx++;
    if (!fail && !mb_wait(full + slot, use & 1u, a.error, flags)) fail = true;
    if (!fail) {
      const uint4* cs = codes + (size_t)slot * (kSlotCodes / 16);
      const uint2* ss = scales + (size_t)slot * (kSlotScales / 8);
      // (two calls, so that acc stays in registers)
      if (which)
        for (uint32_t j = warp; j < nb; j += kCW) bp_dot(cs[j * 32 + lane], ss[j * 8 + g], (int)(2 * (b + j) - kb_base), acc[1]);
      else
        for (uint32_t j = warp; j < nb; j += kCW) bp_dot(cs[j * 32 + lane], ss[j * 8 + g], (int)(2 * (b + j) - kb_base), acc[0]);
    }
    __syncwarp();
    if (lane == 0) mb_arrive(empty + slot, 1u);
  }

  // A head tile: the warp that owns the row group takes all of it.
  FZ_DEV void head_tile(const Q4Matrix& w, uint32_t rg, uint32_t b, uint32_t nb, uint32_t k, bool first, bool last) {
    if (dead) return;
    const uint32_t slot = idx % S, use = idx / S;
    idx++;
    if ((int)(k % kCW) != warp) return;
    if (first) {
#pragma unroll
      for (int q = 0; q < MQ; q++) acc[0][q][0] = acc[0][q][1] = 0.f;
    }
    if (!fail && !mb_wait(full + slot, use & 1u, a.error, flags)) fail = true;
    if (!fail) {
      const uint4* cs = codes + (size_t)slot * (kSlotCodes / 16);
      const uint2* ss = scales + (size_t)slot * (kSlotScales / 8);
      for (uint32_t j = 0; j < nb; j++) bp_dot(cs[j * 32 + lane], ss[j * 8 + g], (int)(2 * (b + j)), acc[0]);
    }
    __syncwarp();
    if (lane == 0) mb_arrive(empty + slot, (uint32_t)kCW);
    if (last && !fail) {
#pragma unroll
      for (int q = 0; q < MQ; q++) {
        const int tok = 4 * q + t;
        if (tok < (int)M) {
          const uint32_t n0 = rg * 16 + g, n8 = n0 + 8;
          a.logits[(size_t)tok * w.n + n0] = acc[0][q][0];
          a.logits[(size_t)tok * w.n + n8] = acc[0][q][1];
          const unsigned long long k0 = head_key(acc[0][q][0], n0), k8 = head_key(acc[0][q][1], n8);
          hbest[q] = max(hbest[q], max(k0, k8));
        }
      }
    }
  }

  FZ_DEV void task_end(uint32_t kind, uint32_t l, uint32_t rg, uint32_t d) {
    if (dead) return;
    constexpr int C = 4 * MQ;
    float* rw = red + warp * (2 * 16 * C);
#pragma unroll
    for (int q = 0; q < MQ; q++) {
      rw[g * C + 4 * q + t] = acc[0][q][0];
      rw[(g + 8) * C + 4 * q + t] = acc[0][q][1];
      if (kind == kPhGate) {
        rw[16 * C + g * C + 4 * q + t] = acc[1][q][0];
        rw[16 * C + (g + 8) * C + 4 * q + t] = acc[1][q][1];
      }
    }
    cbar();
    const uint32_t Hd = a.hidden;
    for (int i = tid; i < 16 * (int)M; i += kCT) {
      const int tok = i / 16, row = i % 16;
      const uint32_t n = rg * 16 + row;
      float v = 0.f;
      for (int w = 0; w < kCW; w++) v = add(v, red[w * (2 * 16 * C) + row * C + tok]);
      if (kind == kPhQkv) {
        a.qkv[(size_t)tok * ((a.heads + 2 * a.kv_heads) * kHd) + n] = v;
      } else if (kind == kPhO) {
        a.y_attn[((size_t)d * M + tok) * Hd + n] = v;
      } else if (kind == kPhDown) {
        a.y_mlp[((size_t)d * M + tok) * Hd + n] = v;
      } else {
        float up = 0.f;
        for (int w = 0; w < kCW; w++) up = add(up, red[w * (2 * 16 * C) + 16 * C + row * C + tok]);
        v = mul(gelu_tanh(v), up);
        if (a.edit_table) v = apply_edits(a.edit_table + (size_t)tok * a.table_stride, l, n, pos, v);
        a.act[(size_t)tok * a.ffn + n] = v;
        if (a.capture) a.capture[(size_t)tok * a.capture_stride + l * a.cap_per_layer + a.cap_neurons + n] = v;
      }
    }
    sync_dead();
    zero_acc();
  }

  FZ_DEV void phase_end(uint32_t kind, uint32_t l, bool has) {
    if (dead || !has) return;
    if (kind == kPhHead) {
#pragma unroll
      for (int q = 0; q < MQ; q++) {
        unsigned long long b = hbest[q];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
        const int tok = 4 * q + t;
        if (g == 0 && tok < (int)M && b) atomicMax(best + tok, b);
      }
      if (sync_dead()) return;
      if (tid < (int)M && best[tid]) atomicMax(a.argmax + tid, best[tid]);
      return;
    }
    // The last task's barrier has ordered every consumer's stores.
    const uint32_t which = kind == kPhQkv ? kSyncQkv : kind == kPhO ? kSyncO : kind == kPhGate ? kSyncGate : kSyncDown;
    if (tid == 0) raise_counter(sync_of(l) + which);
  }

  // ---------------------------------------------------------- attention

  FZ_DEV void attention(uint32_t l) {
    if (dead) return;
    const DecodeLayer& L = a.layers[l];
    const uint32_t G = gridDim.x;
    const uint32_t earliest = pos + 1 > L.window ? pos + 1 - L.window : 0;
    const uint32_t nkeys = pos + 1 - earliest, nsplit = (nkeys + kKeysPerSplit - 1) / kKeysPerSplit;
    const uint32_t KV = a.kv_heads, items = M * KV * nsplit;
    uint32_t item = G - 1 - blockIdx.x;
    if (item >= items) return;
    if (tid == 0 && !wait_counter(sync_of(l) + kSyncQkv, active_ctas(L.qkv.n / 16, 1, G), a.error)) fail = true;
    if (sync_dead()) return;
    const uint32_t group = a.heads / KV;
    for (; item < items; item += G) {
      const uint32_t row = item / (KV * nsplit), kvh = (item / nsplit) % KV, split = item % nsplit;
      if (group == 4) attend<4>(L, l, row, kvh, split, nsplit, earliest);
      else if (group == 2) attend<2>(L, l, row, kvh, split, nsplit, earliest);
      else attend<1>(L, l, row, kvh, split, nsplit, earliest);
      if (dead) return;
    }
  }

  // One (row, KV head, key split): QK-norm and RoPE of the group's queries
  // and of the new key (rope.wgsl:40-138), the KV append by the split that
  // holds the new position (rope_cache.wgsl:16-91), then flash decode over
  // the split's keys: warp w takes keys w, w + 8, ..., K and V loaded
  // together, an online softmax per warp, the warps folded in order; several
  // splits fold in split order in the last CTA (attention.wgsl:403-438).
  template <int GH>
  FZ_DEV void attend(const DecodeLayer& L, uint32_t l, uint32_t row, uint32_t kvh, uint32_t split, uint32_t nsplit,
                     uint32_t earliest) {
    float* qs = reinterpret_cast<float*>(sm + ly.uni);         // [GH][256], times scale * log2(e)
    uint16_t* kvs = reinterpret_cast<uint16_t*>(qs + GH * kHd);  // [2][256] the new key and value
    float* pm = reinterpret_cast<float*>(kvs + 2 * kHd);       // [8][GH]
    float* pl = pm + kCW * GH;                                 // [8][GH]
    float* po = pl + kCW * GH;                                 // [8][GH][256]
    const uint32_t H = a.heads, KV = a.kv_heads;
    const uint32_t j0 = earliest + split * kKeysPerSplit;
    const uint32_t j1 = min(j0 + kKeysPerSplit, pos + 1);
    const bool last = j1 == pos + 1;
    if (warp < GH + 2) {
      RopeArgs r{};
      r.q_gain = L.q_norm;
      r.k_gain = L.k_norm;
      r.turns = L.turns;
      r.eps = a.eps;
      r.heads = H;
      r.kv_heads = KV;
      r.head_dim = kHd;
      const int head = warp < GH ? (int)(kvh * GH) + warp : (warp == GH ? (int)(H + kvh) : (int)(H + KV + kvh));
      float4 va, vb;
      rope_values(r, a.qkv, (H + 2 * KV) * kHd, (int)row, head, pos, lane, va, vb);
      if (warp < GH) {
        if (last && a.capture) {
          float* cq = a.capture + (size_t)row * a.capture_stride + l * a.cap_per_layer + a.cap_query + head * kHd;
          reinterpret_cast<float4*>(cq)[lane] = va;
          reinterpret_cast<float4*>(cq + kHd / 2)[lane] = vb;
        }
        float* q = qs + warp * kHd;
        const float s = a.scale_log2e;
        reinterpret_cast<float4*>(q)[lane] = make_float4(mul(va.x, s), mul(va.y, s), mul(va.z, s), mul(va.w, s));
        reinterpret_cast<float4*>(q + kHd / 2)[lane] =
            make_float4(mul(vb.x, s), mul(vb.y, s), mul(vb.z, s), mul(vb.w, s));
      } else {
        const ushort4 pa = make_ushort4(f16_pack(va.x), f16_pack(va.y), f16_pack(va.z), f16_pack(va.w));
        const ushort4 pb = make_ushort4(f16_pack(vb.x), f16_pack(vb.y), f16_pack(vb.z), f16_pack(vb.w));
        uint16_t* kv = kvs + (warp - GH) * kHd;
        reinterpret_cast<ushort4*>(kv)[lane] = pa;
        reinterpret_cast<ushort4*>(kv + kHd / 2)[lane] = pb;
        if (last) {
          uint16_t* cache = (warp == GH ? L.key_cache : L.value_cache) + row * L.seq_stride +
                            ((size_t)(pos % L.slots) * KV + kvh) * kHd;
          reinterpret_cast<ushort4*>(cache)[lane] = pa;
          reinterpret_cast<ushort4*>(cache + kHd / 2)[lane] = pb;
        }
      }
    }
    cbar();
    // Keys: lane holds dimensions 8 lane .. 8 lane + 7.
    float q[GH][8];
#pragma unroll
    for (int h = 0; h < GH; h++) {
      const float4 x0 = reinterpret_cast<const float4*>(qs + h * kHd + 8 * lane)[0];
      const float4 x1 = reinterpret_cast<const float4*>(qs + h * kHd + 8 * lane)[1];
      q[h][0] = x0.x; q[h][1] = x0.y; q[h][2] = x0.z; q[h][3] = x0.w;
      q[h][4] = x1.x; q[h][5] = x1.y; q[h][6] = x1.z; q[h][7] = x1.w;
    }
    float m[GH], ls[GH], o[GH][8];
#pragma unroll
    for (int h = 0; h < GH; h++) {
      m[h] = -INFINITY;
      ls[h] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i++) o[h][i] = 0.f;
    }
    const uint16_t* kc = L.key_cache + row * L.seq_stride;
    const uint16_t* vc = L.value_cache + row * L.seq_stride;
    constexpr int KU = 4;
    for (uint32_t jb = j0 + warp; jb < j1; jb += kCW * KU) {
      uint4 kw[KU], vw[KU];
#pragma unroll
      for (int u = 0; u < KU; u++) {
        const uint32_t j = jb + kCW * u;
        kw[u] = vw[u] = make_uint4(0, 0, 0, 0);
        if (j < j1) {
          if (j == pos) {
            kw[u] = reinterpret_cast<const uint4*>(kvs)[lane];
            vw[u] = reinterpret_cast<const uint4*>(kvs + kHd)[lane];
          } else {
            const size_t at = ((size_t)(j % L.slots) * KV + kvh) * kHd;
            kw[u] = __ldcg(reinterpret_cast<const uint4*>(kc + at) + lane);
            vw[u] = __ldcg(reinterpret_cast<const uint4*>(vc + at) + lane);
          }
        }
      }
      float sc[KU][GH];
#pragma unroll
      for (int u = 0; u < KU; u++) {
        float k[8];
        {
          const float2 f0 = h2f2(kw[u].x), f1 = h2f2(kw[u].y), f2 = h2f2(kw[u].z), f3 = h2f2(kw[u].w);
          k[0] = f0.x; k[1] = f0.y; k[2] = f1.x; k[3] = f1.y;
          k[4] = f2.x; k[5] = f2.y; k[6] = f3.x; k[7] = f3.y;
        }
#pragma unroll
        for (int h = 0; h < GH; h++) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < 8; i++) s = __fmaf_rn(q[h][i], k[i], s);
          s = warp_sum(s);
          sc[u][h] = jb + kCW * u < j1 ? s : -INFINITY;
        }
      }
#pragma unroll
      for (int h = 0; h < GH; h++) {
        float mx = m[h];
#pragma unroll
        for (int u = 0; u < KU; u++) mx = fmaxf(mx, sc[u][h]);
        const float corr = exp2f(m[h] - mx);
        ls[h] = mul(ls[h], corr);
#pragma unroll
        for (int i = 0; i < 8; i++) o[h][i] = mul(o[h][i], corr);
#pragma unroll
        for (int u = 0; u < KU; u++) {
          if (jb + kCW * u < j1) {
            const float e = exp2f(sc[u][h] - mx);
            ls[h] = add(ls[h], e);
            const float2 f[4] = {h2f2(vw[u].x), h2f2(vw[u].y), h2f2(vw[u].z), h2f2(vw[u].w)};
#pragma unroll
            for (int i = 0; i < 4; i++) {
              o[h][2 * i] = __fmaf_rn(e, f[i].x, o[h][2 * i]);
              o[h][2 * i + 1] = __fmaf_rn(e, f[i].y, o[h][2 * i + 1]);
            }
          }
        }
        m[h] = mx;
      }
    }
#pragma unroll
    for (int h = 0; h < GH; h++) {
      if (lane == 0) {
        pm[warp * GH + h] = m[h];
        pl[warp * GH + h] = ls[h];
      }
      float4* dst = reinterpret_cast<float4*>(po + (warp * GH + h) * kHd + 8 * lane);
      dst[0] = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
      dst[1] = make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
    }
    cbar();
    // Fold the warps in order; thread tid is dimension tid.
    const uint32_t dim = (uint32_t)tid;
#pragma unroll
    for (int h = 0; h < GH; h++) {
      float mm = -INFINITY;
      for (int w = 0; w < kCW; w++) mm = fmaxf(mm, pm[w * GH + h]);
      float lsum = 0.f, acc_o = 0.f;
      for (int w = 0; w < kCW; w++) {
        const float mw = pm[w * GH + h];
        const float f = mw == mm ? 1.0f : exp2f(mw - mm);
        lsum = __fmaf_rn(pl[w * GH + h], f, lsum);
        acc_o = __fmaf_rn(po[(w * GH + h) * kHd + dim], f, acc_o);
      }
      const uint32_t head = kvh * GH + h;
      if (nsplit == 1) {
        a.attn[((size_t)row * H + head) * kHd + dim] = __fdiv_rn(acc_o, lsum);
      } else {
        const size_t at = ((size_t)row * H + head) * a.max_splits + split;
        a.partial_o[at * kHd + dim] = acc_o;
        if (dim == 0) {
          a.partial_ml[at * 2] = mm;
          a.partial_ml[at * 2 + 1] = lsum;
        }
      }
    }
    bool final_cta = nsplit == 1;
    if (!final_cta) {
      cbar();
      if (tid == 0) {
        __threadfence();
        flags[1] = atomicAdd(sync_of(l) + kDecodeSyncFixed + row * KV + kvh, 1u) == nsplit - 1 ? 1u : 0u;
      }
      cbar();
      final_cta = flags[1] != 0;
      if (final_cta) {
        __threadfence();
#pragma unroll
        for (int h = 0; h < GH; h++) {
          const uint32_t head = kvh * GH + h;
          const size_t base = ((size_t)row * H + head) * a.max_splits;
          float mm = -INFINITY;
          for (uint32_t s = 0; s < nsplit; s++) mm = fmaxf(mm, __ldcg(a.partial_ml + (base + s) * 2));
          float lsum = 0.f, acc_o = 0.f;
          for (uint32_t s = 0; s < nsplit; s++) {
            const float ms = __ldcg(a.partial_ml + (base + s) * 2);
            const float f = ms == mm ? 1.0f : exp2f(ms - mm);
            lsum = __fmaf_rn(__ldcg(a.partial_ml + (base + s) * 2 + 1), f, lsum);
            acc_o = __fmaf_rn(__ldcg(a.partial_o + (base + s) * kHd + dim), f, acc_o);
          }
          a.attn[((size_t)row * H + head) * kHd + dim] = __fdiv_rn(acc_o, lsum);
        }
      }
    }
    if (final_cta) {
      cbar();
      if (tid == 0) raise_counter(sync_of(l) + kSyncAttn);
    }
    sync_dead();
  }
};

// ------------------------------------------------------------ kernel

template <int MQ>
__global__ void __launch_bounds__(kDT, 1) decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(1024) unsigned char sm[];
  const uint32_t group = a.heads / a.kv_heads;
  const DLayout ly = layout_for(MQ, ring_slots<MQ>(), a.hidden, group, nkb_max(a.hidden, a.heads, a.ffn));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + ly.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(sm + ly.empty);
  volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(sm + ly.flags);
  unsigned long long* best = reinterpret_cast<unsigned long long*>(sm + ly.best);
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < ring_slots<MQ>(); s++) {
      mb_init(full + s, 1);
      mb_init(empty + s, kCW);
    }
    flags[0] = 0u;
    flags[1] = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < kDecodeMaxRows) best[threadIdx.x] = 0ull;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == kCW) {
    if (lane == 0) {
      Producer<MQ> p{a, sm + ly.codes, sm + ly.scales, full, empty, flags, 0u, false};
      walk(a, p);
      p.drain();
    }
  } else {
    Consumer<MQ> c{a, sm, ly};
    c.codes = reinterpret_cast<const uint4*>(sm + ly.codes);
    c.scales = reinterpret_cast<const uint2*>(sm + ly.scales);
    c.full = full;
    c.empty = empty;
    c.xf = reinterpret_cast<uint2*>(sm + ly.xf);
    c.rowbuf = reinterpret_cast<float*>(sm + ly.rowbuf);
    c.part = reinterpret_cast<float*>(sm + ly.part);
    c.stat = reinterpret_cast<float*>(sm + ly.stat);
    c.red = reinterpret_cast<float*>(sm + ly.red);
    c.best = best;
    c.flags = flags;
    c.idx = 0;
    c.kb_base = 0;
    c.M = a.m;
    c.pos = a.step->position;
    c.W = kDecodeSyncFixed + a.m * a.kv_heads;
    c.tid = threadIdx.x;
    c.warp = warp;
    c.lane = lane;
    c.g = lane >> 2;
    c.t = lane & 3;
    c.fail = false;
    c.dead = false;
    walk(a, c);
  }
  __syncthreads();
}

// Per device: the dynamic shared memory each instantiation was configured
// for, and the SM count (the grid).
std::mutex g_mu;
uint32_t g_configured[2][64] = {};
int g_sms[64] = {};

template <int MQ>
cudaError_t configure_mq(uint32_t hidden, uint32_t ffn, uint32_t heads, uint32_t kv_heads) {
  const DLayout ly = layout_for(MQ, ring_slots<MQ>(), hidden, heads / kv_heads, nkb_max(hidden, heads, ffn));
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_configured[MQ - 1][dev] >= ly.total) return cudaSuccess;
  e = cudaFuncSetAttribute(decode_kernel<MQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ly.total);
  if (e != cudaSuccess) return e;
  int per = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, decode_kernel<MQ>, kDT, ly.total);
  if (e != cudaSuccess) return e;
  if (per < 1) return cudaErrorInvalidConfiguration;
  e = cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  g_configured[MQ - 1][dev] = ly.total;
  return cudaSuccess;
}

template <int MQ>
cudaError_t launch_mq(const DecodeArgs& a, cudaStream_t stream) {
  const DLayout ly = layout_for(MQ, ring_slots<MQ>(), a.hidden, a.heads / a.kv_heads, nkb_max(a.hidden, a.heads, a.ffn));
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  int sms = 0;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_configured[MQ - 1][dev] < ly.total) return cudaErrorNotReady;  // prepare_decode first
    sms = g_sms[dev];
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sms);
  cfg.blockDim = dim3(kDT);
  cfg.dynamicSmemBytes = ly.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_kernel<MQ>, a);
}

}  // namespace

bool decode_supported(uint32_t rows, uint32_t hidden, uint32_t ffn, uint32_t heads, uint32_t kv_heads,
                      uint32_t head_dim) {
  if (rows == 0 || rows > kDecodeMaxRows || head_dim != kHd || kv_heads == 0 || heads % kv_heads) return false;
  const uint32_t group = heads / kv_heads;
  if (group != 1 && group != 2 && group != 4) return false;
  if (hidden % 64 || ffn % 64 || hidden > 8192) return false;
  const int MQ = rows <= 4 ? 1 : 2;
  const DLayout ly = layout_for(MQ, MQ == 1 ? ring_slots<1>() : ring_slots<2>(), hidden, group,
                                nkb_max(hidden, heads, ffn));
  return ly.total <= 227u * 1024u;
}

cudaError_t prepare_decode(uint32_t hidden, uint32_t ffn, uint32_t heads, uint32_t kv_heads) {
  if (!decode_supported(1, hidden, ffn, heads, kv_heads, kHd)) return cudaErrorInvalidValue;
  cudaError_t e = configure_mq<1>(hidden, ffn, heads, kv_heads);
  if (e != cudaSuccess || !decode_supported(kDecodeMaxRows, hidden, ffn, heads, kv_heads, kHd)) return e;
  return configure_mq<2>(hidden, ffn, heads, kv_heads);
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t stream) {
  if (!decode_supported(a.m, a.hidden, a.ffn, a.heads, a.kv_heads, kHd)) return cudaErrorInvalidValue;
  return a.m <= 4 ? launch_mq<1>(a, stream) : launch_mq<2>(a, stream);
}

}  // namespace fz
