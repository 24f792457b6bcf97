// Attention for many query rows (prefill steps of more than 16 rows) on the
// fifth-generation tensor cores: softmax(q.k / 16) . v over keys j in
// [p - W + 1, p] (attention.wgsl:166-438 computes the same sums key by key;
// here it is the flash form, tile by tile).
//
// A CTA takes one sequence, one KV head and QT = 128 / G tokens of each of
// the G query heads that share it: 128 query rows, row r = head (r / QT),
// token (r % QT), one row a TMEM lane.  Keys go 64 at a time:
//   - warps 8 and 10 (one lane each) bring each tile's keys, and its values,
//     by TMA from the cache (4D tensor maps, 32-slot x 64-dimension boxes,
//     two a 64-dimension chunk, 128-byte swizzle) into two-stage key and
//     value rings, freed as each score product, or P V, completes; the value
//     ring first carries Q's f16 part on its way to tensor memory;
//   - warp 9 (one lane) issues tcgen05.mma: S = Q K^T (M = 128, N = 64) into
//     one of two TMEM score buffers, Q as f16 part (read from tensor memory)
//     and remainder (from shared memory), two MMAs a 16-dimension step, so
//     the products are exact and the sums f32; then O += P V (N = 256, V read
//     MN-major straight from the tile) into a TMEM accumulator, P as f16 part
//     and remainder;
//   - warps 0..7, two threads a row (warps w and w ^ 4 share TMEM lanes
//     32 (w % 4) ..; each takes half of a tile's keys and of O's columns),
//     read their 32 scores (tcgen05.ld), mask them (causal, window, rows
//     past the step), agree on the tile's max through shared memory, keep
//     the online softmax (max m, sum l), write P to shared memory and, when
//     a tile's max passes m by more than 8 (log2 units), rescale O in TMEM
//     (tcgen05.ld/st) first;
//     in between, the exponent base may lag the true max by up to 8, which
//     keeps P <= 256 and leaves the result the same softmax.
// A score MMA of N = 32 took ~49 cycles whether A came from shared or tensor
// memory, so the tiles are 64 keys: half the MMAs, barriers and waits a key.
// Every f16 part and remainder is made two values at a time (split2: one
// paired conversion each), since single conversions ran on the slow
// conversion pipe and bounded the query load, the softmax and the epilogue.
// At the end each row's O / l is written as f16 part and remainder (the
// output projection's operands) and, when asked for, as f32.
//
// Causal blocks are uneven: block i of a long prompt has i + 1 key tiles, so
// with one CTA a block the last block sets the launch's time.  When the
// launch's blocks fit one wave, each block gets a pair of CTAs, and a block
// of more than split_tiles tiles runs its two halves of keys on the two: each
// half writes its unnormalised O with its m and l, takes a ticket, and the
// second merges (O1 2^(m1-m) + O2 2^(m2-m)) / (l1 2^(m1-m) + l2 2^(m2-m)),
// m = max(m1, m2), and writes the block out; nothing waits on the other CTA.
//
// Every mbarrier wait is bounded; a wait that gives up records an error, the
// CTA waits (bounded) for the copies and products it issued, releases its
// tensor memory and returns.
#include <cuda.h>
#include <cuda_fp16.h>

#include "kernels.cuh"
#include "q4_device.cuh"

namespace fz {
namespace {

using namespace q4dev;

constexpr uint32_t kD = 256;              // head dimension
constexpr uint32_t kRows = 128;           // query rows a CTA (the MMA's M)
constexpr uint32_t kKT = 64;              // keys a tile
constexpr uint32_t kKStages = 2;          // key tiles in flight
constexpr uint32_t kVStages = 2;          // value tiles in flight
constexpr uint32_t kQChunk = kRows * 128;                 // 64 dimensions of 128 rows, f16: 16 KB
constexpr uint32_t kQBytes = 4 * kQChunk;                 // one of Q's two halves: 64 KB
constexpr uint32_t kCopyKeys = 32;                        // keys a tensor copy brings (the cache maps' box)
constexpr uint32_t kBox = kCopyKeys * 128;                // 32 keys x 64 dimensions f16: 4 KB
constexpr uint32_t kChunk = kKT * 128;                    // a tile's 64 dimensions: 8 KB (two copies)
constexpr uint32_t kHalf = 4 * kChunk;                    // a tile's keys (or values): 32 KB
constexpr uint32_t kPBytes = kRows * kKT * 2;             // P's part (or remainder): 16 KB
constexpr uint32_t kSmem = kQBytes + (kKStages + kVStages) * kHalf + 2 * kPBytes + 1024;   // 225 KB
static_assert(kVStages * kHalf >= kQBytes, "Q's f16 part passes through the value ring");
constexpr uint32_t kThreads = 352;
constexpr uint32_t kTmemCols = 512;       // O [0, 256), S buffers [256, 320) and [320, 384), Q's part [384, 512)
constexpr uint32_t kQhiCol = 384;         // Q's f16 part: row r on lane r, dimensions 2c, 2c + 1 in column c
constexpr uint32_t kSpin = 1u << 22;      // polls a wait takes before it gives up

FZ_DEV uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

FZ_DEV void mb_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
FZ_DEV void mb_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
FZ_DEV void mb_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
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

// The CTA's failure state: a flag in shared memory every wait checks.
struct Fail {
  volatile uint32_t* flag;
  uint32_t* error;
  FZ_DEV void raise(uint32_t code) const {
    *flag = 1u;
    if (error) atomicOr(error, code);
  }
};

// Waits for the phase of `parity` (bounded); false when it gave up or
// another thread of the CTA already did.
FZ_DEV bool mb_wait(uint64_t* b, uint32_t parity, const Fail& f, uint32_t code) {
  for (uint32_t i = 0; i < kSpin; i++) {
    if (mb_try(b, parity)) return true;
    if ((i & 255u) == 255u && *f.flag) return false;
  }
  f.raise(code);
  return false;
}

FZ_DEV void tma_box(void* dst, const void* map, uint64_t* bar, uint32_t x, uint32_t h, uint32_t slot, uint32_t seq) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(su32(dst)),
      "l"(map), "r"(x), "r"(h), "r"(slot), "r"(seq), "r"(su32(bar))
      : "memory");
}

// Shared-memory matrix descriptors (sm_100): start >> 4, leading and stride
// byte offsets >> 4, version 1, layout type (0: no swizzle, 2: 128-byte).
FZ_DEV uint64_t desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)layout << 61);
}
// kind::f16 with an f32 accumulator, M = 128: A K-major; B K-major or MN-major.
constexpr uint32_t idesc(uint32_t n, bool b_mn) {
  return (1u << 4) | ((b_mn ? 1u : 0u) << 16) | ((n >> 3) << 17) | ((kRows >> 4) << 24);
}

FZ_DEV void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t id, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(id), "r"(accumulate)
      : "memory");
}
// The same with A (M x 16, two f16 a 32-bit column, row m on lane m) read
// from tensor memory.
FZ_DEV void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t id, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(db), "r"(id), "r"(accumulate)
      : "memory");
}
FZ_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}
FZ_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FZ_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Named barriers of two softmax warps (64 threads); the _or form returns the
// OR of both sides' predicates to both.
FZ_DEV void pair_sync(uint32_t id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); }
FZ_DEV bool pair_sync_or(uint32_t id, bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred a, b;\n setp.ne.u32 a, %1, 0;\n bar.red.or.pred b, %2, 64, a;\n selp.u32 %0, 1, 0, b;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)p), "r"(id)
      : "memory");
  return r != 0;
}
FZ_DEV void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

FZ_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
FZ_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}



template <int G>
__global__ void __launch_bounds__(kThreads, 1) attention_tc_kernel(const AttentionArgs a) {
  constexpr uint32_t QT = kRows / G;   // tokens a CTA
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t k_full[kKStages], k_empty[kKStages], v_full[kVStages], v_empty[kVStages];
  __shared__ __align__(8) uint64_t s_full[2], s_empty[2];
  __shared__ __align__(8) uint64_t q_full, p_full, pv_done, drain;
  __shared__ uint32_t tmem_base;
  __shared__ uint32_t fail_word, ticket_word;
  __shared__ float xch[2 * kRows];   // a row's two softmax threads: [half][row]
  unsigned char* smem = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
  unsigned char* qlo = smem;
  unsigned char* kring = smem + kQBytes;
  unsigned char* vring = kring + kKStages * kHalf;
  unsigned char* qhi = vring;   // Q's f16 part on its way to tensor memory, before the first value tile
  unsigned char* phi = vring + kVStages * kHalf;
  unsigned char* plo = phi + kPBytes;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t T = a.seq_tokens;
  const uint32_t nblk = (T + QT - 1) / QT;
  const uint32_t parts = gridDim.x / nblk;   // 2 when the longest blocks' keys split in two
  // The latest tokens (the most keys) first; a block's two halves side by side.
  const uint32_t blk = nblk - 1 - blockIdx.x / parts, part = blockIdx.x % parts;
  const uint32_t kvh = blockIdx.y, seq = blockIdx.z, t0 = blk * QT;
  const Fail f{reinterpret_cast<volatile uint32_t*>(&fail_word), a.error};

  if (threadIdx.x == 0) {
    fail_word = 0u;
    for (uint32_t s = 0; s < kKStages; s++) {
      mb_init(&k_full[s], 1);
      mb_init(&k_empty[s], 1);
    }
    for (uint32_t s = 0; s < kVStages; s++) {
      mb_init(&v_full[s], 1);
      mb_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mb_init(&s_full[b], 1);
      mb_init(&s_empty[b], 256);
    }
    mb_init(&q_full, 256);
    mb_init(&p_full, 256);
    mb_init(&pv_done, 1);
    mb_init(&drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_wait();   // the queries and the caches' new rows come from the previous launches

  const uint32_t pos0 = (a.step ? a.step->position : a.position) + t0;
  const uint32_t ntok = min(QT, T - t0);
  const uint32_t p_last = pos0 + ntok - 1;
  const uint32_t k_lo = pos0 + 1 > a.window ? pos0 + 1 - a.window : 0u;   // the earliest key any row reads
  uint32_t kt0 = k_lo / kKT * kKT;
  uint32_t ntiles = (p_last - kt0) / kKT + 1;
  // A block of more than split_tiles tiles: this CTA takes one half of its
  // tiles (the second half holds every row's own key); otherwise the second
  // CTA of the pair has nothing to do.
  const bool split = parts == 2 && ntiles > a.split_tiles;
  if (split) {
    const uint32_t h = ntiles / 2;
    if (part == 0)
      ntiles = h;
    else {
      kt0 += h * kKT;
      ntiles -= h;
    }
  } else if (part == 1)
    ntiles = 0;
  const uint32_t sidx = (seq * gridDim.y + kvh) * nblk + blk;   // the block's split slot and counter

  if (ntiles == 0) {
    // (the empty second CTA of a block that did not split)
  } else if (warp < 8) {
    // ---- softmax: two threads a query row.  Warp w takes rows r = 32 (w %
    // 4) + lane (TMEM lanes r) and half h = w / 4 of each tile's 64 keys, of
    // O's 256 columns and of the query load; a row's two threads (warps w
    // and w ^ 4) meet once a tile in shared memory for the tile's max, and
    // at the end for l.
    const uint32_t half = warp >> 2, quarter = warp & 3;
    const uint32_t r = quarter * 32u + lane, hh = r / QT, t = r % QT;
    const bool live = t < ntok;
    const uint32_t head = kvh * G + hh, p = pos0 + t;
    const size_t row_base = (((size_t)seq * T + t0 + t) * a.heads + head) * kD;
    const uint32_t pair = 2u + quarter;   // the named barrier of warps w and w ^ 4
    const uint32_t lane_addr = tmem + ((quarter * 32u) << 16);
    {
      // The CTA's queries times scale x log2 e, as f16 part and remainder,
      // K-major 64-dimension chunks with 128-byte swizzle (16-byte unit u of
      // row r at unit u ^ (r % 8)).  The warp reads rows 32 (w % 4) + 16 h ..
      // + 15 a whole row at a time (lane l: dimensions 4 l .. 4 l + 3 and 128
      // + 4 l ..), all sixteen rows' loads in flight.
      const float sc = a.scale_log2e;
      const uint32_t r0 = quarter * 32u + half * 16u;
      float4 v[16][2];
#pragma unroll
      for (uint32_t k = 0; k < 16; k++) {
        const uint32_t rr = r0 + k, tt = rr % QT;
        v[k][0] = v[k][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tt < ntok) {
          const float4* q4 = reinterpret_cast<const float4*>(
              a.q + (((size_t)seq * T + t0 + tt) * a.heads + kvh * G + rr / QT) * kD);
          v[k][0] = __ldcg(q4 + lane);
          v[k][1] = __ldcg(q4 + 32 + lane);
        }
      }
#pragma unroll
      for (uint32_t k = 0; k < 16; k++) {
        const uint32_t rr = r0 + k;
#pragma unroll
        for (uint32_t hsel = 0; hsel < 2; hsel++) {
          const float4 w = v[k][hsel];
          uint32_t h0, h1, l0, l1;
          split2(mul(w.x, sc), mul(w.y, sc), h0, l0);
          split2(mul(w.z, sc), mul(w.w, sc), h1, l1);
          const uint32_t dim = 128u * hsel + 4u * lane;
          const uint32_t off = (dim >> 6) * kQChunk + rr * 128u + ((((dim & 63u) >> 3) ^ (rr & 7u)) << 4) +
                               (dim & 7u) * 2u;
          *reinterpret_cast<uint2*>(qhi + off) = make_uint2(h0, h1);
          *reinterpret_cast<uint2*>(qlo + off) = make_uint2(l0, l1);
        }
      }
      // The pair wrote the quarter's rows; each thread now moves its half of
      // its row's f16 part (dimensions 128 h .. + 127) into tensor memory (the
      // score MMAs read it from there, only the remainder from shared memory).
      pair_sync(pair);
#pragma unroll 1
      for (uint32_t c = 2 * half; c < 2 * half + 2; c++) {
        uint32_t qv[32];
#pragma unroll
        for (uint32_t u = 0; u < 8; u++) {
          const uint4 w = *reinterpret_cast<const uint4*>(qhi + c * kQChunk + r * 128u + ((u ^ (r & 7u)) << 4));
          qv[4 * u] = w.x;
          qv[4 * u + 1] = w.y;
          qv[4 * u + 2] = w.z;
          qv[4 * u + 3] = w.w;
        }
        tmem_st32(lane_addr + kQhiCol + 32u * c, qv);
      }
      proxy_fence();
      tc_fence_before();
      mb_arrive(&q_full);
    }
    const uint32_t ocol = 128u * half;   // this thread's columns of O
    float m = -INFINITY, l = 0.f;        // l: the sum over this thread's keys
    uint32_t pv_seen = 0;
    bool ok = true;
#pragma unroll 1
    for (uint32_t i = 0; i < ntiles; i++) {
      const uint32_t sb = i & 1u;
      // (the warp decides together: the tensor-memory loads below are warp-wide)
      bool go = __all_sync(0xffffffffu, mb_wait(&s_full[sb], (i >> 1) & 1u, f, 0x10000u));
      uint32_t sr[32];
      if (go) {
        tc_fence_after();
        tmem_ld32(lane_addr + 256u + kKT * sb + 32u * half, sr);
        tc_fence_before();
        mb_arrive(&s_empty[sb]);
      }
      const uint32_t j0 = kt0 + i * kKT + 32u * half;
      float sv[32];
      float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      // A half tile every lane of the warp keeps whole (the interior of the
      // window) needs no mask.
      const bool whole = live && j0 + 31u <= p && p - j0 < a.window;
      if (__all_sync(0xffffffffu, whole)) {
#pragma unroll
        for (uint32_t c = 0; c < 32; c++) {
          sv[c] = __uint_as_float(sr[c]);
          mq[c & 3] = fmaxf(mq[c & 3], sv[c]);
        }
      } else {
#pragma unroll
        for (uint32_t c = 0; c < 32; c++) {
          const uint32_t j = j0 + c;
          const bool valid = live && j <= p && p - j < a.window;
          sv[c] = valid ? __uint_as_float(sr[c]) : -INFINITY;
          mq[c & 3] = fmaxf(mq[c & 3], sv[c]);
        }
      }
      const float mine = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      // The previous tile's P V is done: P's buffer is free, O may be
      // rescaled, and the partner has read the last tile's exchange word.
      if (go && i > 0) {
        go = __all_sync(0xffffffffu, mb_wait(&pv_done, pv_seen & 1u, f, 0x20000u));
        pv_seen++;
        tc_fence_after();
      }
      xch[half * kRows + r] = mine;
      // Both threads of the row stop together (a wait that gave up, here or
      // anywhere in the CTA), so neither waits at a barrier the other left.
      if (pair_sync_or(pair, !go || *f.flag != 0u)) {
        ok = false;
        break;
      }
      const float mx = fmaxf(mine, xch[(half ^ 1u) * kRows + r]);
      // A new base when the tile's max passes it by more than 8; O is
      // rescaled by the warp together (lanes that keep their base scale by 1).
      const bool moved = mx > m + 8.f;
      const bool rescale = moved && m != -INFINITY;
      const float c = rescale ? exp2f(m - mx) : 1.f;
      if (rescale) l = mul(l, c);
      if (moved) m = mx;
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (uint32_t c0 = ocol; c0 < ocol + 128u; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(lane_addr + c0, o);
#pragma unroll
          for (int k = 0; k < 32; k++) o[k] = __float_as_uint(mul(__uint_as_float(o[k]), c));
          tmem_st32(lane_addr + c0, o);
        }
      }
      float sq[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t ph[16], pl[16];
#pragma unroll
      for (uint32_t c = 0; c < 32; c += 2) {
        const float e0 = sv[c] == -INFINITY ? 0.f : exp2f(sv[c] - m);
        const float e1 = sv[c + 1] == -INFINITY ? 0.f : exp2f(sv[c + 1] - m);
        sq[(c >> 1) & 3] = add(sq[(c >> 1) & 3], add(e0, e1));
        split2(e0, e1, ph[c / 2], pl[c / 2]);
      }
      l = add(l, add(add(sq[0], sq[1]), add(sq[2], sq[3])));
      // P row r, K-major without swizzle: core matrices of 8 rows x 8 keys
      // (128 bytes), 128 bytes apart along the keys, 1024 along the rows;
      // this thread's keys are core matrices 4 h .. 4 h + 3.
#pragma unroll
      for (uint32_t k = 0; k < 4; k++) {
        const uint32_t off = (r >> 3) * (kKT * 16u) + (4u * half + k) * 128u + (r & 7u) * 16u;
        *reinterpret_cast<uint4*>(phi + off) = make_uint4(ph[4 * k], ph[4 * k + 1], ph[4 * k + 2], ph[4 * k + 3]);
        *reinterpret_cast<uint4*>(plo + off) = make_uint4(pl[4 * k], pl[4 * k + 1], pl[4 * k + 2], pl[4 * k + 3]);
      }
      proxy_fence();
      tc_fence_before();
      mb_arrive(&p_full);
    }
    if (ok) {
      if (!__all_sync(0xffffffffu, mb_wait(&pv_done, pv_seen & 1u, f, 0x40000u))) ok = false;
      tc_fence_after();
    }
    // The row's l: both threads' sums, in one order (after the last P V, so
    // the partner has read every earlier exchange word).
    xch[half * kRows + r] = l;
    pair_sync(pair);
    l = add(xch[r], xch[kRows + r]);
    pdl_launch_dependents();
    // A split block: each half writes its O, m and l (row r at column-major
    // offsets, so a warp's stores are consecutive) and takes a ticket; the
    // second to take one merges the other's into its own and writes out.
    bool write = ok;
    const float* other = nullptr;
    float c_own = 1.f, c_oth = 0.f;
    if (split) {
      float* mine = a.split_part + ((size_t)sidx * 2 + part) * kAttnSplitFloats;
      if (ok) {
#pragma unroll 1
        for (uint32_t c0 = ocol; c0 < ocol + 128u; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(lane_addr + c0, o);
          if (!live) continue;   // (after the warp-wide load)
#pragma unroll
          for (int k = 0; k < 32; k++) __stcg(mine + (c0 + k) * kRows + r, __uint_as_float(o[k]));
        }
        if (half == 0) {
          __stcg(mine + kD * kRows + r, m);
          __stcg(mine + (kD + 1) * kRows + r, l);
        }
      }
      __threadfence();
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (threadIdx.x == 0) ticket_word = atomicAdd(a.counters + sidx, 1u);
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (ticket_word == 0u)
        write = false;   // the other half, still running, merges
      else {
        if (threadIdx.x == 0) a.counters[sidx] = 0u;   // zero again for the next launch
        __threadfence();
        other = a.split_part + ((size_t)sidx * 2 + (1u - part)) * kAttnSplitFloats;
        if (write && live) {
          const float m1 = __ldcg(other + kD * kRows + r), l1 = __ldcg(other + (kD + 1) * kRows + r);
          const float mm = fmaxf(m, m1);
          c_own = m == -INFINITY ? 0.f : exp2f(m - mm);
          c_oth = m1 == -INFINITY ? 0.f : exp2f(m1 - mm);
          l = __fmaf_rn(l1, c_oth, mul(l, c_own));
        }
      }
    }
    if (write) {
      // out = O / l (by one reciprocal), and its f16 part and remainder.
      const float inv = __frcp_rn(l);
#pragma unroll 1
      for (uint32_t c0 = ocol; c0 < ocol + 128u; c0 += 32) {
        uint32_t o[32];
        tmem_ld32(lane_addr + c0, o);
        if (!live) continue;   // (after the warp-wide load)
        float v[32];
        if (other) {
#pragma unroll
          for (int k = 0; k < 32; k++)
            v[k] = mul(__fmaf_rn(__ldcg(other + (c0 + k) * kRows + r), c_oth, mul(__uint_as_float(o[k]), c_own)), inv);
        } else {
#pragma unroll
          for (int k = 0; k < 32; k++) v[k] = mul(__uint_as_float(o[k]), inv);
        }
        if (a.out) {   // (the f32 form, when the caller wants it)
          float4* out4 = reinterpret_cast<float4*>(a.out + row_base + c0);
#pragma unroll
          for (int k = 0; k < 8; k++) out4[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        }
        if (a.out_hi) {
          uint32_t hw[16], lw[16];
#pragma unroll
          for (int k = 0; k < 16; k++) split2(v[2 * k], v[2 * k + 1], hw[k], lw[k]);
          uint4* oh = reinterpret_cast<uint4*>(a.out_hi + row_base + c0);
#pragma unroll
          for (int k = 0; k < 4; k++) oh[k] = make_uint4(hw[4 * k], hw[4 * k + 1], hw[4 * k + 2], hw[4 * k + 3]);
          if (a.out_lo) {
            uint4* ol = reinterpret_cast<uint4*>(a.out_lo + row_base + c0);
#pragma unroll
            for (int k = 0; k < 4; k++) ol[k] = make_uint4(lw[4 * k], lw[4 * k + 1], lw[4 * k + 2], lw[4 * k + 3]);
          }
        }
      }
    }
  } else if (warp == 8 || warp == 10) {
    // ---- the tiles' keys (warp 8) or values (warp 10) by TMA (lane 0): a
    // ring of kKStages key tiles, freed as each score product completes, and
    // one of kVStages value tiles, freed as each P V completes.
    if (lane == 0) {
      const bool keys = warp == 8;
      const unsigned char* map = static_cast<const unsigned char*>(a.kv_maps) + (keys ? 0 : 128);
      const uint32_t NS = keys ? kKStages : kVStages;
      uint64_t* full = keys ? k_full : v_full;
      uint64_t* empty = keys ? k_empty : v_empty;
      unsigned char* ring = keys ? kring : vring;
      uint32_t issued = 0;
      // (the value ring holds Q's f16 part until it is in tensor memory)
      const bool go = keys || mb_wait(&q_full, 0u, f, 0x400u);
#pragma unroll 1
      for (uint32_t i = 0; go && i < ntiles; i++) {
        const uint32_t s = i % NS;
        if (i >= NS && !mb_wait(&empty[s], ((i / NS) + 1u) & 1u, f, keys ? 0x1000u : 0x800u)) break;
        if (*f.flag) break;
        mb_expect_tx(&full[s], kHalf);
        unsigned char* dst = ring + s * kHalf;
        // Two 32-key copies a 64-dimension chunk, rows 0..31 then 32..63 of
        // the chunk (each wraps the ring on its own: slots hold whole copies).
#pragma unroll
        for (uint32_t h = 0; h < kKT / kCopyKeys; h++) {
          const uint32_t slot = (kt0 + i * kKT + h * kCopyKeys) % a.slots;
#pragma unroll
          for (uint32_t q = 0; q < 4; q++) tma_box(dst + q * kChunk + h * kBox, map, &full[s], 64u * q, kvh, slot, seq);
        }
        issued++;
      }
      // Every copy issued has landed before the CTA exits (bounded; the last
      // tile of each stage completes after the earlier ones).
      for (uint32_t s = 0; s < NS && s < issued; s++) {
        const uint32_t last = s + ((issued - 1 - s) / NS) * NS;
        for (uint32_t it = 0; it < kSpin && !mb_try(&full[s], (last / NS) & 1u); it++) {
        }
      }
    }
  } else {
    // ---- the MMA issuer (lane 0).
    if (lane == 0) {
      bool ok = mb_wait(&q_full, 0u, f, 0x2000u);
      tc_fence_after();
      constexpr uint32_t id_s = idesc(kKT, false), id_pv = idesc(kD, true);
      const uint32_t ql = su32(qlo), pa = su32(phi), pb = su32(plo);
#pragma unroll 1
      for (uint32_t i = 0; ok && i <= ntiles; i++) {
        if (i < ntiles) {
          const uint32_t s = i % kKStages, sb = i & 1u;
          if (!mb_wait(&k_full[s], (i / kKStages) & 1u, f, 0x4000u) ||
              (i >= 2 && !mb_wait(&s_empty[sb], ((i >> 1) + 1u) & 1u, f, 0x8000u)))
            break;
          tc_fence_after();
          const uint32_t kb = su32(kring + s * kHalf);
          const uint32_t d = tmem + 256u + kKT * sb;
#pragma unroll
          for (uint32_t c = 0; c < 4; c++)
#pragma unroll
            for (uint32_t kk = 0; kk < 4; kk++) {
              // 16 dimensions = 32 bytes along K within the 128-byte swizzled rows.
              const uint64_t db = desc(kb + c * kChunk + kk * 32u, 16u, 1024u, 2u);
              umma_ts(d, tmem + kQhiCol + 32u * c + 8u * kk, db, id_s, (c | kk) != 0u ? 1u : 0u);
              umma(d, desc(ql + c * kQChunk + kk * 32u, 16u, 1024u, 2u), db, id_s, 1u);
            }
          umma_commit(&s_full[sb]);
          umma_commit(&k_empty[s]);
        }
        if (i >= 1) {
          const uint32_t j = i - 1, s = j % kVStages;
          if (!mb_wait(&v_full[s], (j / kVStages) & 1u, f, 0x4000u) || !mb_wait(&p_full, j & 1u, f, 0x8000u)) break;
          tc_fence_after();
          const uint32_t vb = su32(vring + s * kHalf);
#pragma unroll
          for (uint32_t kk = 0; kk < kKT / 16; kk++) {
            // V MN-major: 64-dimension chunks kChunk apart, 8-key row groups 1024 bytes apart.
            const uint64_t dv = desc(vb + kk * 2048u, kChunk, 1024u, 2u);
            umma(tmem, desc(pa + kk * 256u, 128u, kKT * 16u, 0u), dv, id_pv, (j | kk) != 0u ? 1u : 0u);
            umma(tmem, desc(pb + kk * 256u, 128u, kKT * 16u, 0u), dv, id_pv, 1u);
          }
          umma_commit(&v_empty[s]);
          umma_commit(&pv_done);
        }
      }
      // Every product issued has completed before tensor memory is released.
      umma_commit(&drain);
      for (uint32_t it = 0; it < kSpin && !mb_try(&drain, 0u); it++) {
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

template <int G>
cudaError_t launch_g(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
  constexpr uint32_t QT = kRows / G;
  const uint32_t seqs = a.m / a.seq_tokens, nblk = (a.seq_tokens + QT - 1) / QT;
  // Pairs of CTAs a block when its keys may split: one wave of blocks at most
  // (more waves balance without it) and a window past split_tiles tiles.
  const bool pairs = a.split_part && a.counters && a.split_tiles &&
                     (uint64_t)nblk * a.kv_heads * seqs <= kAttnSplitBlocks && a.window > a.split_tiles * kKT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nblk * (pairs ? 2u : 1u), a.kv_heads, seqs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  (void)cudaGetLastError();
  return cudaLaunchKernelEx(&cfg, attention_tc_kernel<G>, a);
}

}  // namespace

bool attention_prefill_supported(uint32_t heads, uint32_t kv_heads, uint32_t head_dim) {
  if (head_dim != kD || kv_heads == 0 || heads % kv_heads) return false;
  const uint32_t g = heads / kv_heads;
  return g == 1 || g == 2 || g == 4 || g == 8;
}

cudaError_t configure_attention_tc() {
  cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attention_tc_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  return e;
}

cudaError_t launch_attention_tc(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
  if (a.head_dim != kD || a.kv_heads == 0 || a.heads % a.kv_heads || a.seq_tokens == 0 || a.m % a.seq_tokens ||
      !a.kv_maps || (reinterpret_cast<uintptr_t>(a.kv_maps) & 63u) || a.slots == 0)
    return cudaErrorInvalidValue;
  switch (a.heads / a.kv_heads) {
    case 1: return launch_g<1>(a, stream, pdl);
    case 2: return launch_g<2>(a, stream, pdl);
    case 4: return launch_g<4>(a, stream, pdl);
    case 8: return launch_g<8>(a, stream, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fz
