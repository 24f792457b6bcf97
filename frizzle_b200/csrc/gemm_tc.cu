// tcgen05/TMEM product over Q4_0 weights (gemm_tc.cuh).
//
// A CTA computes a 128-row x BN-column tile of Y (128 rows of X: tokens; BN
// weight rows).  K is walked 64 columns (one Q4_0 block pair) a stage through
// a ring of shared-memory stages:
//   - warp 0 (one lane) loads the 128 x 64 f16 tile of X with TMA
//     (SWIZZLE_128B, K-major), and of X's remainder for two passes;
//   - warps 2..9 dequantize the BN x 64 weight tile from the fragment-native
//     Q4_0 layout, (code - 8) x d rounded once to f16, into the same
//     swizzled K-major layout;
//   - warp 1 (one lane) issues tcgen05.mma kind::f16 (M = 128, N = BN,
//     K = 16) into an f32 accumulator in tensor memory and commits each stage
//     back to its producers;
//   - warps 10..17 read the accumulator (tcgen05.ld 32x32b) and write Y, or,
//     for a gated product, gelu(gate) * up with the steering edits.
// CTAs are persistent (one per SM) and walk tiles t = blockIdx.x, + gridDim.x,
// ...; the accumulator is double-buffered in TMEM (2 x BN columns), so the
// epilogue of one tile runs while the next tile's MMAs fill the other buffer,
// and the stage ring runs on across tile bounds.
// Every mbarrier wait is bounded: on timeout the kernel records an error,
// stops waiting, and still releases its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gemm_tc.cuh"

namespace fz {
namespace {

constexpr int kBM = 128;              // rows of X a tile (the MMA's M)
constexpr int kBK = 64;               // columns a stage: 128 B of f16 a row
constexpr int kProducers = 8;         // weight-dequant warps (warps 2..9)
constexpr int kEpilogue = 8;          // epilogue warps (warps 10..17)
constexpr int kThreadsG = 32 * (2 + kProducers + kEpilogue);
constexpr int kStageCols = 16;        // accumulator columns an epilogue warp turns around at once
constexpr uint32_t kSpinLimit = 1u << 20;

FZ_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

FZ_DEV void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(n) : "memory");
}
FZ_DEV void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
FZ_DEV void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
FZ_DEV bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase of parity `parity` to complete, at most kSpinLimit
// polls; gives up early once another warp has recorded an error.
FZ_DEV bool mbar_wait(uint64_t* b, uint32_t parity, uint32_t* err, uint32_t code) {
  for (uint32_t i = 0; i < kSpinLimit; i++) {
    if (mbar_try(b, parity)) return true;
    if ((i & 1023u) == 1023u && *reinterpret_cast<volatile uint32_t*>(err)) return false;
  }
  atomicExch(err, code);
  return false;
}

FZ_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes stacked along M/N (stride byte offset 1024), tile base 1024-aligned.
FZ_DEV uint64_t smem_desc(const void* p) {
  const uint32_t a = smem_u32(p);
  uint64_t d = (uint64_t)((a & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;              // leading byte offset (unused by swizzled K-major): 16 B
  d |= (uint64_t)(1024 >> 4) << 32;    // stride byte offset
  d |= (uint64_t)1 << 46;              // descriptor version for sm_100
  d |= (uint64_t)2 << 61;              // SWIZZLE_128B
  return d;
}

template <int BN>
__host__ __device__ constexpr uint32_t instr_desc() {
  // kind::f16: D f32, A and B f16, both K-major, M = 128, N = BN.
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

FZ_DEV void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}
FZ_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
FZ_DEV void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FZ_DEV void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
FZ_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

FZ_DEV void tmem_ld32(uint32_t taddr, uint32_t r[32]) {
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

FZ_DEV uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
FZ_DEV __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Byte offset of element (n, k) in a K-major 128B-swizzled tile of 64 f16 columns.
FZ_DEV uint32_t swz(uint32_t n, uint32_t k) { return n * 128u + ((((k >> 3) ^ (n & 7u)) & 7u) << 4) + (k & 7u) * 2u; }

// A row group's codes and scales for one block pair, in registers.
struct Codes {
  uint4 c;
  uint2 s;
};

FZ_DEV Codes load_codes(const Q4Matrix& w, uint32_t rg, uint32_t bp, bool live, int lane) {
  Codes x;
  x.c = make_uint4(0, 0, 0, 0);
  x.s = make_uint2(0, 0);
  if (live) {
    const uint32_t nbp = w.k / 64;
    x.c = w.codes[((size_t)rg * nbp + bp) * 32 + lane];
    x.s = w.scales[((size_t)rg * nbp + bp) * 8 + (lane >> 2)];
  }
  return x;
}

// One row group's 16 x 64 weights (one block pair) into the stage's B tile at
// rows [row0, row0 + 16).  Lane (g, t) holds rows g and g + 8 of both blocks;
// each of its four code words gives, per row, the f16 pairs at columns
// (2t, 2t+1) and (16 + 2t, 17 + 2t) of half h of block kb.  A row group past
// the matrix is written as zeros (its codes were never loaded).
FZ_DEV void dequant_tile(unsigned char* tile, unsigned char* tile_lo, uint32_t row0, const Codes& x, bool live,
                         int lane) {
  const uint32_t g = lane >> 2, t = lane & 3;
  const uint32_t kLow = 0x000F000Fu, kHigh = 0x00F000F0u, kMagic = 0x64006400u;
  const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6408u));       // 1032
  const __half2 sixteenth = __half2half2(__ushort_as_half((unsigned short)0x2C00u));  // 1/16
  const __half2 bias16 = __half2half2(__ushort_as_half((unsigned short)0xD480u));     // -72
  const uint32_t words[4] = {x.c.x, x.c.y, x.c.z, x.c.w};
#pragma unroll
  for (int wi = 0; wi < 4; wi++) {
    const uint32_t kb = wi >> 1, h = wi & 1;
    const uint32_t wd = words[wi], w8 = wd >> 8;
    const uint32_t sw = kb ? x.s.y : x.s.x;
    // The block's scale for rows g and g + 8, each as a half2 pair.
    const __half2 dg = u2h(__byte_perm(sw, 0, 0x1010)), dg8 = u2h(__byte_perm(sw, 0, 0x3232));
    const uint32_t k0 = 32 * kb + 8 * h + 2 * t;
    const uint32_t r0 = row0 + g, r8 = row0 + g + 8;
    // (code - 8) exactly, as f16 pairs: rows g and g + 8, columns k0 (+1) and k0 + 16 (+1); a nibble
    // at bits 0-3 of a half is 1024 + n less 1032, at bits 4-7 it is (1024 + 16 n) / 16 less 72.
    const __half2 c4[4] = {__hsub2(u2h((wd & kLow) | kMagic), bias),
                           __hfma2(u2h((wd & kHigh) | kMagic), sixteenth, bias16),
                           __hsub2(u2h((w8 & kLow) | kMagic), bias),
                           __hfma2(u2h((w8 & kHigh) | kMagic), sixteenth, bias16)};
    const uint32_t rows[4] = {r0, r0, r8, r8};
    const uint32_t cols[4] = {k0, k0 + 16, k0, k0 + 16};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      // (code - 8) * d is exact as a real product; hi is it rounded once to f16 (one f16 multiply), lo
      // the remainder rounded once (one fused multiply-add): the f32 split of the product, without
      // leaving f16.
      const __half2 d = j < 2 ? dg : dg8;
      const __half2 hi = __hmul2(c4[j], d);
      *reinterpret_cast<uint32_t*>(tile + swz(rows[j], cols[j])) = live ? h2u(hi) : 0u;
      if (tile_lo) {
        const __half2 lo = __hfma2(c4[j], d, __hneg2(hi));
        *reinterpret_cast<uint32_t*>(tile_lo + swz(rows[j], cols[j])) = live ? h2u(lo) : 0u;
      }
    }
  }
}

// One warp a (row group, block pair): lane (g, t) decodes its four code
// words exactly as dequant_tile does and writes the f16 pairs to [n][k].
// With `corr` (a Q4_1 matrix held as its Q4_0 part, corr[row][block] = 8 d
// + m), each weight is (code - 8) d + corr in f32, split into f16 part and
// remainder.
__global__ void dequant_f16_kernel(Q4Matrix w, __half* hi, __half* lo, const float* corr) {
  const uint32_t nbp = w.k / 64, lane = threadIdx.x & 31;
  const uint32_t item = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (item >= (w.n / 16) * nbp) return;
  const uint32_t rg = item / nbp, bp = item % nbp, g = lane >> 2, t = lane & 3;
  const uint4 c = w.codes[(size_t)item * 32 + lane];
  const uint2 sc = w.scales[(size_t)item * 8 + g];
  const uint32_t kLow = 0x000F000Fu, kHigh = 0x00F000F0u, kMagic = 0x64006400u;
  const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6408u));
  const __half2 sixteenth = __half2half2(__ushort_as_half((unsigned short)0x2C00u));
  const __half2 bias16 = __half2half2(__ushort_as_half((unsigned short)0xD480u));
  const uint32_t words[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
  for (int wi = 0; wi < 4; wi++) {
    const uint32_t kb = wi >> 1, h = wi & 1, wd = words[wi], w8 = wd >> 8;
    const uint32_t sw = kb ? sc.y : sc.x;
    const __half2 dg = u2h(__byte_perm(sw, 0, 0x1010)), dg8 = u2h(__byte_perm(sw, 0, 0x3232));
    const uint32_t k0 = 64 * bp + 32 * kb + 8 * h + 2 * t, r0 = rg * 16 + g, r8 = r0 + 8;
    const __half2 c4[4] = {__hsub2(u2h((wd & kLow) | kMagic), bias),
                           __hfma2(u2h((wd & kHigh) | kMagic), sixteenth, bias16),
                           __hsub2(u2h((w8 & kLow) | kMagic), bias),
                           __hfma2(u2h((w8 & kHigh) | kMagic), sixteenth, bias16)};
    const uint32_t rows[4] = {r0, r0, r8, r8};
    const uint32_t cols[4] = {k0, k0 + 16, k0, k0 + 16};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const __half2 d = j < 2 ? dg : dg8;
      const size_t at = (size_t)rows[j] * w.k + cols[j];
      if (corr) {
        const float c = corr[(size_t)rows[j] * (w.k / 32) + cols[j] / 32];
        const float2 cf = __half22float2(c4[j]), df = __half22float2(d);
        const float v0 = __fadd_rn(__fmul_rn(cf.x, df.x), c), v1 = __fadd_rn(__fmul_rn(cf.y, df.y), c);
        const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
        *reinterpret_cast<__half2*>(hi + at) = __halves2half2(h0, h1);
        if (lo)
          *reinterpret_cast<__half2*>(lo + at) = __halves2half2(__float2half_rn(__fsub_rn(v0, __half2float(h0))),
                                                                  __float2half_rn(__fsub_rn(v1, __half2float(h1))));
        continue;
      }
      const __half2 vh = __hmul2(c4[j], d);
      *reinterpret_cast<__half2*>(hi + at) = vh;
      if (lo) *reinterpret_cast<__half2*>(lo + at) = __hfma2(c4[j], d, __hneg2(vh));
    }
  }
}

FZ_DEV float apply_edit_table(const uint32_t* table, uint32_t layer, uint32_t neuron, uint32_t pos, float v) {
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
    float edited = value;
    if (e[1] == 1u) edited = value == 1.0f ? v : __fmul_rn(v, value);
    v = edited;
  }
  return v;
}

template <int BN, int XP, int WP>
struct Layout {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes * XP + kBBytes * WP;
  static constexpr int kStages = (200 * 1024) / kStageBytes > 6 ? 6 : (200 * 1024) / kStageBytes;
  static constexpr int kEpiBytes = kEpilogue * 32 * (kStageCols + 1) * 4;   // epilogue turn-around
  static constexpr int kSmem = kStages * kStageBytes + kEpiBytes + 1024;  // + alignment slack
};

// XP: passes over X (f16 hi, + lo); WP: passes over W (f16 hi, + lo).  The
// MMAs per 16 columns: X_hi.W_hi, X_lo.W_hi (XP = 2), X_hi.W_lo (WP = 2); the
// dropped X_lo.W_lo term is below 2^-22 relative.  WT: the weight tiles
// come by TMA from f16 copies (wmaps: gate or the matrix hi, lo, then up hi,
// lo) and the producer warps stand idle.
struct WMaps {
  CUtensorMap m[4];
};

template <int BN, int XP, int WP, int EPI, bool WT>
__global__ void __launch_bounds__(kThreadsG, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                const __grid_constant__ WMaps wmaps, const GemmArgs a) {
  constexpr int PASSES = XP;
  using L = Layout<BN, XP, WP>;
  constexpr int S = L::kStages;
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full[S];
  __shared__ __align__(8) uint64_t empty[S];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_base;
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  auto a_tile = [&](int s, int p) { return smem + s * L::kStageBytes + p * L::kABytes; };
  auto b_tile = [&](int s) { return smem + s * L::kStageBytes + XP * L::kABytes; };
  auto b_tile_lo = [&](int s) { return smem + s * L::kStageBytes + XP * L::kABytes + L::kBBytes; };
  float* epi_stage = reinterpret_cast<float*>(smem + S * L::kStageBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t K = a.w[0].k, nkt = K / kBK;
  const uint32_t half_bn = BN / 2;
  const uint32_t cols = EPI == kGemmGated ? half_bn : BN;       // weight rows (neurons) a tile
  const uint32_t mtiles = (a.m + kBM - 1) / kBM, ntiles = (a.w[0].n + cols - 1) / cols;
  // Work items: a tile and one of KS slices of its k-stages (KS divides nkt).
  const uint32_t KS = a.k_split > 1 ? a.k_split : 1u, nks = nkt / KS;
  const uint32_t tiles = mtiles * ntiles * KS;
  // Item t: tile t / KS (rows m0 = (tile % mtiles) * 128 of X, weight rows
  // n0 = (tile / mtiles) * cols) over k-stages (t % KS) * nks, + nks.
  auto m0_of = [&](uint32_t item) { return ((item / KS) % mtiles) * kBM; };
  auto n0_of = [&](uint32_t item) { return ((item / KS) / mtiles) * cols; };
  auto k0_of = [&](uint32_t item) { return (item % KS) * nks; };

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], WT ? 1 : 1 + kProducers);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpilogue);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"((uint32_t)(2 * BN))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // X tiles by TMA; X is the previous kernel's output.  The whole warp runs
    // the loop and waits, lane 0 issues.
    pdl_wait();
    uint32_t it = 0;
    bool stop = false;
    for (uint32_t tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x) {
      const uint32_t m0 = m0_of(tile), n0 = n0_of(tile), k0 = k0_of(tile);
      for (uint32_t kr = 0; kr < nks; kr++, it++) {
        const uint32_t kt = k0 + kr;
        const int s = (int)(it % S);
        const uint32_t round = it / S;
        if (!mbar_wait(&empty[s], (round + 1) & 1u, a.error, 1)) {
          stop = true;
          break;
        }
        if (lane == 0) {
          mbar_expect_tx(&full[s], (uint32_t)(L::kABytes * PASSES + (WT ? L::kBBytes * WP : 0)));
          tma_load_2d(a_tile(s, 0), &map_hi, &full[s], (int)(kt * kBK), (int)m0);
          if (PASSES == 2) tma_load_2d(a_tile(s, 1), &map_lo, &full[s], (int)(kt * kBK), (int)m0);
          if (WT) {
            // Weight rows n0 .. as the B tile's rows (gated: gate rows, then up rows).
            if (EPI == kGemmGated) {
              tma_load_2d(b_tile(s), &wmaps.m[0], &full[s], (int)(kt * kBK), (int)n0);
              tma_load_2d(b_tile(s) + half_bn * 128u, &wmaps.m[2], &full[s], (int)(kt * kBK), (int)n0);
              if (WP == 2) {
                tma_load_2d(b_tile_lo(s), &wmaps.m[1], &full[s], (int)(kt * kBK), (int)n0);
                tma_load_2d(b_tile_lo(s) + half_bn * 128u, &wmaps.m[3], &full[s], (int)(kt * kBK), (int)n0);
              }
            } else {
              tma_load_2d(b_tile(s), &wmaps.m[0], &full[s], (int)(kt * kBK), (int)n0);
              if (WP == 2) tma_load_2d(b_tile_lo(s), &wmaps.m[1], &full[s], (int)(kt * kBK), (int)n0);
            }
          }
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // The MMA issuer: the whole warp waits, lane 0 issues and commits.
    constexpr uint32_t idesc = instr_desc<BN>();
    uint32_t it = 0, tl = 0;
    bool stop = false;
    for (uint32_t tile = blockIdx.x; tile < tiles && !stop; tile += gridDim.x, tl++) {
      const uint32_t buf = tl & 1u, use = tl >> 1;
      // The epilogue has drained this accumulator (its previous use).
      if (!mbar_wait(&acc_empty[buf], (use + 1) & 1u, a.error, 5)) break;
      fence_after_sync();
      const uint32_t acc = tmem + buf * BN;
      for (uint32_t kt = 0; kt < nks; kt++, it++) {
        const int s = (int)(it % S);
        const uint32_t round = it / S;
        if (!mbar_wait(&full[s], round & 1u, a.error, 2)) {
          stop = true;
          break;
        }
        fence_after_sync();
        if (lane == 0) {
          const uint64_t db = smem_desc(b_tile(s));
          const uint64_t db_lo = smem_desc(b_tile_lo(s));
          const uint64_t da = smem_desc(a_tile(s, 0));
          const uint64_t da_lo = smem_desc(a_tile(s, XP - 1));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++) {
            // 16 columns of f16 = 32 bytes along K: +2 in the 16-byte address field.
            umma(acc, da + 2 * kk, db + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
            if (XP == 2) umma(acc, da_lo + 2 * kk, db + 2 * kk, idesc, 1u);
            if (WP == 2) umma(acc, da + 2 * kk, db_lo + 2 * kk, idesc, 1u);
          }
          umma_commit(&empty[s]);
        }
        __syncwarp();
      }
      if (!stop) {
        if (lane == 0) umma_commit(&acc_full[buf]);
        __syncwarp();
      }
    }
  } else if (warp < 2 + kProducers) {
    if (WT) {
      // (the weight tiles come by TMA)
    } else {
    // Weight producers: warps 2..9 dequantize BN / 16 row groups a stage, the
    // codes of the next two stages already in flight; the stages run on
    // across tiles (flat index q over this CTA's tiles x k-slices).
    const int pw = warp - 2;
    constexpr int kRgs = BN / 16;
    constexpr int kMine = kRgs / kProducers;       // row groups a warp, a stage
    static_assert(kRgs % kProducers == 0, "row groups split evenly over the producers");
    const uint32_t my_tiles = blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const uint32_t total = my_tiles * nks;
    auto rg_of = [&](uint32_t q, int j) {
      const uint32_t n0 = n0_of(blockIdx.x + (q / nks) * gridDim.x);
      const int r = pw + j * kProducers;
      return EPI == kGemmGated ? (n0 / 16 + (uint32_t)(r % (kRgs / 2))) : (n0 / 16 + (uint32_t)r);
    };
    auto mat_of = [&](int j) -> const Q4Matrix& {
      const int r = pw + j * kProducers;
      return (EPI == kGemmGated && r >= kRgs / 2) ? a.w[1] : a.w[0];
    };
    auto load_q = [&](uint32_t q, Codes (&dst)[kMine]) {
#pragma unroll
      for (int j = 0; j < kMine; j++) {
        const uint32_t rg = rg_of(q, j);
        dst[j] = load_codes(mat_of(j), rg, k0_of(blockIdx.x + (q / nks) * gridDim.x) + q % nks,
                            rg < mat_of(j).n / 16, lane);
      }
    };
    Codes A[kMine], B[kMine], C[kMine];
    bool stop = false;
    // One stage: stage q's codes are in `cur`; stage q + 2's load into `later`.
    auto step = [&](uint32_t q, Codes (&cur)[kMine], Codes (&later)[kMine]) {
      const int s = (int)(q % S);
      const uint32_t round = q / S;
      if (q + 2 < total) load_q(q + 2, later);
      if (!mbar_wait(&empty[s], (round + 1) & 1u, a.error, 3)) {
        stop = true;
        return;
      }
      unsigned char* tile = b_tile(s);
#pragma unroll
      for (int j = 0; j < kMine; j++) {
        const uint32_t rg = rg_of(q, j);
        dequant_tile(tile, WP == 2 ? b_tile_lo(s) : nullptr, (uint32_t)(pw + j * kProducers) * 16, cur[j],
                     rg < mat_of(j).n / 16, lane);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    };
    if (total > 0) load_q(0, A);
    if (total > 1) load_q(1, B);
    for (uint32_t q = 0; q < total && !stop; q += 3) {
      step(q, A, C);
      if (q + 1 < total && !stop) step(q + 1, B, A);
      if (q + 2 < total && !stop) step(q + 2, C, B);
    }
    }
  } else {
    // Epilogue: warps 10..17; warp w reads TMEM lanes 32 * (w % 4) .. + 31,
    // warps 10..13 the first half of the columns, warps 14..17 the second.
    const int ew = warp - 2 - kProducers;
    const uint32_t quarter = (uint32_t)warp & 3u;
    const int side = ew < 4 ? 0 : 1;
    float* stage = epi_stage + ew * 32 * (kStageCols + 1);
    uint32_t tl = 0;
    for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, tl++) {
      const uint32_t buf = tl & 1u, use = tl >> 1;
      if (!mbar_wait(&acc_full[buf], use & 1u, a.error, 4)) break;
      fence_after_sync();
      const uint32_t m0 = m0_of(tile), n0 = n0_of(tile);
      const uint32_t row = m0 + quarter * 32 + lane;
      const uint32_t lane_addr = tmem + buf * BN + ((quarter * 32u) << 16);
      if (EPI == kGemmWrite) {
        const uint32_t N = a.w[0].n;
        for (int c0 = side * (BN / 2); c0 < (side + 1) * (BN / 2); c0 += 32) {
          uint32_t r[32];
          tmem_ld32(lane_addr + (uint32_t)c0, r);
#pragma unroll
          for (int h = 0; h < 2; h++) {
#pragma unroll
            for (int i = 0; i < kStageCols; i++) stage[lane * (kStageCols + 1) + i] = __uint_as_float(r[h * kStageCols + i]);
            __syncwarp();
            // 16 consecutive columns of two rows a store instruction.
            const uint32_t n = n0 + (uint32_t)c0 + h * kStageCols + (lane & 15);
            for (int rr = lane >> 4; rr < 32; rr += 2) {
              const uint32_t orow = m0 + quarter * 32 + rr;
              if (orow < a.m && n < N) {
                float* o = a.out + (size_t)orow * a.out_stride + n;
                const float v = stage[rr * (kStageCols + 1) + (lane & 15)];
                if (KS > 1) atomicAdd(o, v);   // (a reduction: the result is not read)
                else *o = v;
              }
            }
            __syncwarp();
          }
        }
      } else {
        const uint32_t F = a.w[0].n;
        const uint32_t seq = row / a.seq_tokens;
        const uint32_t pos = (a.step ? a.step->position : a.position) + row % a.seq_tokens;
        const bool last = row % a.seq_tokens == a.seq_tokens - 1;
        for (int c0 = side * (int)(half_bn / 2); c0 < (side + 1) * (int)(half_bn / 2); c0 += 32) {
          uint32_t gr[32], ur[32];
          tmem_ld32(lane_addr + (uint32_t)c0, gr);
          tmem_ld32(lane_addr + half_bn + (uint32_t)c0, ur);
#pragma unroll
          for (int h = 0; h < 2; h++) {
#pragma unroll
            for (int i = 0; i < kStageCols; i++) {
              const uint32_t neuron = n0 + c0 + h * kStageCols + i;
              float v = __fmul_rn(gelu_tanh(__uint_as_float(gr[h * kStageCols + i])),
                                  __uint_as_float(ur[h * kStageCols + i]));
              if (a.edit_table && row < a.m && neuron < F)
                v = apply_edit_table(a.edit_table + seq * a.table_stride, a.layer, neuron, pos, v);
              if (a.capture_neurons && last && row < a.m && neuron < F)
                a.capture_neurons[seq * a.capture_stride + neuron] = v;
              stage[lane * (kStageCols + 1) + i] = v;
            }
            __syncwarp();
            const uint32_t n = n0 + (uint32_t)c0 + h * kStageCols + (lane & 15);
            for (int rr = lane >> 4; rr < 32; rr += 2) {
              const uint32_t orow = m0 + quarter * 32 + rr;
              if (orow < a.m && n < F) {
                const float v = stage[rr * (kStageCols + 1) + (lane & 15)];
                const size_t at = (size_t)orow * F + n;
                if (a.out) a.out[(size_t)orow * a.out_stride + n] = v;
                const __half hi = __float2half_rn(v);
                a.act_hi[at] = hi;
                if (a.act_lo) a.act_lo[at] = __float2half_rn(__fsub_rn(v, __half2float(hi)));
              }
            }
            __syncwarp();
          }
        }
      }
      // This accumulator may take the tile after next.
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  pdl_launch_dependents();
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * BN)) : "memory");
  }
}

__global__ void split_f16_kernel(const float* __restrict__ x, size_t n, __half* hi, __half* lo) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const __half h = __float2half_rn(v);
    hi[i] = h;
    if (lo) lo[i] = __float2half_rn(__fsub_rn(v, __half2float(h)));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// A 2D tensor map over an [rows][cols] f16 matrix: boxes of box_rows rows x
// 64 columns, 128-byte swizzle, rows past `rows` read as zeros.
bool make_map(CUtensorMap* map, const __half* base, uint32_t rows, uint32_t cols, uint32_t box_rows = kBM) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int XP, int WP, int EPI, bool WT>
cudaError_t launch_tiles(const GemmArgs& a, cudaStream_t stream, bool pdl) {
  constexpr int PASSES = XP;
  using L = Layout<BN, XP, WP>;
  static std::once_flag once;
  static cudaError_t configured = cudaSuccess;
  std::call_once(once, [] {
    configured = cudaFuncSetAttribute(gemm_kernel<BN, XP, WP, EPI, WT>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem);
  });
  if (configured != cudaSuccess) return configured;
  CUtensorMap map_hi, map_lo;
  if (!make_map(&map_hi, a.x_hi, a.m, a.w[0].k)) return cudaErrorInvalidValue;
  if (!make_map(&map_lo, PASSES == 2 ? a.x_lo : a.x_hi, a.m, a.w[0].k)) return cudaErrorInvalidValue;
  const uint32_t cols = EPI == kGemmGated ? BN / 2 : BN;
  WMaps wm{};
  if (WT) {
    const uint32_t n = a.w[0].n, k = a.w[0].k;
    const __half* lo0 = WP == 2 ? a.w_lo[0] : a.w_hi[0];
    if (!make_map(&wm.m[0], a.w_hi[0], n, k, cols) || !make_map(&wm.m[1], lo0, n, k, cols)) return cudaErrorInvalidValue;
    if (EPI == kGemmGated) {
      const __half* lo1 = WP == 2 ? a.w_lo[1] : a.w_hi[1];
      if (!make_map(&wm.m[2], a.w_hi[1], n, k, cols) || !make_map(&wm.m[3], lo1, n, k, cols))
        return cudaErrorInvalidValue;
    }
  }
  const uint32_t tiles = ((a.w[0].n + cols - 1) / cols) * ((a.m + kBM - 1) / kBM);
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  // Few tiles (few rows, or a narrow product): split K so that every SM has
  // an item, at least two k-stages an item, the slice count dividing the
  // stages; the partials meet in `out` by f32 reductions, so it is zeroed.
  GemmArgs g = a;
  g.k_split = 1;
  const uint32_t nkt = a.w[0].k / kBK;
  if (EPI == kGemmWrite && tiles < (uint32_t)sms) {
    for (uint32_t d = 2; d <= nkt / 2; d++)
      if (nkt % d == 0 && tiles * d <= (uint32_t)sms) g.k_split = d;
    if (g.k_split > 1) {
      const cudaError_t z = cudaMemset2DAsync(a.out, (size_t)a.out_stride * 4, 0, (size_t)a.w[0].n * 4, a.m, stream);
      if (z != cudaSuccess) return z;
    }
  }
  const uint32_t items = tiles * g.k_split;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min<uint32_t>(items, (uint32_t)sms));
  cfg.blockDim = dim3(kThreadsG);
  cfg.dynamicSmemBytes = L::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_kernel<BN, XP, WP, EPI, WT>, map_hi, map_lo, wm, g);
  if (e != cudaSuccess) (void)cudaGetLastError();
  return e;
}

}  // namespace

cudaError_t launch_gemm(const GemmArgs& a, int epilogue, cudaStream_t stream, bool pdl) {
  if (a.m == 0 || a.w[0].k % 64 || a.w[0].n % 16 || !a.x_hi || !a.error) return cudaErrorInvalidValue;
  // TMA wants 16-byte aligned rows: K f16 values a row, K a multiple of 64.
  if ((reinterpret_cast<uintptr_t>(a.x_hi) & 15) || (a.x_lo && (reinterpret_cast<uintptr_t>(a.x_lo) & 15)))
    return cudaErrorInvalidValue;
  // Exact weights (WP = 2) go with both halves of X: the f32-level product.
  const bool two = a.x_lo != nullptr, exact = two && a.exact_w;
  const bool wt = a.w_hi[0] != nullptr;
  if (wt) {
    if ((reinterpret_cast<uintptr_t>(a.w_hi[0]) & 15) || (exact && !a.w_lo[0])) return cudaErrorInvalidValue;
    if (epilogue == kGemmGated && (!a.w_hi[1] || (exact && !a.w_lo[1]))) return cudaErrorInvalidValue;
  }
  if (epilogue == kGemmGated) {
    if (!a.act_hi || a.w[1].n != a.w[0].n || a.w[1].k != a.w[0].k) return cudaErrorInvalidValue;
    if (wt)
      return exact ? launch_tiles<128, 2, 2, kGemmGated, true>(a, stream, pdl)
             : two ? launch_tiles<256, 2, 1, kGemmGated, true>(a, stream, pdl)
                   : launch_tiles<256, 1, 1, kGemmGated, true>(a, stream, pdl);
    return exact ? launch_tiles<128, 2, 2, kGemmGated, false>(a, stream, pdl)
           : two ? launch_tiles<256, 2, 1, kGemmGated, false>(a, stream, pdl)
                 : launch_tiles<256, 1, 1, kGemmGated, false>(a, stream, pdl);
  }
  if (!a.out) return cudaErrorInvalidValue;
  if (wt)
    return exact ? launch_tiles<128, 2, 2, kGemmWrite, true>(a, stream, pdl)
           : two ? launch_tiles<256, 2, 1, kGemmWrite, true>(a, stream, pdl)
                 : launch_tiles<256, 1, 1, kGemmWrite, true>(a, stream, pdl);
  return exact ? launch_tiles<128, 2, 2, kGemmWrite, false>(a, stream, pdl)
         : two ? launch_tiles<256, 2, 1, kGemmWrite, false>(a, stream, pdl)
               : launch_tiles<256, 1, 1, kGemmWrite, false>(a, stream, pdl);
}

cudaError_t launch_dequant_f16(const Q4Matrix& w, __half* hi, __half* lo, cudaStream_t stream, const float* corr) {
  if (!hi || w.k % 64 || w.n % 16) return cudaErrorInvalidValue;
  const size_t items = (size_t)(w.n / 16) * (w.k / 64);
  (void)cudaGetLastError();
  dequant_f16_kernel<<<(unsigned)((items + 7) / 8), 256, 0, stream>>>(w, hi, lo, corr);
  return cudaGetLastError();
}

cudaError_t launch_split_f16(const float* x, size_t n, __half* hi, __half* lo, cudaStream_t stream) {
  if (!n) return cudaSuccess;
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
  (void)cudaGetLastError();
  split_f16_kernel<<<blocks, 256, 0, stream>>>(x, n, hi, lo);
  return cudaGetLastError();
}

}  // namespace fz
