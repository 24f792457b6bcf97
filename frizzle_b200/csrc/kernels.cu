// Attention (split-K flash-decode with an in-kernel combine), the embedding
// gather, and top-64 selection with the draw.
#include <algorithm>

#include "kernels.cuh"
#include "q4_device.cuh"

namespace fz {
namespace {

constexpr int kHeadDim = 256;    // Gemma 3's d: one thread a dimension

// ------------------------------------------------------------ attention
//
// softmax(q . k_j / sqrt(d)) . v_j over keys j in [p - W + 1, p]
// (attention.h:18-30), in log2 units: q is staged times scale*log2(e) and
// exp2 replaces exp (attention.wgsl:198-215).  A CTA takes one row, one KV
// head (the G query heads that share it, so each key and value is read once
// per group) and one split of `split_keys` keys.  Rows whose keys span
// several splits leave (m, l, O) partials; the last of their CTAs folds them
// in split order and divides (the combine, attention.wgsl:403-438).  The
// fold factors keep the side holding the maximum at exactly 1
// (fold_factors, attention.wgsl:135-151).
template <int G>
__global__ void __launch_bounds__(256) attention_kernel(const AttentionArgs a) {
  __shared__ float sc[G][512];      // scores, then weights
  __shared__ float red[G][8];
  __shared__ float s_m[G], s_l[G];
  __shared__ uint32_t s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t row = blockIdx.z, kvh = blockIdx.y, split = blockIdx.x;
  pdl_wait();
  const uint32_t p = (a.step ? a.step->position : a.position) + row % a.seq_tokens;
  const uint32_t seq = row / a.seq_tokens;
  const uint32_t earliest = p + 1 > a.window ? p + 1 - a.window : 0;
  const uint32_t nkeys = p + 1 - earliest;
  const uint32_t nsplits = (nkeys + a.split_keys - 1) / a.split_keys;
  if (split >= nsplits) return;
  const uint32_t j0 = earliest + split * a.split_keys;
  const uint32_t j1 = min(j0 + a.split_keys, p + 1);
  const int n = (int)(j1 - j0);
  const uint16_t* kc = a.key_cache + seq * a.seq_stride;
  const uint16_t* vc = a.value_cache + seq * a.seq_stride;
  auto slot_of = [&](int jj) { return (size_t)((j0 + (uint32_t)jj) % a.slots) * a.kv_heads + kvh; };

  // q for the group, dims 8*lane .. 8*lane+7, times scale*log2(e).
  float qv[G][8];
#pragma unroll
  for (int h = 0; h < G; h++) {
    const float* q = a.q + ((size_t)row * a.heads + kvh * G + h) * kHeadDim + 8 * lane;
    const float4 x0 = reinterpret_cast<const float4*>(q)[0], x1 = reinterpret_cast<const float4*>(q)[1];
    const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int i = 0; i < 8; i++) qv[h][i] = mul(v[i], a.scale_log2e);
  }
  // Scores: each warp takes four keys at a time, loads first.
  constexpr int KU = 4;
  for (int base = warp * KU; base < n; base += 8 * KU) {
    uint4 kw[KU];
#pragma unroll
    for (int u = 0; u < KU; u++)
      if (base + u < n) kw[u] = *reinterpret_cast<const uint4*>(kc + slot_of(base + u) * kHeadDim + 8 * lane);
#pragma unroll
    for (int u = 0; u < KU; u++) {
      if (base + u < n) {
        const uint32_t w4[4] = {kw[u].x, kw[u].y, kw[u].z, kw[u].w};
        float k[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
          k[2 * i] = f.x;
          k[2 * i + 1] = f.y;
        }
#pragma unroll
        for (int h = 0; h < G; h++) {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < 8; i++) s = __fmaf_rn(qv[h][i], k[i], s);
          s = warp_sum(s);
          if (lane == 0) sc[h][base + u] = s;
        }
      }
    }
  }
  __syncthreads();
  // Per head: maximum, weights exp2(s - m), sum.
#pragma unroll
  for (int h = 0; h < G; h++) {
    float m = -INFINITY;
    for (int jj = tid; jj < n; jj += 256) m = fmaxf(m, sc[h][jj]);
    m = warp_max(m);
    if (lane == 0) red[h][warp] = m;
  }
  __syncthreads();
  if (tid < G) {
    float m = red[tid][0];
    for (int w = 1; w < 8; w++) m = fmaxf(m, red[tid][w]);
    s_m[tid] = m;
  }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < G; h++) {
    float l = 0.f;
    for (int jj = tid; jj < n; jj += 256) {
      const float e = exp2f(sc[h][jj] - s_m[h]);
      sc[h][jj] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) red[h][warp] = l;
  }
  __syncthreads();
  if (tid < G) {
    float l = 0.f;
    for (int w = 0; w < 8; w++) l += red[tid][w];
    s_l[tid] = l;
  }
  __syncthreads();
  // O = sum_j w_j v_j, thread tid the dimension tid, eight keys' loads at a time.
  float o[G];
#pragma unroll
  for (int h = 0; h < G; h++) o[h] = 0.f;
  constexpr int VU = 8;
  for (int base = 0; base < n; base += VU) {
    float v[VU];
#pragma unroll
    for (int u = 0; u < VU; u++) v[u] = base + u < n ? f16_unpack(vc[slot_of(base + u) * kHeadDim + tid]) : 0.f;
#pragma unroll
    for (int u = 0; u < VU; u++)
      if (base + u < n)
#pragma unroll
        for (int h = 0; h < G; h++) o[h] = __fmaf_rn(sc[h][base + u], v[u], o[h]);
  }
  pdl_launch_dependents();
  if (nsplits == 1) {
#pragma unroll
    for (int h = 0; h < G; h++) {
      const size_t at = ((size_t)row * a.heads + kvh * G + h) * kHeadDim + tid;
      const float v = __fdiv_rn(o[h], s_l[h]);
      a.out[at] = v;
      if (a.out_hi) {
        const __half hh = __float2half_rn(v);
        a.out_hi[at] = hh;
        if (a.out_lo) a.out_lo[at] = __float2half_rn(__fsub_rn(v, __half2float(hh)));
      }
    }
    return;
  }
#pragma unroll
  for (int h = 0; h < G; h++) {
    const size_t at = ((size_t)row * a.heads + kvh * G + h) * a.splits + split;
    a.partial_o[at * kHeadDim + tid] = o[h];
    if (tid == 0) {
      a.partial_ml[at * 2] = s_m[h];
      a.partial_ml[at * 2 + 1] = s_l[h];
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(a.counters + row * a.kv_heads + kvh, 1u) == nsplits - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
#pragma unroll
  for (int h = 0; h < G; h++) {
    const size_t base = ((size_t)row * a.heads + kvh * G + h) * a.splits;
    float m = -INFINITY;
    for (uint32_t s = 0; s < nsplits; s++) m = fmaxf(m, __ldcg(a.partial_ml + (base + s) * 2));
    float l = 0.f, acc = 0.f;
    for (uint32_t s = 0; s < nsplits; s++) {
      const float ms = __ldcg(a.partial_ml + (base + s) * 2);
      const float f = ms == m ? 1.0f : exp2f(ms - m);
      l = __fmaf_rn(__ldcg(a.partial_ml + (base + s) * 2 + 1), f, l);
      acc = __fmaf_rn(__ldcg(a.partial_o + (base + s) * kHeadDim + tid), f, acc);
    }
    const size_t at = ((size_t)row * a.heads + kvh * G + h) * kHeadDim + tid;
    const float v = __fdiv_rn(acc, l);
    a.out[at] = v;
    if (a.out_hi) {
      const __half hh = __float2half_rn(v);
      a.out_hi[at] = hh;
      if (a.out_lo) a.out_lo[at] = __float2half_rn(__fsub_rn(v, __half2float(hh)));
    }
  }
  if (tid == 0) a.counters[row * a.kv_heads + kvh] = 0u;
}

// ------------------------------------------------------------ embed

__global__ void embed_kernel(const EmbedArgs a) {
  const uint32_t i = blockIdx.x;
  pdl_wait();
  if (i == 0 && threadIdx.x < a.seqs) a.argmax[threadIdx.x] = 0ull;
  const uint32_t seq = i / a.seq_tokens;
  const uint32_t token = a.step->fed ? a.records[seq * 4] : a.ids[i];
  const Q4Matrix& mat = a.table;
  if (token >= mat.n) return;
  if (a.q8_codes) {
    // Q8_0 (q8_0.wgsl's unpack): code x d in f32, then the scale.
    const uint8_t* row = a.q8_codes + (size_t)token * mat.k;
    const uint16_t* d = a.q8_scales + (size_t)token * (mat.k / 32);
    float* o = a.hidden + (size_t)i * mat.k;
    for (uint32_t j = threadIdx.x; j < mat.k; j += blockDim.x)
      o[j] = mul(mul((float)(int8_t)row[j], f16_unpack(d[j / 32])), a.scale);
    pdl_launch_dependents();
    return;
  }
  const uint32_t NBP = mat.k / 64, KB = mat.k / 32;
  const uint32_t rg = token / 16, rr = token % 16, g = rr % 8, hsel = rr / 8;
  for (uint32_t j = threadIdx.x; j < KB * 8; j += blockDim.x) {
    const uint32_t kb = j / 8, h = (j / 4) % 2, t = j % 4;
    const uint32_t bp = kb / 2, kbi = kb % 2;
    const uint4 c = mat.codes[((size_t)rg * NBP + bp) * 32 + g * 4 + t];
    const uint32_t wi = kbi * 2 + h;
    const uint32_t w = wi == 0 ? c.x : wi == 1 ? c.y : wi == 2 ? c.z : c.w;
    const uint2 sc = mat.scales[((size_t)rg * NBP + bp) * 8 + g];
    const uint32_t sw = kbi ? sc.y : sc.x;
    const float d = __half2float(__ushort_as_half((unsigned short)(hsel ? sw >> 16 : sw & 0xffffu)));
    const uint32_t q0 = (w >> (8 * hsel)) & 0xffu, q1 = (w >> (16 + 8 * hsel)) & 0xffu;
    const uint32_t k0 = 32 * kb + 8 * h + 2 * t;
    float* o = a.hidden + (size_t)i * mat.k;
    o[k0] = mul(mul((float)(q0 & 0xF) - 8.0f, d), a.scale);
    o[k0 + 1] = mul(mul((float)(q1 & 0xF) - 8.0f, d), a.scale);
    o[k0 + 16] = mul(mul((float)(q0 >> 4) - 8.0f, d), a.scale);
    o[k0 + 17] = mul(mul((float)(q1 >> 4) - 8.0f, d), a.scale);
  }
  pdl_launch_dependents();
}

// ------------------------------------------------------------ selection

constexpr int kTile = 4096;      // logits a selection CTA sorts
constexpr int kCandidates = 64;  // kernels::kCandidates

FZ_DEV unsigned long long packed_key(float v, uint32_t id) {
  return ((unsigned long long)topk_key(__float_as_uint(v)) << 32) | (0xFFFFFFFFu - id);
}

// Descending bitonic sort of n (a power of two) keys in shared memory.
FZ_DEV void bitonic_desc(unsigned long long* k, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long x = k[lo], y = k[hi];
        if ((x < y) == desc) {
          k[lo] = y;
          k[hi] = x;
        }
      }
      __syncthreads();
    }
  }
}

FZ_DEV float temperature_of(const SelectArgs& a) { return a.step->temperature; }

// The top 64 of one tile of a row of logits into best[0 .. 63] (topk.wgsl
// first/merge: the same set and order, by a sort of the tile).
FZ_DEV void tile_top64(const float* l, uint32_t vocab, uint32_t tile, unsigned long long* keys,
                       unsigned long long* best) {
  for (int i = threadIdx.x; i < kTile; i += blockDim.x) {
    const uint32_t id = tile * kTile + i;
    keys[i] = id < vocab ? packed_key(l[id], id) : 0ull;
  }
  __syncthreads();
  bitonic_desc(keys, kTile);
  if (threadIdx.x < kCandidates) best[threadIdx.x] = keys[threadIdx.x];
}

// The best 64 of the tiles' candidates (n of them at `tile_best`), as
// (logit bits, token) pairs: pair i's bits at out[2i], its token at
// out[2i + 1] (kernels::kCandidates pairs, best first).
FZ_DEV void merge_top64(const unsigned long long* tile_best, int n, unsigned long long* keys, uint32_t* out) {
  int padded = 64;
  while (padded < n) padded <<= 1;
  for (int i = threadIdx.x; i < padded; i += blockDim.x) keys[i] = i < n ? tile_best[i] : 0ull;
  __syncthreads();
  bitonic_desc(keys, padded);
  if (threadIdx.x < kCandidates) {
    const unsigned long long k = keys[threadIdx.x];
    out[2 * threadIdx.x] = k ? topk_bits((uint32_t)(k >> 32)) : 0u;
    out[2 * threadIdx.x + 1] = k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFu) : 0xFFFFFFFFu;
  }
}

// Each CTA keeps the top 64 of its tile of logits.
__global__ void __launch_bounds__(512) select_tiles_kernel(const SelectArgs a) {
  __shared__ unsigned long long keys[kTile];
  pdl_wait();
  if (!(temperature_of(a) > 0.0f)) return;
  const uint32_t seq = blockIdx.y, tile = blockIdx.x, tiles = gridDim.x;
  tile_top64(a.logits + (size_t)seq * a.vocab, a.vocab, tile, keys,
             a.tile_best + ((size_t)seq * tiles + tile) * kCandidates);
}

FZ_DEV float unit_interval(uint32_t w) {
  return __fadd_rn(__fmul_rn((float)(w >> 9), 1.0f / 8388608.0f), 1.0f / 16777216.0f);
}

// Merge the tiles' candidates and draw (draw.wgsl:78-170); at temperature 0
// the record is the head's greedy maximum.
__global__ void __launch_bounds__(512) select_draw_kernel(const SelectArgs a, uint32_t tiles) {
  __shared__ unsigned long long keys[kTile];
  __shared__ float tempered[kCandidates], weight[kCandidates], running[kCandidates];
  __shared__ uint32_t above[kCandidates];
  pdl_wait();
  const uint32_t seq = blockIdx.x;
  const DeviceStep& st = *a.step;
  const uint2 seed = a.seeds ? make_uint2(a.seeds[2 * seq], a.seeds[2 * seq + 1]) : make_uint2(st.seed[0], st.seed[1]);
  const uint4 rnd = philox(make_uint4(st.position + st.tokens, 0u, 0u, 0u), seed);
  const float u = unit_interval(rnd.x);
  uint32_t* rec = a.records + seq * 4;
  if (!(st.temperature > 0.0f)) {
    if (threadIdx.x == 0) {
      const unsigned long long best = a.argmax[seq];
      const uint32_t bits = topk_bits((uint32_t)(best >> 32));
      const bool failed = (bits & 0x7F800000u) == 0x7F800000u;
      rec[0] = failed ? 0u : 0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu);
      rec[1] = failed ? 1u : 0u;
      rec[2] = __float_as_uint(u);
      rec[3] = 0u;
    }
    return;
  }
  uint32_t* cand = a.candidates + seq * kCandidates * 2;
  merge_top64(a.tile_best + (size_t)seq * tiles * kCandidates, (int)(tiles * kCandidates), keys, cand);
  __syncthreads();
  const uint32_t k = min(st.top_k, (uint32_t)kCandidates);
  const bool use_top_p = st.top_p < 1.0f;
  const uint32_t first_bits = cand[0];
  const bool failed = (first_bits & 0x7F800000u) == 0x7F800000u;
  const uint32_t t = threadIdx.x;
  if (t < k) {
    const uint32_t mine_bits = cand[2 * t];
    weight[t] = 0.f;
    tempered[t] = 0.f;
    above[t] = 0u;
    if (!failed && mine_bits != 0xFF800000u) {
      const float first = __uint_as_float(first_bits), mine = __uint_as_float(mine_bits);
      if (use_top_p) weight[t] = expf(sub(mine, first));
      tempered[t] = expf(__fdiv_rn(sub(mine, first), st.temperature));
      above[t] = (st.min_p == 0.0f || mine >= add(first, st.log_min_p)) ? 1u : 0u;
    }
  }
  __syncthreads();
  if (t != 0) return;
  if (use_top_p) {
    float sum = 0.f;
    for (uint32_t i = 0; i < k; i++) sum = add(sum, weight[i]);
    if (!failed)
      for (uint32_t i = 0; i < k; i++) weight[i] = __fdiv_rn(weight[i], sum);
  }
  uint32_t kept = k;
  float cumulative = 0.f, tsum = 0.f;
  for (uint32_t i = 0; i < k; i++) {
    tsum = add(tsum, tempered[i]);
    running[i] = tsum;
    if (use_top_p) {
      cumulative = add(cumulative, weight[i]);
      if (cumulative >= st.top_p) {
        kept = i + 1;
        break;
      }
    }
  }
  uint32_t survivors = 1;
  while (survivors < kept && above[survivors] == 1u) survivors++;
  const float goal = mul(u, running[survivors - 1]);
  uint32_t chosen = survivors - 1;
  for (uint32_t i = 0; i < survivors; i++)
    if (running[i] > goal) {
      chosen = i;
      break;
    }
  rec[0] = failed ? 0u : cand[2 * chosen + 1];
  rec[1] = failed ? 1u : 0u;
  rec[2] = __float_as_uint(u);
  rec[3] = 0u;
}

// ------------------------------------------------------------ capture
//
// The capture's attention weights and statistics (capture/weights.h:24-62;
// the scores of attention.wgsl:277-295, the fold's m and l, :394-395 and
// :434-436) for the captured row of each sequence, at p = position + tokens
// - 1.  A CTA takes one (KV head, layer, sequence) and the G query heads
// that share the KV head.  Key i < count = min(p + 1, keys), at position
// earliest + i (earliest = p + 1 - count), is scored by one thread in the
// order the CPU restatement follows: q staged times scale*log2(e), then
// s += ((q0 k0 + q1 k1) + q2 k2) + q3 k3 over the head's 64 quads.  m is the
// largest score, l the sum of exp2(s - m) (each thread's keys in order, then
// a fixed tree), and the weights exp2(s - m) / l overwrite the scores; keys
// count .. keys - 1 get 0.  The scores are formed here from the captured
// query and the key cache rather than kept by the attention kernels, whose
// tensor-core products round differently: the weights are a function of
// these scores and these statistics, as weights.h states them.
template <int G>
__global__ void __launch_bounds__(256) attention_weights_kernel(const WeightsArgs a) {
  __shared__ float qs[G][kHeadDim];
  __shared__ float red[G][8];
  __shared__ float stat[2][G];
  pdl_wait();
  const uint32_t kvh = blockIdx.x, seq = blockIdx.z;
  const CaptureLayer L = a.layers[blockIdx.y];
  const DeviceStep& st = *a.step;
  const uint32_t p = st.position + st.tokens - 1;
  const uint32_t count = min(p + 1, L.keys), earliest = p + 1 - count;
  float* store = a.store + (size_t)seq * a.store_stride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int h = 0; h < G; h++)
    qs[h][tid] = mul(store[L.query + (size_t)(kvh * G + h) * kHeadDim + tid], a.scale_log2e);
  __syncthreads();
  const uint16_t* kc = L.key_cache + (size_t)seq * L.seq_stride;
  auto at = [&](int h, uint32_t i) { return L.weights + (size_t)(kvh * G + h) * L.keys + i; };
  float top[G];
#pragma unroll
  for (int h = 0; h < G; h++) top[h] = -INFINITY;
  for (uint32_t i = tid; i < count; i += 256) {
    const uint2* kr =
        reinterpret_cast<const uint2*>(kc + ((size_t)((earliest + i) % L.slots) * a.kv_heads + kvh) * kHeadDim);
    float s[G];
#pragma unroll
    for (int h = 0; h < G; h++) s[h] = 0.f;
#pragma unroll 4
    for (int w = 0; w < kHeadDim / 4; w++) {
      const uint2 u = __ldg(kr + w);
      const float k0 = f16_unpack((uint16_t)(u.x & 0xFFFFu)), k1 = f16_unpack((uint16_t)(u.x >> 16));
      const float k2 = f16_unpack((uint16_t)(u.y & 0xFFFFu)), k3 = f16_unpack((uint16_t)(u.y >> 16));
#pragma unroll
      for (int h = 0; h < G; h++) {
        const float* q = &qs[h][4 * w];
        s[h] = add(s[h], add(add(add(mul(q[0], k0), mul(q[1], k1)), mul(q[2], k2)), mul(q[3], k3)));
      }
    }
#pragma unroll
    for (int h = 0; h < G; h++) {
      store[at(h, i)] = s[h];
      top[h] = fmaxf(top[h], s[h]);
    }
  }
#pragma unroll
  for (int h = 0; h < G; h++) {
    const float v = warp_max(top[h]);
    if (lane == 0) red[h][warp] = v;
  }
  __syncthreads();
  if (tid < G) {
    float m = red[tid][0];
    for (int w = 1; w < 8; w++) m = fmaxf(m, red[tid][w]);
    stat[0][tid] = m;
  }
  __syncthreads();
  float sum[G];
#pragma unroll
  for (int h = 0; h < G; h++) sum[h] = 0.f;
  for (uint32_t i = tid; i < count; i += 256) {
#pragma unroll
    for (int h = 0; h < G; h++) sum[h] = add(sum[h], exp2f(sub(store[at(h, i)], stat[0][h])));
  }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < G; h++) {
    const float v = warp_sum(sum[h]);
    if (lane == 0) red[h][warp] = v;
  }
  __syncthreads();
  if (tid < G) {
    float l = red[tid][0];
    for (int w = 1; w < 8; w++) l = add(l, red[tid][w]);
    stat[1][tid] = l;
    store[L.stats + 2 * (kvh * G + tid)] = stat[0][tid];
    store[L.stats + 2 * (kvh * G + tid) + 1] = l;
  }
  __syncthreads();
  for (uint32_t i = tid; i < L.keys; i += 256) {
#pragma unroll
    for (int h = 0; h < G; h++)
      store[at(h, i)] = i < count ? __fdiv_rn(exp2f(sub(store[at(h, i)], stat[0][h])), stat[1][h]) : 0.f;
  }
}

// Readout row g (sequence g / (layers - 1), layer g % (layers - 1)): the
// residual stream as that layer leaves it, which is the next layer's
// captured residual (capture.h:26-33), copied into rows [n][width].
__global__ void __launch_bounds__(256) readout_rows_kernel(const ReadoutArgs a, uint32_t g0) {
  pdl_wait();
  const uint32_t g = g0 + blockIdx.x, per = a.n_layers - 1, seq = g / per, l = g % per;
  const float4* src = reinterpret_cast<const float4*>(a.store + (size_t)seq * a.store_stride + a.layers[l + 1].residual);
  float4* dst = reinterpret_cast<float4*>(a.rows + (size_t)blockIdx.x * a.width);
  for (uint32_t i = threadIdx.x; i < a.width / 4; i += blockDim.x) dst[i] = src[i];
}

// The top 64 of each tile of each readout row's logits.
__global__ void __launch_bounds__(512) readout_tiles_kernel(const ReadoutArgs a) {
  __shared__ unsigned long long keys[kTile];
  pdl_wait();
  const uint32_t r = blockIdx.y, tile = blockIdx.x, tiles = gridDim.x;
  tile_top64(a.logits + (size_t)r * a.vocab, a.vocab, tile, keys, a.tile_best + ((size_t)r * tiles + tile) * kCandidates);
}

// Merges row r's tiles into its layer's readout slot: row g0 + r of the
// layers before the last, or with `last`, sequence g0 + r's last layer.
__global__ void __launch_bounds__(512) readout_merge_kernel(const ReadoutArgs a, uint32_t g0, uint32_t tiles,
                                                            uint32_t last) {
  __shared__ unsigned long long keys[kTile];
  pdl_wait();
  const uint32_t g = g0 + blockIdx.x, per = a.n_layers - 1;
  const uint32_t seq = last ? g : g / per, l = last ? per : g % per;
  uint32_t* out = reinterpret_cast<uint32_t*>(a.store + (size_t)seq * a.store_stride + a.layers[l].readout);
  merge_top64(a.tile_best + (size_t)blockIdx.x * tiles * kCandidates, (int)(tiles * kCandidates), keys, out);
}

cudaError_t launch(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
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

cudaError_t launch_attention(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
  if (a.head_dim != kHeadDim || a.heads % a.kv_heads || a.heads / a.kv_heads > 8 || a.split_keys > 512 ||
      a.split_keys == 0)
    return cudaErrorInvalidValue;
  AttentionArgs copy = a;
  void* args[] = {&copy};
  const dim3 grid(a.splits, a.kv_heads, a.m);
  switch (a.heads / a.kv_heads) {
    case 1: return launch((const void*)attention_kernel<1>, grid, dim3(256), 0, stream, pdl, args);
    case 2: return launch((const void*)attention_kernel<2>, grid, dim3(256), 0, stream, pdl, args);
    case 4: return launch((const void*)attention_kernel<4>, grid, dim3(256), 0, stream, pdl, args);
    case 8: return launch((const void*)attention_kernel<8>, grid, dim3(256), 0, stream, pdl, args);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_embed(const EmbedArgs& a, cudaStream_t stream, bool pdl) {
  if (a.seqs > 256) return cudaErrorInvalidValue;
  EmbedArgs copy = a;
  void* args[] = {&copy};
  return launch((const void*)embed_kernel, dim3(a.m), dim3(256), 0, stream, pdl, args);
}

cudaError_t launch_attention_weights(const WeightsArgs& a, uint32_t layers, uint32_t seqs, cudaStream_t stream,
                                     bool pdl) {
  if (a.head_dim != kHeadDim || a.kv_heads == 0 || a.heads % a.kv_heads) return cudaErrorInvalidValue;
  WeightsArgs copy = a;
  void* args[] = {&copy};
  const dim3 grid(a.kv_heads, layers, seqs);
  switch (a.heads / a.kv_heads) {
    case 1: return launch((const void*)attention_weights_kernel<1>, grid, dim3(256), 0, stream, pdl, args);
    case 2: return launch((const void*)attention_weights_kernel<2>, grid, dim3(256), 0, stream, pdl, args);
    case 4: return launch((const void*)attention_weights_kernel<4>, grid, dim3(256), 0, stream, pdl, args);
    case 8: return launch((const void*)attention_weights_kernel<8>, grid, dim3(256), 0, stream, pdl, args);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_readout_rows(const ReadoutArgs& a, uint32_t g0, uint32_t n, cudaStream_t stream, bool pdl) {
  if (a.n_layers < 2 || a.width % 4 || n == 0) return cudaErrorInvalidValue;
  ReadoutArgs copy = a;
  void* args[] = {&copy, &g0};
  return launch((const void*)readout_rows_kernel, dim3(n), dim3(256), 0, stream, pdl, args);
}

cudaError_t launch_readout_select(const ReadoutArgs& a, uint32_t g0, uint32_t n, bool last, cudaStream_t stream,
                                  bool pdl) {
  uint32_t tiles = (a.vocab + kTile - 1) / kTile;
  if (tiles * kCandidates > (uint32_t)kTile || n == 0) return cudaErrorInvalidValue;
  ReadoutArgs copy = a;
  void* args1[] = {&copy};
  cudaError_t e = launch((const void*)readout_tiles_kernel, dim3(tiles, n), dim3(512), 0, stream, pdl, args1);
  if (e != cudaSuccess) return e;
  uint32_t lf = last ? 1u : 0u;
  void* args2[] = {&copy, &g0, &tiles, &lf};
  return launch((const void*)readout_merge_kernel, dim3(n), dim3(512), 0, stream, pdl, args2);
}

uint32_t select_tiles(uint32_t vocab) { return (vocab + kTile - 1) / kTile; }

cudaError_t launch_select(const SelectArgs& a, cudaStream_t stream, bool pdl) {
  const uint32_t tiles = select_tiles(a.vocab);
  if (tiles * kCandidates > (uint32_t)kTile) return cudaErrorInvalidValue;
  SelectArgs copy = a;
  void* args1[] = {&copy};
  cudaError_t e = launch((const void*)select_tiles_kernel, dim3(tiles, a.seqs), dim3(512), 0, stream, pdl, args1);
  if (e != cudaSuccess) return e;
  uint32_t t = tiles;
  void* args2[] = {&copy, &t};
  return launch((const void*)select_draw_kernel, dim3(a.seqs), dim3(512), 0, stream, pdl, args2);
}


// ------------------------------------------------------------ step inputs and outputs

namespace {

__global__ void __launch_bounds__(256) stage_kernel(const StageArgs a) {
  const uint32_t n = gridDim.x * blockDim.x, i0 = blockIdx.x * blockDim.x + threadIdx.x;
  constexpr uint32_t kStepWords = sizeof(DeviceStep) / 4;
  const uint32_t* sh = reinterpret_cast<const uint32_t*>(a.step_h);
  uint32_t* sd = reinterpret_cast<uint32_t*>(a.step_d);
  for (uint32_t i = i0; i < kStepWords; i += n) sd[i] = sh[i];
  for (uint32_t i = i0; i < a.seed_words; i += n) a.seeds_d[i] = a.seeds_h[i];
  for (uint32_t i = i0; i < a.id_words; i += n) a.ids_d[i] = a.ids_h[i];
  for (uint32_t i = i0; i < a.zero_words; i += n) a.zero[i] = 0u;
}

__global__ void q4_1_split_kernel(const uint8_t* src, size_t blocks, uint8_t* dst, float* corr) {
  for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < blocks; b += (size_t)gridDim.x * blockDim.x) {
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src + 20 * b);
    const uint32_t dm = s32[0];
    uint16_t* d16 = reinterpret_cast<uint16_t*>(dst + 18 * b);
    d16[0] = (uint16_t)(dm & 0xffffu);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      d16[1 + 2 * i] = (uint16_t)(s32[1 + i] & 0xffffu);
      d16[2 + 2 * i] = (uint16_t)(s32[1 + i] >> 16);
    }
    corr[b] = add(mul(8.0f, f16_unpack((uint16_t)(dm & 0xffffu))), f16_unpack((uint16_t)(dm >> 16)));
  }
}

// A CTA: the block sums of every row of x into shared memory (32 values in
// order), then each warp one output at a time over the blocks.
__global__ void __launch_bounds__(256) block_correction_kernel(const float* x, uint32_t m, uint32_t k,
                                                               const float* corr, uint32_t n, float* y) {
  extern __shared__ float sums[];   // [m][k / 32]
  const uint32_t kb = k / 32, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t i = threadIdx.x; i < m * kb; i += blockDim.x) {
    const float* v = x + (size_t)(i / kb) * k + (i % kb) * 32;
    float s = 0.f;
    for (int j = 0; j < 32; j++) s = add(s, v[j]);
    sums[i] = s;
  }
  __syncthreads();
  for (uint32_t o = blockIdx.x * 8 + warp; o < n; o += gridDim.x * 8) {
    const float* c = corr + (size_t)o * kb;
    for (uint32_t r = 0; r < m; r++) {
      float acc = 0.f;
      for (uint32_t b = lane; b < kb; b += 32) acc = __fmaf_rn(c[b], sums[r * kb + b], acc);
      acc = warp_sum(acc);
      if (lane == 0) y[(size_t)r * n + o] = add(y[(size_t)r * n + o], acc);
    }
  }
}

__global__ void __launch_bounds__(256) argmax_rows_kernel(const float* logits, uint32_t v, unsigned long long* argmax) {
  const uint32_t r = blockIdx.y;
  unsigned long long best = 0ull;
  for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < v; t += gridDim.x * blockDim.x)
    best = max(best, q4dev::head_key(logits[(size_t)r * v + t], t));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0 && best) atomicMax(argmax + r, best);
}

__global__ void delay_kernel(uint32_t ns) {
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t i = 0; i < (1u << 20); i++) {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 >= ns) break;
    __nanosleep(500);
  }
}

__global__ void __launch_bounds__(64) publish_kernel(const PublishArgs a) {
  for (uint32_t i = threadIdx.x; i < a.record_words; i += blockDim.x) a.records_h[i] = a.records_d[i];
  if (threadIdx.x == 0) a.error_h[0] = *reinterpret_cast<const volatile uint32_t*>(a.error_d);
}

}  // namespace

cudaError_t launch_stage(const StageArgs& a, cudaStream_t stream) {
  const uint32_t words = std::max(std::max(a.id_words, a.zero_words), std::max(a.seed_words, 16u));
  const uint32_t blocks = std::min(64u, (words + 255u) / 256u);
  stage_kernel<<<blocks, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_q4_1_split(const uint8_t* q4_1_blocks, size_t blocks, uint8_t* q4_0_blocks, float* corr,
                              cudaStream_t stream) {
  if (reinterpret_cast<uintptr_t>(q4_1_blocks) % 4 || reinterpret_cast<uintptr_t>(q4_0_blocks) % 2)
    return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)std::min<size_t>((blocks + 255) / 256, 148 * 8);
  q4_1_split_kernel<<<std::max(1u, grid), 256, 0, stream>>>(q4_1_blocks, blocks, q4_0_blocks, corr);
  return cudaGetLastError();
}

cudaError_t launch_block_correction(const float* x, uint32_t m, uint32_t k, const float* corr, uint32_t n, float* y,
                                    cudaStream_t stream) {
  const size_t smem = (size_t)m * (k / 32) * 4;
  if (k % 32 || smem > 48 * 1024) return cudaErrorInvalidValue;
  const unsigned grid = std::min(148u, (n + 7) / 8);
  block_correction_kernel<<<grid, 256, smem, stream>>>(x, m, k, corr, n, y);
  return cudaGetLastError();
}

cudaError_t launch_argmax_rows(const float* logits, uint32_t m, uint32_t v, unsigned long long* argmax,
                               cudaStream_t stream) {
  argmax_rows_kernel<<<dim3(64, m), 256, 0, stream>>>(logits, v, argmax);
  return cudaGetLastError();
}

cudaError_t launch_delay(uint32_t ns, cudaStream_t stream) {
  delay_kernel<<<1, 1, 0, stream>>>(ns);
  return cudaGetLastError();
}

cudaError_t launch_publish(const PublishArgs& a, cudaStream_t stream) {
  publish_kernel<<<1, 64, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace fz
