// The whole decode step (one token for each of up to 8 sequences) as one
// persistent kernel: every layer's norms, products, QK-norm/RoPE, attention
// and steering, then the final norm and the tied head, in one launch.
//
// Frizzle runs the step as ~300 dispatches (graph/graph.h:189-199); at batch 1
// the separate launches cost more than the 563 MB the step reads.  Here one
// CTA per SM walks the step's phases in order; a phase that needs another
// phase's whole output (the product's input vector) waits on a counter in
// global memory that the producing CTAs raise, and each CTA's weight tiles
// stream into a shared-memory ring by bulk copies (cp.async.bulk) issued by a
// producer warp that runs ahead of the phases, so the weights of the next
// phases arrive while the current phase waits.
#pragma once

#include "q4_matvec.cuh"

namespace fz {

// One layer as the decode kernel reads it (a device array of these).
struct DecodeLayer {
  Q4Matrix qkv, o, gate, up, down;
  const float *attn_norm, *q_norm, *k_norm, *post_attn_norm, *ffn_norm, *post_ffw_norm;
  const float* turns;              // RoPE theta_k / 2 pi, [d/2]
  uint16_t *key_cache, *value_cache;
  uint64_t seq_stride;             // cache elements between sequences
  uint32_t slots, window;
  // A Q4_1 down projection is held as its Q4_0 part (`down`) and the
  // correction corr[row][block] = 8 d + m, added times the block's sum of
  // the activation; null for a Q4_0 one.
  const float* down_corr;
};

// A layer's TMA tensor maps (CUtensorMap) of its key and value caches, 4D
// [sequence][slot][KV head][256]: boxes of 32 slots x 64 dimensions,
// 128-byte swizzle.
struct alignas(64) DecodeKvMaps {
  unsigned char map[2][128];
};

// Encodes m from d's caches (slots, seq_stride) for `sequences` sequences of
// kv_heads heads; false when the driver refuses.
bool make_kv_maps(DecodeKvMaps& m, const DecodeLayer& d, uint32_t kv_heads, uint32_t sequences);

constexpr uint32_t kDecodeMaxRows = 8;      // sequences one decode launch takes
constexpr uint32_t kDecodeOSlices = 2;      // K slices of the output projection
constexpr uint32_t kDecodeDownSlices = 4;   // K slices of the down projection
constexpr uint32_t kDecodeSyncFixed = 8;    // per-layer phase counters
constexpr uint32_t kDecodeMaxGroup = 6;     // query heads a KV head may serve
constexpr uint32_t kDecodeSplitKeys = 64;   // fewest keys of a split attention item
constexpr uint32_t kDecodeMaxSplits = 256;  // key splits the partial buffers are sized for
constexpr uint32_t kDecodeFoldSplits = 8;   // up to this many, the output projection folds the splits

// Byte offsets of the decode kernel's shared-memory regions (set by the launch).
struct DecodeLayout {
  uint32_t codes, scales, full, empty, uni, xf, rowbuf, part, stat, red, task_rg, best, flags, gains, tags, uses,
      kvbuf, kvbar, kvstate, corr, total;
};

struct DecodeArgs {
  const DeviceStep* step;          // position (every row is one sequence's next token)
  const DecodeLayer* layers;       // [n_layers], device memory
  const DecodeKvMaps* kv_maps;     // [n_layers], device memory
  uint32_t n_layers;
  uint32_t m;                      // sequences = rows
  uint32_t hidden, ffn, heads, kv_heads;
  float eps, scale_log2e;
  float* hidden_a;                 // [m][hidden]: the embedding rows in, the residual stream
  float* hidden_b;                 // [m][hidden]
  float* qkv;                      // [m][(heads + 2 kv_heads) 256] raw products (unused by the kernel)
  // The QKV products as flag-in-data words: value bits low, the producing
  // phase's epoch high ([kDecodeMaxRows][(heads + 2 kv_heads) 256]); the
  // attention polls them instead of a phase counter.
  unsigned long long* qkv_ll;       // (the epochs' step serial is step->padding[0], set by the engine)
  // The attention's output [kDecodeMaxRows][heads 256], and for 2..8 key
  // splits its split partials [rows][heads][8][256] and (max, sum) pairs
  // [rows][heads][8][2], all as flag-in-data words the output projection polls.
  unsigned long long* attn_ll;
  unsigned long long* act_ll;      // the gated activation [kDecodeMaxRows][ffn] (flag-in-data)
  // Several rows: each norm's normed rows [kDecodeMaxRows][hidden] (flag-in-data), row r made by CTA r
  // and read by every CTA for its fragments.
  unsigned long long* norm_ll;
  unsigned long long* part_o_ll;
  unsigned long long* part_ml_ll;
  float* attn;                     // [m][heads 256]
  float* y_attn;                   // [kDecodeOSlices][m][hidden] output-projection partials
  float* act;                      // [m][ffn]
  float* y_mlp;                    // [kDecodeDownSlices][m][hidden] down-projection partials
  float* partial_o;                // [m][heads][max_splits][256] attention split partials
  float* partial_ml;               // [m][heads][max_splits][2]
  uint32_t max_splits;
  uint32_t* sync;                  // decode_sync_words(...) words, zero at launch
  const uint32_t* edit_table;      // sequence 0's edit table, or null
  uint64_t table_stride;           // words between sequences' tables
  float* capture;                  // sequence 0's capture store, or null
  uint64_t capture_stride;         // floats between sequences' stores
  // The store's layout (capture.cpp:31-73): layer l's neurons at l * ffn;
  // its block of residual, attention addition, feed-forward addition and
  // query (then weights, stats, readout) at cap_region2 + l * cap_block +
  // heads * (keys of the layers before it), a layer of every cap_pattern
  // holding cap_keys_global keys a head, the others cap_keys_local.
  uint64_t cap_region2, cap_block;
  uint32_t cap_keys_local, cap_keys_global, cap_pattern;
  Q4Matrix head;                   // tied embedding
  const float* output_norm;
  float* logits;                   // [m][vocab], or null for no head
  unsigned long long* argmax;      // [m], cleared before the launch
  uint32_t* error;                 // nonzero when a bounded wait gave up
  // Optional phase timeline (global timer, ns): CTA c's event e at
  // trace[c * trace_stride + e], e = (layer * 6 + phase) * 5 + k with phase
  // 0 QKV, 1 attention, 2 O, 3 gate/up, 4 down, 5 head (in the last layer's
  // slots) and k 0 began waiting, 1 counter reached, 2 inputs staged (after
  // the prologue; attention: queries roped), 3 products done (attention:
  // keys folded), 4 done.  Then kDecodeTraceTail words: per phase the
  // time thread 0 waited for weight tiles (ns), the producer's time waiting
  // for free slots and issuing copies (ns), its tile count, and the global
  // timer at the CTA's entry and at its exit.  Null: no trace.
  unsigned long long* trace;
  uint32_t trace_stride;
  DecodeLayout lay;                // filled by launch_decode
};

constexpr uint32_t kDecodeTracePhases = 6;
constexpr uint32_t kDecodeTraceStamps = 5;
constexpr uint32_t kDecodeTraceTail = 11;   // (+ the CTA's entry and exit times)

inline size_t decode_sync_words(uint32_t layers, uint32_t rows, uint32_t kv_heads) {
  return (size_t)layers * (kDecodeSyncFixed + (size_t)rows * kv_heads);
}

// Whether the decode kernel takes this shape (head_dim 256, the grouping,
// hidden/ffn multiples of the slices, at most kDecodeMaxRows rows).
bool decode_supported(uint32_t rows, uint32_t hidden, uint32_t ffn, uint32_t heads, uint32_t kv_heads,
                      uint32_t head_dim);

// Raises the kernel's shared-memory limit on the current device for this
// shape (both row counts); call before the first launch and outside stream
// capture.
cudaError_t prepare_decode(uint32_t hidden, uint32_t ffn, uint32_t heads, uint32_t kv_heads);

// Cooperative launch, one CTA per SM.
cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t stream);

}  // namespace fz
