// Attention, embedding gather, selection and draw kernels (launch side).
#pragma once

#include "fz_common.cuh"
#include "q4_matvec.cuh"

namespace fz {

struct AttentionArgs {
  const DeviceStep* step;          // or null for `position`
  uint32_t position;
  const float* q;                  // [m][heads][d], after rope
  const uint16_t* key_cache;       // [seqs][slots][kv_heads][d]
  const uint16_t* value_cache;
  uint64_t seq_stride;
  uint32_t slots;
  uint32_t heads, kv_heads, head_dim;
  uint32_t window;
  uint32_t seq_tokens;             // T
  uint32_t m;                      // rows
  float scale_log2e;
  uint32_t split_keys;             // keys a split
  uint32_t splits;                 // grid.x: the most splits any row needs
  float* partial_o;                // [m][heads][splits][d]
  float* partial_ml;               // [m][heads][splits][2]
  uint32_t* counters;              // [m][kv_heads], zero between launches
  float* out;                      // [m][heads][d]
  __half* out_hi;                  // [m][heads][d] f16 of out, or null
  __half* out_lo;                  // its f16 remainder, or null
  // The tensor-core prefill form: the layer's key and value cache tensor maps
  // (two CUtensorMaps, 4D [sequence][slot][KV head][256], 32-slot x
  // 64-dimension boxes, 128-byte swizzle; device memory, 64-byte aligned)
  // and a device word set nonzero when one of its bounded waits gives up.
  const void* kv_maps;
  uint32_t* error;
  // Its key-range split: with split_part set, at most kAttnSplitBlocks
  // (sequence, KV head, query block)s in the launch and a window longer than
  // split_tiles 64-key tiles, a block of more than split_tiles tiles runs as
  // two CTAs over the two halves of its keys; each writes its unnormalised O,
  // m and l to split_part[block][half] (kAttnSplitFloats floats) and takes a
  // ticket from counters[block], and the second merges the two.
  float* split_part;
  uint32_t split_tiles;
};

constexpr uint32_t kAttnSplitBlocks = 148;          // one wave of CTAs
constexpr uint32_t kAttnSplitFloats = 258u * 128u;  // O [256][128 rows], m [128], l [128]

cudaError_t launch_attention(const AttentionArgs& a, cudaStream_t stream, bool pdl);

// The tensor-core form for steps of many rows (attention_tc.cu, tcgen05):
// head dimension 256, 1, 2, 4 or 8 query heads a KV head, every row of a
// sequence at consecutive positions from the step's, a.kv_maps the layer's
// cache tensor maps; configure_attention_tc raises its shared-memory limit
// on the current device (call outside stream capture).
bool attention_prefill_supported(uint32_t heads, uint32_t kv_heads, uint32_t head_dim);
cudaError_t configure_attention_tc();
cudaError_t launch_attention_tc(const AttentionArgs& a, cudaStream_t stream, bool pdl);

// The embedding rows of the step's tokens (or, for a fed step, the last draw)
// times `scale`, into hidden [m][width]; also clears the argmax slots.
struct EmbedArgs {
  const DeviceStep* step;
  Q4Matrix table;
  const uint32_t* ids;             // [m]
  const uint32_t* records;         // [seqs][4], the last step's draws (fed)
  uint32_t seq_tokens;
  uint32_t m;
  float scale;
  float* hidden;
  unsigned long long* argmax;      // [seqs] cleared
  uint32_t seqs;
  // A Q8_0 table instead (codes [n][k], scales [n][k/32] f16; `table` then
  // gives only n and k), or null.
  const uint8_t* q8_codes;
  const uint16_t* q8_scales;
};
cudaError_t launch_embed(const EmbedArgs& a, cudaStream_t stream, bool pdl);

// Q4_1 blocks (20 bytes: d, m, 16 code bytes) as Q4_0 blocks (18 bytes: d
// and the same code bytes) plus a per-block correction c = 8 d + m: since
// code x d + m = (code - 8) x d + (8 d + m), a Q4_1 product is the Q4_0
// product over the same codes and scales plus c times the block's sum of x.
cudaError_t launch_q4_1_split(const uint8_t* q4_1_blocks, size_t blocks, uint8_t* q4_0_blocks, float* corr,
                              cudaStream_t stream);
// y[r][o] += sum over blocks b of corr[o][b] x (the sum of x[r] over block b),
// x [m][k] f32, corr [n][k/32], y [m][n] (the Q4_1 product's correction).
cudaError_t launch_block_correction(const float* x, uint32_t m, uint32_t k, const float* corr, uint32_t n, float* y,
                                    cudaStream_t stream);
// argmax[r] = max over the row's logits of the head's key (largest logit,
// ties to the lower token): `argmax` cleared first.
cudaError_t launch_argmax_rows(const float* logits, uint32_t m, uint32_t v, unsigned long long* argmax,
                               cudaStream_t stream);

// Selection and the draw (topk.wgsl, draw.wgsl) over each sequence's logits.
struct SelectArgs {
  const DeviceStep* step;
  const float* logits;             // [seqs][vocab]
  uint32_t vocab;
  uint32_t seqs;
  const unsigned long long* argmax;  // [seqs], the head's greedy maximum
  const uint32_t* seeds;           // [seqs][2], or null for the step's seed
  unsigned long long* tile_best;   // [seqs][tiles][64] scratch
  uint32_t* candidates;            // [seqs][64][2] (logit bits, token)
  uint32_t* records;               // [seqs][4] {token, failed, u bits, 0}
};
// A layer's view for the capture kernels: its key cache and its slots in a
// sequence's capture store (words from the store's start).
struct CaptureLayer {
  const uint16_t* key_cache;       // [seqs][slots][kv_heads][d]
  uint64_t seq_stride;             // cache elements between sequences
  uint32_t slots;                  // ring slots
  uint32_t keys;                   // min(window, trained context)
  uint64_t residual, query, weights, stats, readout;
};

// The capture's attention weights and statistics (capture/weights.h) for
// every layer of every sequence, at the step's last position; grid (KV
// heads, layers, sequences).
struct WeightsArgs {
  const DeviceStep* step;
  float* store;                    // sequence 0's capture store
  uint64_t store_stride;           // words between sequences' stores
  const CaptureLayer* layers;      // [layers]
  uint32_t heads, kv_heads, head_dim;
  float scale_log2e;
};
cudaError_t launch_attention_weights(const WeightsArgs& a, uint32_t layers, uint32_t seqs, cudaStream_t stream,
                                     bool pdl);

// The per-layer readouts (capture.h:26-33): readout rows are built from the
// captured residuals, run through the final norm and the head by the
// matvec launch, and their top 64 (logit bits, token) pairs are written into
// each layer's readout slot.
struct ReadoutArgs {
  float* store;                    // sequence 0's capture store
  uint64_t store_stride;
  const CaptureLayer* layers;
  uint32_t n_layers;
  uint32_t width;                  // embedding width
  float* rows;                     // [n][width] readout rows
  const float* logits;             // [n][vocab]
  uint32_t vocab;
  unsigned long long* tile_best;   // [n][tiles][64] scratch
};
cudaError_t launch_readout_rows(const ReadoutArgs& a, uint32_t g0, uint32_t n, cudaStream_t stream, bool pdl);
// Rows g0 .. g0 + n - 1 of the layers before the last, or with `last` the
// last layer of sequences g0 .. g0 + n - 1 (logits: their rows).
cudaError_t launch_readout_select(const ReadoutArgs& a, uint32_t g0, uint32_t n, bool last, cudaStream_t stream,
                                  bool pdl);

uint32_t select_tiles(uint32_t vocab);
cudaError_t launch_select(const SelectArgs& a, cudaStream_t stream, bool pdl);

// A step's inputs and outputs moved by kernels instead of copies: the stage
// kernel, the step's first launch, reads the host slot's Step, seeds and
// token ids straight from pinned host memory (mapped into the device's
// address space) into their device copies and clears `zero_words` words;
// the publish kernel, its last, writes the step's records and error word
// into the slot's pinned memory.  (Each small host-device copy on the
// step's stream cost several microseconds between the launches.)
struct StageArgs {
  const DeviceStep* step_h;
  const uint32_t* seeds_h;
  const uint32_t* ids_h;
  DeviceStep* step_d;
  uint32_t* seeds_d;
  uint32_t* ids_d;
  uint32_t seed_words, id_words;
  uint32_t* zero;
  uint32_t zero_words;
};
struct PublishArgs {
  const uint32_t* records_d;
  uint32_t* records_h;
  uint32_t record_words;
  const uint32_t* error_d;
  uint32_t* error_h;
};
cudaError_t launch_stage(const StageArgs& a, cudaStream_t stream);
// One thread waits `ns` nanoseconds by the global timer (bounded): queued
// ahead of a timed launch, it keeps the stream busy while the host submits
// the launch, so that events around the launch bracket the kernel alone.
cudaError_t launch_delay(uint32_t ns, cudaStream_t stream);
cudaError_t launch_publish(const PublishArgs& a, cudaStream_t stream);

}  // namespace fz
