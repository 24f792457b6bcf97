// Q4_0 weights in the fragment-native device layout, and the skinny product
// Y[m][n] = sum_k W[n][k] X[m][k] over them for up to 16 rows of X.
//
// Device layout (written once at load by q4_repack_kernel).  A matrix of N
// rows by K columns (N % 16 == 0, K % 64 == 0) is cut into row groups of 16
// rows and block pairs of 64 columns (two Q4_0 blocks).  For row group rg and
// block pair bp, 512 code bytes hold, for lane L = 4g + t of a warp, four
// 32-bit words: (block 2bp, half 0), (2bp, half 1), (2bp+1, half 0),
// (2bp+1, half 1), where the word of (block kb, half h) is the code bytes
//   [row g byte 8h+2t, row g+8 byte 8h+2t, row g byte 8h+2t+1, row g+8 byte 8h+2t+1]
// of block kb's 16 code bytes.  Those are exactly the eight nibbles lane L
// holds as the A fragment of one mma.m16n8k16 (rows g and g+8, and, in a
// fixed permutation of the block's columns, columns 2t, 2t+1, 2t+8, 2t+9),
// so one 128-bit load gives a lane its A fragments for two blocks.  The
// scales of the pair follow in their own stream, 64 bytes per (rg, bp): for
// g = 0..7 the halves d(g, 2bp), d(g+8, 2bp), d(g, 2bp+1), d(g+8, 2bp+1).
// Codes take N*K/2 bytes and scales N*K/16: the file's 0.5625 bytes a weight,
// no more.  The codes stay the file's bits (formats/device_layout.h: a
// transform done once at upload that moves no bits within a field).
#pragma once

#include "fz_common.cuh"

namespace fz {

constexpr int kMaxTokens = 16;   // rows of X one skinny launch takes

struct Q4Matrix {
  const uint4* codes;
  const uint2* scales;
  uint32_t n, k;
};

inline size_t q4_codes_bytes(uint32_t n, uint32_t k) { return (size_t)n * k / 2; }
inline size_t q4_scales_bytes(uint32_t n, uint32_t k) { return (size_t)n * k / 16; }

enum Prologue : int { kPrologueInput = 0, kPrologueNorm = 1 };
enum Epilogue : int { kEpilogueWrite = 0, kEpilogueQkv = 1, kEpilogueGated = 2, kEpilogueHead = 3 };

// What a launch's norm prologue reads and writes (norm.wgsl:97-198 fused into
// the product that consumes `normed`).
struct NormArgs {
  const float* hidden_in;   // X rows, [m][width]
  const float* y;           // the block output added in, or null
  const float* post_gain;   // its post-norm gain, or null
  const float* gain;        // the norm's gain
  float* hidden_out;        // X after the add, written by CTA 0 (may be null)
  float eps;
  uint32_t width;
  uint32_t row_of_token_stride;  // rows of hidden per token slot: 1, or T for "last row of each sequence"
  uint32_t row_of_token_offset;  // added to the row index
  float* capture_residual;  // [m][width] X after the add, or null
  float* capture_added;     // [m][width] y as added, or null
  uint32_t y_parts;         // y is the sum of this many K-slice partials (0 or 1: y itself)
  uint64_t y_part_stride;   // floats between the partials
};

struct RopeArgs {
  const float* q_gain;      // QK-norm gains, [d]
  const float* k_gain;
  const float* turns;       // theta_k / 2 pi, [d/2]
  float eps;
  uint32_t heads, kv_heads, head_dim;
  uint16_t* key_cache;      // [sequences][slots][kv_heads][d]
  uint16_t* value_cache;
  uint32_t slots;
  uint64_t seq_stride;      // elements between sequences' caches
  float* query_out;         // [m][heads*d], after rope
  float* capture_query;     // [m][heads*d] or null
};

struct EditArgs {
  const uint32_t* table;    // the reference's edit table (edit/edit.h:50-60), or null
  uint64_t table_stride;    // words between sequences' tables
  uint32_t layer;
  float* capture_neurons;   // sequence 0's slot, or null
};

struct HeadArgs {
  unsigned long long* argmax;  // [m] packed (key << 32) | ~row, max-reduced
};

struct MatvecArgs {
  const DeviceStep* step;   // the position the rows start at, or null for `position`
  uint32_t position;
  Q4Matrix mat[2];          // mat[1]: the up projection of a gated product
  uint32_t m;               // rows of X
  uint32_t seq_tokens;      // rows a sequence holds in X (sequence of row i = i / seq_tokens)
  uint64_t capture_stride;  // floats between sequences' capture stores
  const float* x;           // [m][k] for the input prologue
  NormArgs norm;
  float* out;               // [m][out_stride]
  uint32_t out_stride;
  RopeArgs rope;
  EditArgs edit;
  HeadArgs head;
  uint32_t* counter;        // last-CTA counter (QKV epilogue), zero between launches
  uint32_t rg_per_cta;      // row groups a CTA (gated: 1 pair)
  uint32_t k_split;         // warps splitting K inside a CTA
  uint32_t cluster;         // CTAs splitting K across a cluster
};

// Host-side launch (q4_matvec.cu).  configure_kernels() raises every
// instantiation's dynamic shared memory limit on the current device; call it
// once per device before the first launch (and before any graph capture).
cudaError_t configure_kernels();
cudaError_t launch_matvec(const MatvecArgs& a, int prologue, int epilogue, cudaStream_t stream, bool pdl);
// Wide steps (more rows than the skinny product takes): the norm per row into
// f16 hi/lo, and QK-norm/RoPE/KV append per (row, head) over a.out's raw QKV.
cudaError_t launch_norm_f16(const MatvecArgs& a, __half* out_hi, __half* out_lo, cudaStream_t stream, bool pdl);
cudaError_t launch_rope_rows(const MatvecArgs& a, cudaStream_t stream, bool pdl);
// The norm prologue's rows as f32 [m][width] (CTA i the row the prologue
// reads for slot i), with no product after it.
cudaError_t launch_norm_f32(const MatvecArgs& a, float* out, cudaStream_t stream, bool pdl);
cudaError_t launch_repack(const uint8_t* file_blocks, uint32_t n, uint32_t k, uint4* codes, uint2* scales,
                          cudaStream_t stream);
cudaError_t launch_dequant_rows(const Q4Matrix& mat, const uint32_t* rows, uint32_t count, float scale,
                                float* out, cudaStream_t stream);

}  // namespace fz
