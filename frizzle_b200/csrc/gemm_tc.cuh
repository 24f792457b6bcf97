// Prefill products on the 5th-generation tensor cores: Y[m][n] = sum_k W[n][k] X[m][k]
// for many rows of X (prefill blocks, wide batches), W in the fragment-native
// Q4_0 layout (q4_matvec.cuh), X as f16 (optionally f16 hi + lo of an f32).
#pragma once

#include <cuda_fp16.h>

#include "fz_common.cuh"
#include "q4_matvec.cuh"

namespace fz {

enum GemmEpilogue : int { kGemmWrite = 0, kGemmGated = 1 };

struct GemmArgs {
  const DeviceStep* step;     // position of row 0, or null for `position`
  uint32_t position;
  Q4Matrix w[2];              // w[1]: the up projection of a gated product
  // Optional f16 copies of w[0], w[1] ([n][k], the weights as f16 hi and
  // remainder lo, from dequant_f16): when w_hi[0] is set the tiles arrive by
  // TMA and no CTA dequantizes (w_lo with exact_w).
  const __half* w_hi[2];
  const __half* w_lo[2];
  uint32_t m;                 // rows of X
  const __half* x_hi;         // [m][k] f16
  const __half* x_lo;         // [m][k] f16 remainder, or null (one pass)
  uint32_t exact_w;           // with x_lo: weights as f16 hi + lo too (three MMAs, f32-level)
  float* out;                 // [m][out_stride] f32 (Write; Gated: optional)
  uint32_t out_stride;
  // Gated epilogue: act = gelu(gate) * up, edits, then f16 hi/lo for the next product.
  __half* act_hi;             // [m][f]
  __half* act_lo;             // [m][f] or null
  const uint32_t* edit_table; // or null
  uint64_t table_stride;
  uint32_t layer;
  uint32_t seq_tokens;        // rows a sequence holds
  float* capture_neurons;     // sequence 0's capture slot, or null
  uint64_t capture_stride;
  uint32_t* error;            // set nonzero when a bounded wait gives up
  // K split (set by launch_gemm for a Write product of few tiles): each
  // (tile, K slice) is a work item whose partial is added into `out` with
  // f32 reductions (out zeroed first by launch_gemm), so the slices' sums
  // meet in no fixed order.  1 = none.
  uint32_t k_split;
};

// Launches the product: X_hi.W (x_lo null), X_hi.W + X_lo.W (x_lo), or with
// exact_w also X_hi.W_lo (three MMAs a k-slice); W rounded once to f16
// unless exact_w.
cudaError_t launch_gemm(const GemmArgs& a, int epilogue, cudaStream_t stream, bool pdl);

// The Q4_0 matrix as f16 [n][k]: hi = f16((code - 8) d), lo = the f16
// remainder of the exact product (lo may be null).
cudaError_t launch_dequant_f16(const Q4Matrix& w, __half* hi, __half* lo, cudaStream_t stream,
                               const float* corr = nullptr);

// x -> f16 hi = f16(x), lo = f16(x - hi) (lo may be null).
cudaError_t launch_split_f16(const float* x, size_t n, __half* hi, __half* lo, cudaStream_t stream);

}  // namespace fz
