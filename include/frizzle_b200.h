/*
 * frizzle_b200: the Gemma 3 1B Q4_0 forward pass and neuron-steering hook of
 * plainsight-systems/frizzle, as hand-written sm_100a CUDA kernels behind a
 * plain C ABI.  No torch or CUDA types appear in the signatures: device
 * buffers are `void*`/typed pointers, streams are `void*` (a cudaStream_t or
 * NULL for the library's own stream), sizes are explicit.
 *
 * Two levels:
 *   - Engine level: device, model load (GGUF bytes in chunks), sequences
 *     ("batch" of sequences stepped together), steps, readback.  This replaces
 *     the WebGPU Program/Upload/Device layer under Frizzle's C++ engine.
 *   - Kernel level: each hot kernel over caller-owned device buffers, for a
 *     host that drives its own launch list (as kernels::Program does) and for
 *     parity tests.
 *
 * Every call returns an fz_status; on failure fz_last_error() (thread-local)
 * names what was refused and why.  Calls on one fz_device are not
 * thread-safe against each other; distinct devices may be driven from
 * distinct threads.
 */
#ifndef FRIZZLE_B200_H
#define FRIZZLE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors ProgramError (src/core/kernels/program.h:264-278), LoadError
 * (src/core/runtime/engine.h:150-165) and EditError (src/core/edit/edit.h:140-150)
 * folded into one code space. */
typedef enum fz_status {
  FZ_OK = 0,
  FZ_ERR_ARGUMENT = 1,       /* a pointer, size or value outside the contract */
  FZ_ERR_CUDA = 2,           /* a CUDA call failed (ProgramError::Step) */
  FZ_ERR_INDEX = 3,          /* not a GGUF index this engine reads (LoadError::Index) */
  FZ_ERR_ARCHITECTURE = 4,   /* not a Gemma 3 file this engine runs (LoadError::Architecture) */
  FZ_ERR_FIT = 5,            /* does not fit device memory (LoadError::Fit) */
  FZ_ERR_UPLOAD = 6,         /* bytes outside the file, or missing at finish (LoadError::Upload) */
  FZ_ERR_STATE = 7,          /* called in the wrong load/run state (LoadError::Busy/NotLoading) */
  FZ_ERR_EDITS = 8,          /* an edit table that is not well formed (OperationError::Edits) */
  FZ_ERR_TRUNCATED = 9,      /* more index bytes are needed: see fz_model_index_needed */
  FZ_ERR_DEVICE_LOST = 10,   /* the context is unusable (ProgramError::DeviceLost) */
  FZ_ERR_NOT_SUPPORTED = 11  /* a shape this build does not run */
} fz_status;

typedef struct fz_device fz_device;
typedef struct fz_model fz_model;
typedef struct fz_batch fz_batch;

/* The step's parameters: kernels::Step's 64-byte head
 * (src/core/kernels/interface.h:163-185), the token identifiers passed beside
 * it.  `capture` (a padding word in the reference) asks for the per-layer
 * activation capture of each sequence's last row. */
typedef struct fz_step {
  uint32_t position;      /* the first token's position in the context */
  uint32_t tokens;        /* tokens a sequence this step: 1 .. 65536 / sequences (the reference takes
                             1 .. 512, interface.h:165; a fed step is 1) */
  uint32_t logits;        /* 1: the last row's logits, selection and draw */
  uint32_t fed;           /* 1: the one token is each sequence's last draw, read on the device */
  uint32_t seed[2];       /* the draw's seed, low word first */
  uint32_t top_k;
  float temperature;      /* 0: greedy */
  float top_p;
  float min_p;
  float log_min_p;        /* ln min_p (sampler::apply, src/core/sampler/sampler.cpp:51-62) */
  uint32_t capture;
  uint32_t padding[4];
} fz_step;

/* What the draw writes per sequence: SampledRecord (src/core/sampler/sampler.h:187-193). */
typedef struct fz_record {
  uint32_t token;
  uint32_t failed;        /* 1 when the top logit was not finite */
  float u;                /* the uniform the draw used */
  uint32_t padding;
} fz_record;

typedef struct fz_model_info {
  uint32_t layers, hidden, ffn, heads, kv_heads, head_dim, vocab, window, pattern, context;
  float eps, rope_global, rope_local;
  uint64_t weight_bytes;  /* device bytes of the repacked weights */
} fz_model_info;

/* ------------------------------------------------------------------ errors */

/* The message of the calling thread's last failed call. */
const char *fz_last_error(void);

/* ------------------------------------------------------------------ device
 * Replaces gpu::Device (src/core/gpu/device.h:132): a CUDA device and the
 * stream the engine runs on. */
fz_status fz_device_open(int ordinal, fz_device **out);
fz_status fz_device_close(fz_device *device);
/* The device's stream as a cudaStream_t (for hosts that order their own work after it). */
void *fz_device_stream(fz_device *device);

/* ------------------------------------------------------------------ load
 * Replaces Upload::begin/write/finish (src/core/residency/upload.h:263-337)
 * with the describe (src/core/arch/describe.cpp:205-320) and residency plan
 * (src/core/residency/plan.h:319-324) it depends on.
 *
 * begin: `head` holds the file's first `head_bytes` bytes, at least through
 * its tensor infos; FZ_ERR_TRUNCATED asks for fz_model_index_needed() bytes.
 * write: any chunk of the file by its absolute offset, each byte once; bytes
 * outside tensor data are ignored.  finish: repacks every weight on the
 * device into the kernels' layout and frees the staging copy. */
/* Parses and describes a file's index without a device: the checks
 * fz_model_load_begin makes before it allocates (LoadError::Index and
 * ::Architecture), and the shape it would load. */
fz_status fz_model_index_check(const void *head, uint64_t head_bytes, uint64_t file_bytes, fz_model_info *out);
fz_status fz_model_load_begin(fz_device *device, const void *head, uint64_t head_bytes, uint64_t file_bytes,
                              fz_model **out);
uint64_t fz_model_index_needed(void);
fz_status fz_model_load_write(fz_model *model, uint64_t offset, const void *chunk, uint64_t bytes);
fz_status fz_model_load_finish(fz_model *model);
fz_status fz_model_info_get(const fz_model *model, fz_model_info *out);

/* The residency plan for one batch on one GPU (residency::plan_residency and
 * place_cache, src/core/residency/plan.cpp:321-419, restated for a B200's
 * 180 GB and a batch of sequences): the device bytes of the weights (every
 * tensor's bytes and the RoPE turns), of their f16 prefill copies, of the
 * batch's scratch for `rows` token rows a step, and of its key/value rings
 * (per sequence and layer: a window layer window + 512 + rollback slots
 * rounded up to whole 32-slot chunks, a global layer `context` slots; f16
 * keys and values), plus 64 MiB of slack.  In: `sequences` (1 .. 16; 0: the
 * most that fit at `context`), `context` (0: the largest that fits, found by
 * bisection between min(512, trained context) and the trained context, as
 * place_cache finds the context offered, plan.cpp:373-383), `rollback`,
 * `rows` (0: 4096), `budget` (bytes; 0 with a loaded model: the device's free
 * memory now, the model's own bytes counted as already placed).  Out: the
 * sequences and context chosen and the byte counts; FZ_ERR_FIT when even the
 * shortest context does not fit (PlanError::ExceedsBudget). */
typedef struct fz_plan {
  uint32_t sequences, context, rollback, rows;
  uint64_t budget;
  uint64_t weight_bytes, copy_bytes, scratch_bytes, cache_bytes, total_bytes;
} fz_plan;
fz_status fz_model_plan(const fz_model *model, fz_plan *plan);
/* The same from a file's index, without a device (a budget is required). */
fz_status fz_model_index_plan(const void *head, uint64_t head_bytes, uint64_t file_bytes, fz_plan *plan);
fz_status fz_model_free(fz_model *model);

/* ------------------------------------------------------------------ sequences
 * A batch is `sequences` independent sequences stepped together at the same
 * positions, each with its own KV cache (cache/kv.h), edit table and seed.
 * Window layers keep rings of window + 512 + rollback slots
 * (src/core/residency/plan.cpp:335-336); global layers keep `context`. */
fz_status fz_batch_create(fz_model *model, uint32_t sequences, uint32_t context, uint32_t rollback,
                          fz_batch **out);
fz_status fz_batch_free(fz_batch *batch);

/* The run's edits for one sequence, as edit::table lays them out
 * (src/core/edit/edit.h:50-60, edit.cpp:147-170): per layer [first, count],
 * then 5 words an edit {neuron, kind, value bits, first position, end}.
 * NULL/0 clears them.  Checked for shape (offsets inside the table, neurons
 * inside the layer, kinds 0..2); edit::check's semantic checks stay the
 * caller's, as in the reference (engine.cpp:706-708 writes a checked table). */
fz_status fz_batch_set_edits(fz_batch *batch, uint32_t sequence, const uint32_t *words, size_t count);

/* One step over every sequence: replaces Program::run (src/core/kernels/program.h:380-388).
 * `ids` holds sequences x step->tokens identifiers (ignored when fed);
 * `seeds` 2 words a sequence or NULL for step->seed.  Enqueued on the
 * device's stream; fz_batch_wait returns the records. */
fz_status fz_batch_step(fz_batch *batch, const fz_step *step, const uint32_t *ids, const uint32_t *seeds);
fz_status fz_batch_wait(fz_batch *batch, fz_record *records);
/* The oldest step not yet reported: waits for it and returns its records, so
 * that a caller may keep two steps in flight and read each step's records in
 * the order the steps ran (kernels/order.h:50-100, Order::run/next with
 * kOutstanding 2).  A step enqueued while two are unreported overwrites the
 * older one's records.  FZ_ERR_STATE when no step is outstanding;
 * fz_batch_wait reports the last step and with it every earlier one. */
fz_status fz_batch_wait_oldest(fz_batch *batch, fz_record *records);

/* Readback: each sequence's last logits row (vocab floats), and its capture
 * store of the last row of the step that asked for it: fz_capture_floats
 * 32-bit words laid out as capture::layout lays them
 * (src/core/capture/capture.h:217-255, capture.cpp:31-73).  Region 1 is
 * every layer's neurons after edits; region 2, a layer at a time, the
 * residual entering the layer, the attention and feed-forward blocks'
 * additions, the query after rope, the attention weights over the keys the
 * row read (capture/weights.h; zeros past them), the softmax statistics (m
 * then l, log2 units, a head) and the readout: the top 64 (logit bits,
 * token) pairs of the residual the layer leaves through the final norm and
 * head, the last layer's being the step's own logits' (zeros when the step
 * asked for no logits).  Token and logit-bit words are integers stored in
 * the float array. */
fz_status fz_batch_read_logits(fz_batch *batch, uint32_t sequence, float *out, size_t count);
size_t fz_capture_floats(const fz_model *model);
fz_status fz_batch_read_capture(fz_batch *batch, uint32_t sequence, float *out, size_t count);

/* One layer's slots of the capture store (capture::Slot and
 * capture::LayerSlots, src/core/capture/capture.h:188-207): first word and
 * width of each, and the layer's attention.  FZ_ERR_NOT_SUPPORTED for a
 * store past 2^32 words (capture.cpp:37-41 aborts there). */
typedef struct fz_capture_slot {
  uint32_t first;
  uint32_t width;
} fz_capture_slot;
typedef struct fz_capture_slots {
  fz_capture_slot neurons, residual, attention_added, mlp_added, query, weights, stats, readout;
  uint32_t keys;            /* min(attention window, trained context) */
  uint32_t query_heads;
  uint32_t window;          /* attention window, in tokens */
  uint32_t full_attention;  /* 1: the window reaches the trained context */
} fz_capture_slots;
fz_status fz_capture_layout(const fz_model *model, uint32_t layer, fz_capture_slots *out);
/* The KV cache's bookkeeping (cache::KvCache, src/core/cache/kv.h:15-63),
 * shared by the batch's sequences, which step together.  A step advances
 * the cache to position + tokens; its position must be the cache's length
 * or earlier, and an earlier one rewinds the cache first (a rewind that
 * fails, below, empties the cache and refuses the step with
 * FZ_ERR_ARGUMENT).  fz_batch_truncate(tokens) is KvCache::truncate with
 * Runtime::rewind's clamp (runtime.cpp:291-299): it keeps min(tokens,
 * length) tokens when every window layer still holds the window before
 * that position, otherwise it empties the cache; *kept is the new length.
 * fz_batch_cache_state reports the length and the high-water mark. */
fz_status fz_batch_truncate(fz_batch *batch, uint32_t tokens, uint32_t *kept);
fz_status fz_batch_cache_state(fz_batch *batch, uint32_t *length, uint32_t *written);
/* KvCache::truncate's rule, as a pure function of the layers' windows and
 * ring slots, the high-water mark and the tokens kept: 1 when the cache
 * survives the truncation (kv.h:56-63).  Host only; needs no device. */
int fz_cache_truncate_keeps(const uint32_t *windows, const uint32_t *slots, uint32_t layers, uint32_t written,
                            uint32_t tokens);
/* KvCache::advance (src/core/cache/kv.h:64, kv.cpp:52-55): the length grows
 * by `tokens` and the high-water mark follows it, for a caller that wrote
 * the caches' keys and values itself (through fz_batch_cache); refused past
 * the batch's context. */
fz_status fz_batch_cache_advance(fz_batch *batch, uint32_t tokens);
/* Device pointer of sequence s's key or value cache for `layer` ([slots][kv_heads][d] f16). */
fz_status fz_batch_cache(fz_batch *batch, uint32_t sequence, uint32_t layer, int values, void **ptr,
                         uint32_t *slots);
/* Phase timeline of one-token steps (the GPU timestamps of Frizzle's profiled
 * step, one after each launch, src/core/kernels/program.h:142-168; here the
 * step is one launch, so the stamps are taken inside it): when enabled, each decode
 * step records, per CTA of the persistent decode kernel, the GPU global timer
 * (ns) when each phase began waiting, saw its inputs complete, had them
 * staged, had its products and finished. fz_batch_read_trace copies the last
 * step's record: `ctas` x `events` values, event e = (layer * 6 + phase) * 5
 * + k (phase 0 QKV, 1 attention, 2 output projection, 3 gate/up, 4 down,
 * 5 head in the last layer's slots; k 0 began waiting, 1 inputs complete,
 * 2 inputs staged, 3 products done, 4 done), 0 where a CTA had no work;
 * then 11 words: per phase the ns spent waiting for weight tiles, the ns the
 * copy issuer waited for free slots, the ns it spent issuing, its tile count,
 * and the global timer at the CTA's entry and at its exit.
 * With out = NULL it only reports the shape. */
fz_status fz_batch_trace(fz_batch *batch, int enable);
fz_status fz_batch_read_trace(fz_batch *batch, uint64_t *out, size_t count, uint32_t *ctas, uint32_t *events);

/* Times the persistent decode kernel of each following one-token step with
 * CUDA events recorded around its launch on the step's stream (Frizzle's
 * profiled step times its launches, src/core/kernels/program.h:142-168);
 * timed steps are launched directly rather than from the step's graph, so
 * the events bracket the kernel alone.  fz_batch_decode_time gives the last
 * such step's kernel duration once the step has run. */
fz_status fz_batch_time_decode(fz_batch *batch, int enable);
fz_status fz_batch_decode_time(fz_batch *batch, float *microseconds);

/* Every wait inside a one-token step (a phase waiting for another's output,
 * a weight tile, a key/value chunk) is bounded; when one gives up, the step
 * is abandoned by every CTA and fz_batch_wait reports FZ_ERR_CUDA naming the
 * wait, and the next step runs normally (the device-lost and step-failure
 * reports of src/core/kernels/program.cpp:621-625 and
 * src/core/runtime/turn.h:108-113, and the reference tests' bounded pump,
 * tests/support/gpu.h:41-54).  This sets the limit for the batch's
 * following steps, in microseconds (100 .. 10,000,000; 0 restores the
 * default of 2 s). */
fz_status fz_batch_set_wait_limit(fz_batch *batch, uint32_t microseconds);

/* Test hook, no counterpart in the reference: while enabled, each one-token
 * step publishes its QKV products under the previous step's epoch, so the
 * attention's bounded wait for them runs out and the step reports the
 * failure as above.  Nothing faults; the batch's cache then holds the
 * tokens before the failed step's position only after fz_batch_truncate. */
fz_status fz_batch_inject_stale_epoch(fz_batch *batch, int enable);

/* ------------------------------------------------------------------ kernel level
 * Device pointers throughout; `stream` is a cudaStream_t or NULL (the legacy
 * default stream). */

/* Bytes of the fragment-native layout of an n x k Q4_0 matrix (n % 16 == 0, k % 64 == 0). */
size_t fz_q4_0_codes_bytes(uint32_t n, uint32_t k);
size_t fz_q4_0_scales_bytes(uint32_t n, uint32_t k);

/* GGUF Q4_0 blocks (18 bytes each, row-major) into the layout
 * (PieceWriter's transpose, src/core/residency/piece_writer.h:165-245). */
fz_status fz_q4_0_repack(const void *file_blocks, uint32_t n, uint32_t k, void *codes, void *scales,
                         void *stream);

/* Rows of a repacked matrix back to f32, times `scale` (the gather,
 * src/core/kernels/gather/gather.wgsl:25-48). */
fz_status fz_q4_0_rows(const void *codes, const void *scales, uint32_t n, uint32_t k, const uint32_t *rows,
                       uint32_t count, float scale, float *out, void *stream);

/* y[m][n] = sum_k W[n][k] x[m][k], m <= 16 (matmul_launches with the Write
 * epilogue, src/core/kernels/matmul/matmul.cpp:258-312). */
fz_status fz_q4_0_matvec(const void *codes, const void *scales, uint32_t n, uint32_t k, const float *x,
                         uint32_t m, float *y, void *stream);

/* act[m][f] = gelu_tanh(gate . x) * (up . x), then the edit table applied to
 * rows at positions position + r (the GatedActivation epilogue,
 * matmul.wgsl:247-270, and the edit launch, src/core/edit/edit.wgsl:55-76);
 * `table` may be NULL. */
fz_status fz_q4_0_gated(const void *gate_codes, const void *gate_scales, const void *up_codes,
                        const void *up_scales, uint32_t f, uint32_t k, const float *x, uint32_t m,
                        const uint32_t *table, uint32_t layer, uint32_t position, float *act, void *stream);

/* The head: logits[m][n] and, per row, the greedy choice (largest logit,
 * ties to the lower id; topk.wgsl:32-61) packed as (key << 32) | ~id into
 * argmax[m] (max-reduced: clear it first). */
fz_status fz_q4_0_head(const void *codes, const void *scales, uint32_t n, uint32_t k, const float *x,
                       uint32_t m, float *logits, unsigned long long *argmax, void *stream);

/* Q8_0 (the pinned file's token embedding and tied head) and Q4_1 (its
 * ffn_down in layers 0-2): src/core/formats/q8_0/q8_0.h, q4_1/q4_1.h.  The
 * device layout is the reference's piece layout over the whole matrix
 * (src/core/formats/device_layout.h:115-121): every block's code bytes, row
 * after row (32 a block for Q8_0, 16 for Q4_1), then every block's scale word
 * (Q8_0: d; Q4_1: d then m).  n >= 1, k a multiple of 32; codes and x 16-byte
 * aligned. */
size_t fz_q8_0_codes_bytes(uint32_t n, uint32_t k);
size_t fz_q8_0_scales_bytes(uint32_t n, uint32_t k);
size_t fz_q4_1_codes_bytes(uint32_t n, uint32_t k);
size_t fz_q4_1_scales_bytes(uint32_t n, uint32_t k);

/* GGUF blocks (34 or 20 bytes, row-major; 2- or 4-byte aligned) into the
 * layout (PieceWriter's transpose, src/core/residency/piece_writer.h:165-245). */
fz_status fz_q8_0_repack(const void *file_blocks, uint32_t n, uint32_t k, void *codes, void *scales,
                         void *stream);
fz_status fz_q4_1_repack(const void *file_blocks, uint32_t n, uint32_t k, void *codes, void *scales,
                         void *stream);

/* Rows back to f32 times `scale`, bit-exact (the gather,
 * src/core/kernels/gather/gather.wgsl:25-48, over q8_0.wgsl:11-23 and
 * q4_1.wgsl:12-26). */
fz_status fz_q8_0_rows(const void *codes, const void *scales, uint32_t n, uint32_t k, const uint32_t *rows,
                       uint32_t count, float scale, float *out, void *stream);
fz_status fz_q4_1_rows(const void *codes, const void *scales, uint32_t n, uint32_t k, const uint32_t *rows,
                       uint32_t count, float scale, float *out, void *stream);

/* y[m][n] = sum_k W[n][k] x[m][k], 1 <= m <= 8, x staged in shared memory as
 * 8-bit digit planes at 3.125 bytes a value (3.25 for Q4_1), at most 200 KiB
 * (m = 8 at k = 6912 fits); a non-finite x gives NaN sums for its row (matmul_launches with the Write epilogue,
 * src/core/kernels/matmul/matmul.cpp:258-312). */
fz_status fz_q8_0_matvec(const void *codes, const void *scales, uint32_t n, uint32_t k, const float *x,
                         uint32_t m, float *y, void *stream);
fz_status fz_q4_1_matvec(const void *codes, const void *scales, uint32_t n, uint32_t k, const float *x,
                         uint32_t m, float *y, void *stream);

/* Y[m][n] = sum_k W[n][k] X[m][k] for many rows on the tensor cores
 * (tcgen05.mma into tensor memory; the reference's prefill form,
 * src/core/kernels/matmul/matmul.wgsl:287-485): X as f16 `x_hi` [m][k] and
 * optionally its f16 remainder `x_lo` (NULL: one pass).  Weights are rounded
 * once to f16 as they are dequantized, unless `exact_weights` (with x_lo):
 * then they too are f16 hi + lo and the product is f32-level (three MMAs a
 * k-slice; two with x_lo alone, one without).  `error` is a device word the
 * caller zeroes; nonzero after the call completes means a bounded wait inside
 * the kernel gave up (no result). */
fz_status fz_q4_0_gemm(const void *codes, const void *scales, uint32_t n, uint32_t k, const void *x_hi,
                       const void *x_lo, uint32_t exact_weights, uint32_t m, float *y, uint32_t *error,
                       void *stream);

/* The gated product for many rows: act = gelu_tanh(gate . x) * (up . x), the
 * edit table applied to rows at positions position + r, written as f32 `act`
 * (may be NULL) and as f16 hi/lo (`act_lo` may be NULL) for the next product. */
fz_status fz_q4_0_gemm_gated(const void *gate_codes, const void *gate_scales, const void *up_codes,
                             const void *up_scales, uint32_t f, uint32_t k, const void *x_hi, const void *x_lo,
                             uint32_t exact_weights, uint32_t m, const uint32_t *table, uint32_t layer,
                             uint32_t position, float *act, void *act_hi, void *act_lo, uint32_t *error,
                             void *stream);

/* The Q4_0 matrix (repacked codes and scales, n x k) as f16 [n][k]: w_hi =
 * f16((code - 8) d), w_lo = the f16 remainder of that exact product (may be
 * NULL).  The engine makes these once at load for its prefill products. */
fz_status fz_q4_0_to_f16(const void *codes, const void *scales, uint32_t n, uint32_t k, void *w_hi, void *w_lo,
                         void *stream);

/* fz_q4_0_gemm and fz_q4_0_gemm_gated with the weights as f16 copies
 * (fz_q4_0_to_f16; `*_lo` needed with exact_weights): the weight tiles come
 * by TMA like X's and no CTA dequantizes. */
fz_status fz_f16_gemm(const void *w_hi, const void *w_lo, uint32_t n, uint32_t k, const void *x_hi,
                      const void *x_lo, uint32_t exact_weights, uint32_t m, float *y, uint32_t *error, void *stream);
fz_status fz_f16_gemm_gated(const void *gate_hi, const void *gate_lo, const void *up_hi, const void *up_lo,
                            uint32_t f, uint32_t k, const void *x_hi, const void *x_lo, uint32_t exact_weights,
                            uint32_t m, const uint32_t *table, uint32_t layer, uint32_t position, float *act,
                            void *act_hi, void *act_lo, uint32_t *error, void *stream);

/* x -> f16 hi = f16(x) and lo = f16(x - hi) (`lo` may be NULL). */
fz_status fz_split_f16(const float *x, size_t n, void *hi, void *lo, void *stream);

/* Attention of `rows` consecutive query rows (positions position .. position +
 * rows - 1, one sequence) over a KV cache: softmax(q . k / sqrt(d)) . v over
 * keys in [p - window + 1, p], keys read from slot j mod slots (the attention
 * launch and its combine, src/core/kernels/attention/attention.cpp:36-102).
 * q, out: [rows][heads][256] f32; key_cache, value_cache: [slots][kv_heads][256]
 * f16.  Keys split into CTAs of 512; rows whose keys span several splits leave
 * partials in caller scratch: partial_o rows x heads x splits x 256 floats,
 * partial_ml rows x heads x splits x 2 floats, counters rows x kv_heads words
 * that start at zero (the kernel leaves them zero), with
 * splits = ceil(min(window, position + rows) / 512).  heads / kv_heads must
 * be 1, 2, 4 or 8 (FZ_ERR_ARGUMENT otherwise). */
fz_status fz_attention(const float *q, const void *key_cache, const void *value_cache, uint32_t slots,
                       uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t window, uint32_t position,
                       uint32_t rows, float *partial_o, float *partial_ml, uint32_t *counters, float *out,
                       void *stream);
uint32_t fz_attention_splits(uint32_t window, uint32_t position, uint32_t rows);

/* fz_attention for steps of many rows, on the tensor cores (the engine's
 * attention for steps of more than 16 rows; the same sums as attention.wgsl:
 * 166-438): tiles of 64 keys by TMA, S = Q K^T and O += P V by tcgen05 with Q
 * and P as f16 part and remainder, the online softmax a thread a row.  The
 * rows are one sequence at positions position .. position + rows - 1; q, out
 * and the caches as in fz_attention, the caches 16-byte aligned and slots a
 * multiple of 32.  maps: 256
 * bytes of device memory, 64-byte aligned, where the call writes the caches'
 * tensor maps (stream-ordered).  split_part: null, or
 * FZ_ATTENTION_WIDE_SPLIT_FLOATS floats of scratch with counters (148 words
 * that start at zero; the kernel leaves them zero): then, when the launch's
 * blocks of 128 / (heads / kv_heads) rows fit one wave of 148 CTAs and the
 * window is longer than 1280 keys, a block of more than 1280 keys runs as
 * two CTAs over the halves of its keys, merged by the second to finish.
 * error: null or a device word set nonzero when a bounded wait gave up. */
#define FZ_ATTENTION_WIDE_SPLIT_FLOATS (148u * 2u * 258u * 128u)
fz_status fz_attention_wide(const float *q, const void *key_cache, const void *value_cache, uint32_t slots,
                            uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t window,
                            uint32_t position, uint32_t rows, void *maps, float *split_part, uint32_t *counters,
                            float *out, uint32_t *error, void *stream);

/* fz_attention for callers that cannot allocate device memory: no
 * counterpart in the reference.  Some hosts own no device allocator (a
 * runtime that hands out only pre-registered buffers, a memory pool fixed
 * before plugins load, a caller recording work that must stay free of
 * allocation), so this entry point takes only inputs and outputs and keeps
 * the split scratch in a static device array the library holds on every
 * device that loads it, until the process exits: 2 MiB + 16 KiB + 512 B.
 * Limits: rows x heads x key splits <= FZ_ATTENTION_STATIC_MAX_PARTIALS and
 * rows x kv_heads <= FZ_ATTENTION_STATIC_MAX_COUNTERS; larger calls are
 * refused with FZ_ERR_ARGUMENT, as are heads per KV head other than 1, 2, 4
 * or 8.  It calls no cudaMalloc or cudaFree: the first call in a CUDA
 * context looks up the array's device address in that context
 * (cudaGetSymbolAddress) and keeps it under the context's ID, so make that
 * first call before any stream capture, and again first after
 * cudaDeviceReset or when a different context is made current.  Every call
 * shares the one array and clears its split counters before the launch;
 * calls whose launches overlap on the GPU race on the scratch. */
#define FZ_ATTENTION_STATIC_MAX_PARTIALS 2048u
#define FZ_ATTENTION_STATIC_MAX_COUNTERS 128u
fz_status fz_attention_static(const float *q, const void *key_cache, const void *value_cache, uint32_t slots,
                              uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t window,
                              uint32_t position, uint32_t rows, float *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* FRIZZLE_B200_H */
