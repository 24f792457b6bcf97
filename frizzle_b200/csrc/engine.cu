// The engine behind the C ABI (include/frizzle_b200.h): device, load with
// on-device repack, batches of sequences with their KV rings, and the step's
// launch chain (embed, 26 x [QKV+RoPE, attention, O, gate/up+GELU+edits,
// down], head+argmax, selection+draw) captured once per step shape into a
// CUDA graph whose kernels read the position from device memory.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "frizzle_b200.h"
#include "decode_step.cuh"
#include "gemm_tc.cuh"
#include "gguf_index.h"
#include "kernels.cuh"
#include "last_error.h"
#include "q4_matvec.cuh"

using fz::DeviceStep;
using fz::GgufIndex;
using fz::Q4Matrix;

namespace {

thread_local std::string g_error;
thread_local uint64_t g_index_needed = 0;

fz_status fail(fz_status s, const std::string& msg) {
  g_error = msg;
  return s;
}

}  // namespace

void fz::set_last_error(const char* message) { g_error = message; }

namespace {

#define FZ_CUDA(x)                                                                           \
  do {                                                                                       \
    cudaError_t e_ = (x);                                                                    \
    if (e_ != cudaSuccess) return fail(FZ_ERR_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

constexpr uint32_t kMaxEdits = 4096;  // edit::kMaxEdits
constexpr uint32_t kSplitKeys = 512;  // most keys a per-op attention CTA takes (its score buffer)

// Keys a per-op attention CTA takes for a layer reading up to `keys` keys:
// 64-key splits while that gives at most 64 of them (a 512-key window is 8
// CTAs a row and KV head, not one), longer splits, in 64s, beyond.
uint32_t split_keys_for(uint32_t keys) {
  const uint32_t per = (keys + 63) / 64;                     // splits of 64 keys
  const uint32_t split = std::max<uint32_t>(64, (per + 63) / 64 * 64);
  return std::min(split, kSplitKeys);
}

}  // namespace

struct fz_device {
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t capture = nullptr;
};

namespace {

struct DevMatrix {
  uint4* codes = nullptr;
  uint2* scales = nullptr;
  uint32_t n = 0, k = 0;
  // The layer products' f16 copies for the tensor-core prefill ([n][k]: f16
  // of (code - 8) d and the remainder), so that its tiles come by TMA.
  __half *f16_hi = nullptr, *f16_lo = nullptr;
  Q4Matrix view() const { return Q4Matrix{codes, scales, n, k}; }
};

// GGML type ids of the formats the model reads.
constexpr uint32_t kTypeF32 = 0, kTypeQ4_0 = 2, kTypeQ4_1 = 3, kTypeQ8_0 = 8;

struct Layer {
  DevMatrix qkv, o, gate, up, down;
  // A Q4_1 down projection (the pinned file's layers 0-2) is held as its
  // Q4_0 part in `down` and the per-block correction 8 d + m [hidden][ffn/32].
  uint32_t down_type = kTypeQ4_0;
  float* down_corr = nullptr;
  float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *post_attn_norm = nullptr,
        *ffn_norm = nullptr, *post_ffw_norm = nullptr;
  float* turns = nullptr;
  bool global = false;
  uint32_t window = 0;
  float rope_base = 0.f;
};

struct Shape {
  uint32_t layers = 0, hidden = 0, ffn = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0, window = 0,
           pattern = 6, context = 0;
  float eps = 0.f, rope_global = 0.f, rope_local = 0.f;
};

// The capture store's layout in 32-bit words (capture::layout,
// src/core/capture/capture.cpp:31-73): region 1 holds every layer's neurons
// (its feed-forward width) in layer order; region 2, for each layer in turn,
// its residual, attention addition and feed-forward addition (the width
// each), its query (heads x head dimension), its attention weights (heads x
// keys, keys = min(window, trained context)), its softmax statistics (m then
// l a head) and its readout (64 pairs of logit bits and token).
struct CaptureSlot {
  uint64_t neurons, residual, attn_added, mlp_added, query, weights, stats, readout;
  uint32_t keys, window;
};
constexpr uint32_t kReadoutWords = 128;  // capture::kReadoutWords: 2 x kCandidates
struct CaptureLayout {
  std::vector<CaptureSlot> layer;
  uint64_t words = 0;  // the store, one sequence's
};
CaptureLayout capture_layout(const Shape& s) {
  CaptureLayout c;
  c.layer.resize(s.layers);
  uint64_t at = 0;
  const auto take = [&at](uint64_t width) {
    const uint64_t first = at;
    at += width;
    return first;
  };
  for (uint32_t l = 0; l < s.layers; l++) c.layer[l].neurons = take(s.ffn);
  for (uint32_t l = 0; l < s.layers; l++) {
    CaptureSlot& k = c.layer[l];
    k.window = s.window == 0 || l % s.pattern == s.pattern - 1 ? s.context : s.window;
    k.keys = std::min(k.window, s.context);
    k.residual = take(s.hidden);
    k.attn_added = take(s.hidden);
    k.mlp_added = take(s.hidden);
    k.query = take((uint64_t)s.heads * s.head_dim);
    k.weights = take((uint64_t)s.heads * k.keys);
    k.stats = take(2ull * s.heads);
    k.readout = take(kReadoutWords);
  }
  c.words = at;
  return c;
}

// The kernels write the residual, additions and query slots, and read the
// residuals back, four words at a time: each slot, and each sequence's store,
// starts on a 16-byte boundary (true whenever the head count is even).
bool capture_aligned(const CaptureLayout& c) {
  if (c.words % 4) return false;
  for (const CaptureSlot& k : c.layer)
    if ((k.neurons | k.residual | k.attn_added | k.mlp_added | k.query) % 4) return false;
  return true;
}

}  // namespace

struct fz_model {
  fz_device* dev = nullptr;
  GgufIndex index;
  Shape shape;
  uint64_t file_bytes = 0;
  // The streaming load (PieceWriter, src/core/residency/piece_writer.h:165-245):
  // each tensor the engine reads is a sink, in file order; chunks arrive in
  // order, a Q4_0 matrix's bytes pass through a bounded device stage and are
  // repacked a 16-row group at a time as soon as a group is whole, an f32
  // vector's bytes go straight to its buffer.
  struct Sink {
    uint64_t begin = 0, end = 0;   // the tensor's bytes in the file (absolute offsets)
    DevMatrix* mat = nullptr;      // a Q4_0 matrix ...
    uint32_t row0 = 0, k = 0;      //   ... its first row in `mat`, its row length
    uint32_t type = kTypeQ4_0;     //   ... the file's format (Q4_1: split into Q4_0 and `corr`)
    float* corr = nullptr;         //   ... a Q4_1 matrix's corrections [rows][k/32]
    uint8_t* q8_codes = nullptr;   // or a Q8_0 table, repacked a row at a time
    uint16_t* q8_scales = nullptr;
    float* gain = nullptr;         // or an f32 vector
    int group = -1;                // the layer product whose f16 copies it completes, or -1
    std::string name;
  };
  std::vector<Sink> sinks;
  size_t next_sink = 0;            // the sink the cursor is in (or before)
  uint64_t cursor = 0;             // the next file offset the load expects
  uint32_t rows_done = 0;          // rows of the current matrix sink repacked
  uint8_t* stage = nullptr;        // bounded device staging of a matrix's partial row groups
  uint64_t stage_fill = 0;
  uint8_t* stage_q4_0 = nullptr;   // a Q4_1 stage's row groups as Q4_0 blocks (Q4_1 files only)
  std::vector<DevMatrix*> groups;  // the layer products (f16 copies made once complete)
  std::vector<uint32_t> group_left;
  std::vector<Layer> layers;
  DevMatrix embd;                  // the tied embedding and head (n, k; codes when Q4_0)
  uint32_t embd_type = kTypeQ4_0;
  uint8_t* embd_q8 = nullptr;      // a Q8_0 table: codes [vocab][hidden], scales [vocab][hidden/32]
  uint16_t* embd_q8_scales = nullptr;
  float* output_norm = nullptr;
  bool finished = false;
  uint64_t weight_bytes = 0;
  std::vector<void*> allocations;

  ~fz_model() {
    for (void* p : allocations) cudaFree(p);
    if (stage) cudaFree(stage);
    if (stage_q4_0) cudaFree(stage_q4_0);
  }
  template <typename T>
  fz_status alloc(T** p, size_t bytes) {
    void* v = nullptr;
    cudaError_t e = cudaMalloc(&v, bytes ? bytes : 16);
    if (e != cudaSuccess) return fail(FZ_ERR_FIT, "device allocation of " + std::to_string(bytes) + " bytes: " +
                                                     cudaGetErrorString(e));
    allocations.push_back(v);
    *p = static_cast<T*>(v);
    weight_bytes += bytes;
    return FZ_OK;
  }
};

namespace {

// A step graph's shape; `slot` names the host slot its first and last
// launches read from and write to (two steps may be in flight).
struct GraphKey {
  uint32_t tokens, logits, capture, edits, timed, slot;
  bool operator<(const GraphKey& o) const {
    return std::tie(tokens, logits, capture, edits, timed, slot) <
           std::tie(o.tokens, o.logits, o.capture, o.edits, o.timed, o.slot);
  }
};

}  // namespace

struct fz_batch {
  fz_model* model = nullptr;
  uint32_t S = 0, context = 0, rollback = 0;
  std::vector<uint16_t*> kc, vc;
  std::vector<uint32_t> slots;
  std::vector<uint64_t> seq_stride;
  float *hidden_a = nullptr, *hidden_b = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr,
        *y_attn = nullptr, *y_mlp = nullptr, *act = nullptr, *logits = nullptr;
  float *partial_o = nullptr, *partial_ml = nullptr;
  float* attn_split = nullptr;   // the tensor-core attention's split halves (kAttnSplitBlocks x 2)
  uint32_t* counters = nullptr;   // per layer: 1 QKV + M*kv attention counters
  uint32_t counters_per_layer = 0;
  uint32_t splits_max = 0;
  unsigned long long* argmax = nullptr;
  unsigned long long* tile_best = nullptr;
  uint32_t *records = nullptr, *candidates = nullptr;
  DeviceStep* dstep = nullptr;
  uint32_t *dids = nullptr, *dseeds = nullptr;
  uint32_t* edit_tables = nullptr;
  uint32_t table_words = 0;
  std::vector<bool> has_edits;
  float* captures = nullptr;
  uint64_t capture_floats = 0;
  // The capture kernels' per-layer view and the readouts' scratch (up to
  // kMaxTokens readout rows a head launch).
  fz::CaptureLayer* cap_layers = nullptr;
  float *ro_rows = nullptr, *ro_logits = nullptr;
  float* head_x = nullptr;         // a Q8_0 head's normed rows [head_rows][hidden]
  uint32_t head_rows = 0;
  unsigned long long *ro_argmax = nullptr, *ro_tile_best = nullptr;
  // Rows the per-row scratch holds (sequences x tokens of the widest step so
  // far); grown on demand, which drops the captured graphs.
  uint32_t rows_cap = 0;
  __half *x16_hi = nullptr, *x16_lo = nullptr, *act16_hi = nullptr, *act16_lo = nullptr;
  uint32_t* gemm_error = nullptr;  // set by a device wait (tensor-core product, decode step) that gave up
  // The persistent decode step: its per-layer view, K-slice partials, phase counters.
  fz::DecodeLayer* dlayers = nullptr;
  fz::DecodeKvMaps* kv_maps = nullptr;   // the decode kernel's key/value tensor maps
  float* y_parts = nullptr;        // [O slices + down slices][rows][hidden]
  uint32_t* dsync = nullptr;
  size_t dsync_words = 0;
  unsigned long long* trace = nullptr;  // phase timeline, when enabled
  uint32_t trace_ctas = 0, trace_events = 0;
  // Tensor-core products: 1 = X and W each rounded once to f16; 2 = X as f16
  // hi + lo, W rounded once (two MMAs a k-slice); 3 = W as hi + lo too
  // (three MMAs, f32-level).  The model runs 3: with one f16 rounding of X or
  // of W alone, config 1's logits land at 1.1-1.3e-3 relative RMS from the
  // fp32 oracle, above the 1e-3 parity bar.
  uint32_t passes = 3;
  std::vector<void*> row_allocs;
  // Host staging, two slots (at most two steps in flight, kernels/order.h:70).
  struct Slot {
    DeviceStep* step = nullptr;
    uint32_t* ids = nullptr;
    uint32_t* seeds = nullptr;
    uint32_t* records = nullptr;
    uint32_t* error = nullptr;     // the tensor-core products' error word, read back
    cudaEvent_t copied = nullptr;  // the H2D copy of this slot has run
    cudaEvent_t done = nullptr;    // the step's records are home
    bool used = false;
    bool pending = false;          // its records not reported yet
  } slot[2];
  int next_slot = 0;
  int last_slot = -1;
  uint32_t serial = 1;             // steps run (the decode kernel's epochs)
  uint32_t wait_us = 0;            // the decode step's wait limit (0: the kernel's default)
  bool time_decode = false;        // record events around the persistent decode kernel
  cudaEvent_t dk_start = nullptr, dk_end = nullptr;
  uint32_t stale_epoch = 0;        // test hook: publish QKV under the previous epoch
  // The KV cache's bookkeeping (cache::KvCache, src/core/cache/kv.h): the
  // tokens every sequence's cache holds, and the most written since it was
  // last emptied; each layer's attention window beside b.slots.
  uint32_t length = 0, written = 0;
  std::vector<uint32_t> windows;
  // The decode kernel's flag-in-data words: QKV products, attention output and
  // few-split partials, gated activation.
  unsigned long long *norm_ll = nullptr;
  unsigned long long *qkv_ll = nullptr, *attn_ll = nullptr, *part_o_ll = nullptr, *part_ml_ll = nullptr,
                     *act_ll = nullptr;
  std::map<GraphKey, cudaGraphExec_t> graphs;
  std::vector<void*> allocations;

  ~fz_batch() {
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    if (trace) cudaFree(trace);
    if (dk_start) cudaEventDestroy(dk_start);
    if (dk_end) cudaEventDestroy(dk_end);
    for (void* p : allocations) cudaFree(p);
    for (void* p : row_allocs) cudaFree(p);
    for (auto& s : slot) {
      if (s.step) cudaFreeHost(s.step);
      if (s.ids) cudaFreeHost(s.ids);
      if (s.seeds) cudaFreeHost(s.seeds);
      if (s.records) cudaFreeHost(s.records);
      if (s.error) cudaFreeHost(s.error);
      if (s.copied) cudaEventDestroy(s.copied);
      if (s.done) cudaEventDestroy(s.done);
    }
  }
  template <typename T>
  fz_status alloc(T** p, size_t bytes) {
    void* v = nullptr;
    cudaError_t e = cudaMalloc(&v, bytes ? bytes : 16);
    if (e != cudaSuccess)
      return fail(FZ_ERR_FIT, "device allocation of " + std::to_string(bytes) + " bytes: " + cudaGetErrorString(e));
    allocations.push_back(v);
    *p = static_cast<T*>(v);
    return cudaMemset(v, 0, bytes ? bytes : 16) == cudaSuccess ? FZ_OK : fail(FZ_ERR_CUDA, "memset");
  }
  template <typename T>
  fz_status alloc_row(T** p, size_t bytes) {
    void* v = nullptr;
    cudaError_t e = cudaMalloc(&v, bytes ? bytes : 16);
    if (e != cudaSuccess)
      return fail(FZ_ERR_FIT, "device allocation of " + std::to_string(bytes) + " bytes: " + cudaGetErrorString(e));
    row_allocs.push_back(v);
    *p = static_cast<T*>(v);
    return cudaMemset(v, 0, bytes ? bytes : 16) == cudaSuccess ? FZ_OK : fail(FZ_ERR_CUDA, "memset");
  }
};

namespace {

// ------------------------------------------------------------ describe

fz_status describe(fz_model& m) {
  const GgufIndex& ix = m.index;
  auto it = ix.metadata.find("general.architecture");
  if (it == ix.metadata.end() || it->second.s != "gemma3")
    return fail(FZ_ERR_ARCHITECTURE, "general.architecture is not gemma3");
  Shape& s = m.shape;
  const std::string a = "gemma3.";
  struct Req { const char* key; uint32_t* v; } req[] = {
      {"block_count", &s.layers}, {"context_length", &s.context}, {"embedding_length", &s.hidden},
      {"feed_forward_length", &s.ffn}, {"attention.head_count", &s.heads},
      {"attention.head_count_kv", &s.kv_heads}};
  for (auto& r : req)
    if (!ix.get_u32(a + r.key, *r.v) || *r.v == 0) return fail(FZ_ERR_ARCHITECTURE, a + r.key + " missing or zero");
  if (!ix.get_f32(a + "attention.layer_norm_rms_epsilon", s.eps))
    return fail(FZ_ERR_ARCHITECTURE, a + "attention.layer_norm_rms_epsilon missing");
  if (!ix.get_f32(a + "rope.freq_base", s.rope_global)) return fail(FZ_ERR_ARCHITECTURE, a + "rope.freq_base missing");
  s.rope_local = 10000.f;
  ix.get_f32(a + "rope.freq_base_swa", s.rope_local);
  s.head_dim = s.hidden / s.heads;
  ix.get_u32(a + "attention.key_length", s.head_dim);
  uint32_t vlen = s.head_dim;
  ix.get_u32(a + "attention.value_length", vlen);
  if (vlen != s.head_dim) return fail(FZ_ERR_ARCHITECTURE, "value length differs from key length");
  s.window = 0;
  ix.get_u32(a + "attention.sliding_window", s.window);
  s.pattern = 6;
  ix.get_u32(a + "attention.sliding_window_pattern", s.pattern);
  if (s.pattern == 0) return fail(FZ_ERR_ARCHITECTURE, "sliding window pattern 0");
  float cap = 0.f;
  if ((ix.get_f32(a + "attn_logit_softcapping", cap) && cap != 0.f) ||
      (ix.get_f32(a + "final_logit_softcapping", cap) && cap != 0.f))
    return fail(FZ_ERR_ARCHITECTURE, "logit softcapping is not run");
  if (s.heads % s.kv_heads) return fail(FZ_ERR_ARCHITECTURE, "head_count_kv does not divide head_count");
  if (s.head_dim != 256) return fail(FZ_ERR_NOT_SUPPORTED, "head dimension other than 256");
  if (s.heads / s.kv_heads > 8) return fail(FZ_ERR_NOT_SUPPORTED, "more than 8 query heads a KV head");
  if (s.hidden % 64 || s.ffn % 64 || (s.heads * s.head_dim) % 64 || s.hidden > 8192)
    return fail(FZ_ERR_NOT_SUPPORTED, "widths must be multiples of 64 (hidden at most 8192)");
  const fz::GgufTensor* embd = ix.find("token_embd.weight");
  if (!embd || embd->dims.size() != 2 || embd->dims[0] != s.hidden)
    return fail(FZ_ERR_ARCHITECTURE, "token_embd.weight missing or not [hidden, vocab]");
  if (embd->type != kTypeQ4_0 && embd->type != kTypeQ8_0)
    return fail(FZ_ERR_NOT_SUPPORTED, "token_embd.weight: type " + std::to_string(embd->type) + " (Q4_0 or Q8_0)");
  m.embd_type = embd->type;
  s.vocab = (uint32_t)embd->dims[1];
  if (s.vocab % 16) return fail(FZ_ERR_NOT_SUPPORTED, "vocabulary not a multiple of 16");
  if (ix.find("output.weight")) return fail(FZ_ERR_NOT_SUPPORTED, "an untied output head");
  // (type 3 names a down projection, which may be Q4_0 or Q4_1)
  auto need = [&](const std::string& name, uint32_t type, uint64_t d0, uint64_t d1) -> fz_status {
    const fz::GgufTensor* t = ix.find(name);
    if (!t) return fail(FZ_ERR_ARCHITECTURE, "missing tensor " + name);
    const bool ok = type == kTypeQ4_1 ? (t->type == kTypeQ4_0 || t->type == kTypeQ4_1) : t->type == type;
    if (!ok) return fail(FZ_ERR_NOT_SUPPORTED, name + ": type " + std::to_string(t->type));
    if (t->dims[0] != d0 || (d1 && (t->dims.size() != 2 || t->dims[1] != d1)))
      return fail(FZ_ERR_ARCHITECTURE, name + ": unexpected shape");
    return FZ_OK;
  };
  fz_status st;
  if ((st = need("output_norm.weight", 0, s.hidden, 0))) return st;
  const uint32_t Q = s.heads * s.head_dim, KV = s.kv_heads * s.head_dim;
  for (uint32_t l = 0; l < s.layers; l++) {
    const std::string p = "blk." + std::to_string(l) + ".";
    if ((st = need(p + "attn_norm.weight", 0, s.hidden, 0)) || (st = need(p + "attn_q.weight", 2, s.hidden, Q)) ||
        (st = need(p + "attn_k.weight", 2, s.hidden, KV)) || (st = need(p + "attn_v.weight", 2, s.hidden, KV)) ||
        (st = need(p + "attn_q_norm.weight", 0, s.head_dim, 0)) ||
        (st = need(p + "attn_k_norm.weight", 0, s.head_dim, 0)) ||
        (st = need(p + "attn_output.weight", 2, Q, s.hidden)) ||
        (st = need(p + "post_attention_norm.weight", 0, s.hidden, 0)) ||
        (st = need(p + "ffn_norm.weight", 0, s.hidden, 0)) || (st = need(p + "ffn_gate.weight", 2, s.hidden, s.ffn)) ||
        (st = need(p + "ffn_up.weight", 2, s.hidden, s.ffn)) || (st = need(p + "ffn_down.weight", kTypeQ4_1, s.ffn, s.hidden)) ||
        (st = need(p + "post_ffw_norm.weight", 0, s.hidden, 0)))
      return st;
  }
  return FZ_OK;
}

fz_status place_matrix(fz_model& m, DevMatrix& d, uint32_t n, uint32_t k) {
  d.n = n;
  d.k = k;
  fz_status st;
  if ((st = m.alloc(&d.codes, fz::q4_codes_bytes(n, k)))) return st;
  return m.alloc(&d.scales, fz::q4_scales_bytes(n, k));
}

constexpr uint64_t kLoadStage = 32ull << 20;   // the streaming load's device stage

// Places every buffer the model's tensors go to and lists them as sinks in
// file order (done at load_begin, so that chunks are repacked as they come).
fz_status place_model(fz_model& m) {
  const Shape& s = m.shape;
  const uint32_t Q = s.heads * s.head_dim, KV = s.kv_heads * s.head_dim;
  fz_status st;
  m.weight_bytes = 0;
  auto add_matrix = [&](const std::string& name, DevMatrix& d, uint32_t row0, int group, float* corr = nullptr) {
    const fz::GgufTensor* t = m.index.find(name);
    fz_model::Sink k;
    k.begin = m.index.data_offset + t->offset;
    k.end = k.begin + t->bytes;
    k.mat = &d;
    k.row0 = row0;
    k.k = (uint32_t)t->dims[0];
    k.type = t->type;
    k.corr = corr;
    k.group = group;
    k.name = name;
    m.sinks.push_back(k);
  };
  auto add_gain = [&](const std::string& name, float** out) -> fz_status {
    const fz::GgufTensor* t = m.index.find(name);
    fz_status g;
    if ((g = m.alloc(out, t->bytes))) return g;
    fz_model::Sink k;
    k.begin = m.index.data_offset + t->offset;
    k.end = k.begin + t->bytes;
    k.gain = *out;
    k.name = name;
    m.sinks.push_back(k);
    return FZ_OK;
  };
  if (m.embd_type == kTypeQ8_0) {
    m.embd.n = s.vocab;
    m.embd.k = s.hidden;
    if ((st = m.alloc(&m.embd_q8, (size_t)s.vocab * s.hidden)) ||
        (st = m.alloc(&m.embd_q8_scales, (size_t)s.vocab * (s.hidden / 32) * 2)))
      return st;
    add_matrix("token_embd.weight", m.embd, 0, -1);
    m.sinks.back().q8_codes = m.embd_q8;
    m.sinks.back().q8_scales = m.embd_q8_scales;
  } else {
    if ((st = place_matrix(m, m.embd, s.vocab, s.hidden))) return st;
    add_matrix("token_embd.weight", m.embd, 0, -1);
  }
  bool any_q4_1 = false;
  if ((st = add_gain("output_norm.weight", &m.output_norm))) return st;
  m.layers.resize(s.layers);
  for (uint32_t l = 0; l < s.layers; l++) {
    Layer& L = m.layers[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    if ((st = place_matrix(m, L.qkv, Q + 2 * KV, s.hidden)) || (st = place_matrix(m, L.o, s.hidden, Q)) ||
        (st = place_matrix(m, L.gate, s.ffn, s.hidden)) || (st = place_matrix(m, L.up, s.ffn, s.hidden)) ||
        (st = place_matrix(m, L.down, s.hidden, s.ffn)))
      return st;
    // The layer's products, each a group whose f16 copies are made once its tensors are whole.
    const int g0 = (int)m.groups.size();
    for (DevMatrix* d : {&L.qkv, &L.o, &L.gate, &L.up, &L.down}) m.groups.push_back(d);
    m.group_left.insert(m.group_left.end(), {3u, 1u, 1u, 1u, 1u});
    add_matrix(p + "attn_q.weight", L.qkv, 0, g0);
    add_matrix(p + "attn_k.weight", L.qkv, Q, g0);
    add_matrix(p + "attn_v.weight", L.qkv, Q + KV, g0);
    add_matrix(p + "attn_output.weight", L.o, 0, g0 + 1);
    add_matrix(p + "ffn_gate.weight", L.gate, 0, g0 + 2);
    add_matrix(p + "ffn_up.weight", L.up, 0, g0 + 3);
    L.down_type = m.index.find(p + "ffn_down.weight")->type;
    if (L.down_type == kTypeQ4_1) {
      if ((st = m.alloc(&L.down_corr, (size_t)s.hidden * (s.ffn / 32) * 4))) return st;
      any_q4_1 = true;
    }
    add_matrix(p + "ffn_down.weight", L.down, 0, g0 + 4, L.down_corr);
    if ((st = add_gain(p + "attn_norm.weight", &L.attn_norm)) || (st = add_gain(p + "attn_q_norm.weight", &L.q_norm)) ||
        (st = add_gain(p + "attn_k_norm.weight", &L.k_norm)) ||
        (st = add_gain(p + "post_attention_norm.weight", &L.post_attn_norm)) ||
        (st = add_gain(p + "ffn_norm.weight", &L.ffn_norm)) ||
        (st = add_gain(p + "post_ffw_norm.weight", &L.post_ffw_norm)))
      return st;
    // Window layers: every pattern-th layer attends globally (gemma3.cpp:79-85).
    L.global = s.window == 0 || l % s.pattern == s.pattern - 1;
    L.window = L.global ? s.context : s.window;
    L.rope_base = L.global ? s.rope_global : s.rope_local;
    // theta_k / 2 pi in f64, rounded once (rope.cpp:95-107).
    std::vector<float> turns(s.head_dim / 2);
    for (uint32_t k = 0; k < s.head_dim / 2; k++) {
      const double theta = std::pow((double)L.rope_base, -2.0 * (double)k / (double)s.head_dim);
      turns[k] = (float)(theta / (2.0 * 3.14159265358979323846));
    }
    if ((st = m.alloc(&L.turns, turns.size() * 4))) return st;
    FZ_CUDA(cudaMemcpy(L.turns, turns.data(), turns.size() * 4, cudaMemcpyHostToDevice));
    // f16 hi and lo copies of the layer's products for the prefill GEMM
    // (2.8 GB for Gemma 3 1B beside its 0.39 GB of Q4_0 layers).
    for (DevMatrix* d : {&L.qkv, &L.o, &L.gate, &L.up, &L.down}) {
      const size_t bytes = (size_t)d->n * d->k * 2;
      if ((st = m.alloc(&d->f16_hi, bytes)) || (st = m.alloc(&d->f16_lo, bytes))) return st;
    }
  }
  std::sort(m.sinks.begin(), m.sinks.end(),
            [](const fz_model::Sink& a, const fz_model::Sink& b) { return a.begin < b.begin; });
  FZ_CUDA(cudaMalloc(&m.stage, kLoadStage));
  if (any_q4_1) FZ_CUDA(cudaMalloc(&m.stage_q4_0, kLoadStage));
  m.cursor = 0;
  return FZ_OK;
}

// Repacks the whole 16-row groups the stage holds of the current matrix sink
// and moves the remainder (part of a group) to the stage's start.
// A Q8_0 table is repacked a whole row at a time instead; a Q4_1 matrix's
// groups are first split into Q4_0 blocks and their corrections.
fz_status drain_stage(fz_model& m, fz_model::Sink& k) {
  const uint32_t kb = k.k / 32;
  const bool q8 = k.type == kTypeQ8_0;
  const uint64_t group_bytes = q8 ? (uint64_t)kb * 34 : 16ull * kb * (k.type == kTypeQ4_1 ? 20 : 18);
  const uint64_t groups = m.stage_fill / group_bytes;
  if (!groups) return FZ_OK;
  DevMatrix& d = *k.mat;
  const uint32_t row = k.row0 + m.rows_done;
  const uint32_t rows = (uint32_t)(q8 ? groups : 16 * groups);
  if (q8) {
    fz_status st;
    if ((st = fz_q8_0_repack(m.stage, rows, k.k, k.q8_codes + (size_t)row * k.k, k.q8_scales + (size_t)row * kb,
                             m.dev->stream)))
      return st;
  } else {
    const uint8_t* blocks = m.stage;
    if (k.type == kTypeQ4_1) {
      FZ_CUDA(fz::launch_q4_1_split(m.stage, (size_t)rows * kb, m.stage_q4_0, k.corr + (size_t)row * kb,
                                    m.dev->stream));
      blocks = m.stage_q4_0;
    }
    FZ_CUDA(fz::launch_repack(blocks, rows, k.k, d.codes + (size_t)(row / 16) * (k.k / 64) * 32,
                              d.scales + (size_t)(row / 16) * (k.k / 64) * 8, m.dev->stream));
  }
  m.rows_done += rows;
  const uint64_t rest = m.stage_fill - groups * group_bytes;
  if (rest)   // (rest < one group <= the bytes just repacked: the ranges do not overlap)
    FZ_CUDA(cudaMemcpyAsync(m.stage, m.stage + groups * group_bytes, rest, cudaMemcpyDeviceToDevice, m.dev->stream));
  m.stage_fill = rest;
  return FZ_OK;
}

// A sink's last byte has arrived: the layer product's f16 copies once all
// of its tensors are whole.
fz_status finish_sink(fz_model& m, const fz_model::Sink& k) {
  if (k.mat && m.stage_fill) return fail(FZ_ERR_UPLOAD, "tensor " + k.name + " is not whole 16-row groups");
  if (k.group >= 0 && --m.group_left[k.group] == 0) {
    DevMatrix* d = m.groups[k.group];
    // (a layer's Q4_1 down projection is a group of its own: its corrections are k.corr)
    FZ_CUDA(fz::launch_dequant_f16(d->view(), d->f16_hi, d->f16_lo, m.dev->stream, k.corr));
  }
  m.rows_done = 0;
  m.stage_fill = 0;
  return FZ_OK;
}

// ------------------------------------------------------------ launch configs

struct Split {
  uint32_t rg, ks, cluster;
};

Split split_for(uint32_t n, uint32_t k, uint32_t m, int epi) {
  const uint32_t nbp = k / 64;
  // Eight warps a CTA: a gated pair splits K four ways; the head streams
  // whole row groups, one a warp; everything else splits K eight ways.
  if (epi == fz::kEpilogueGated) return {2, 4, 1};
  if (epi == fz::kEpilogueHead) return {8, 1, 1};
  Split s{1, 8, 1};
  const uint32_t mq = (m + 3) / 4;
  // Keep each CTA's share of X fragments under ~110 KB of shared memory, and
  // give narrow products with long rows enough CTAs.
  while ((size_t)2 * ((nbp + s.cluster - 1) / s.cluster) * 2 * mq * 32 * 8 > 110 * 1024 && s.cluster < 8)
    s.cluster *= 2;
  if (n / 16 < 100 && nbp >= 64 && s.cluster < 2) s.cluster = 2;
  if (const char* v = std::getenv("FRIZZLE_B200_CLUSTER")) s.cluster = (uint32_t)std::max(1, std::atoi(v));
  return s;
}

fz_status run_matvec(fz::MatvecArgs a, int pro, int epi, cudaStream_t stream, bool pdl) {
  const Split s = split_for(a.mat[0].n, a.mat[0].k, a.m, epi);
  a.rg_per_cta = s.rg;
  a.k_split = s.ks;
  a.cluster = s.cluster;
  FZ_CUDA(fz::launch_matvec(a, pro, epi, stream, pdl));
  return FZ_OK;
}

// The tied head over h.m rows with the norm prologue h.norm (logits into
// h.out, the greedy keys max-reduced into h.head.argmax, cleared by the
// caller).  A Q4_0 table streams through the head matvec with the norm and
// argmax fused; a Q8_0 one (the pinned file's) as the norm's rows in f32,
// the Q8_0 product eight rows a launch, then the argmax over each row.
fz_status run_head(fz_batch& b, const fz::MatvecArgs& h, cudaStream_t st, bool pdl) {
  const fz_model& m = *b.model;
  if (m.embd_type != kTypeQ8_0) return run_matvec(h, fz::kPrologueNorm, fz::kEpilogueHead, st, pdl);
  const uint32_t width = m.shape.hidden, vocab = m.shape.vocab;
  if (h.m > b.head_rows || h.out_stride != vocab) return fail(FZ_ERR_ARGUMENT, "head rows outside its scratch");
  FZ_CUDA(fz::launch_norm_f32(h, b.head_x, st, pdl));
  fz_status stt;
  for (uint32_t r0 = 0; r0 < h.m; r0 += 8) {
    const uint32_t n = std::min<uint32_t>(8, h.m - r0);
    if ((stt = fz_q8_0_matvec(m.embd_q8, m.embd_q8_scales, vocab, width, b.head_x + (size_t)r0 * width, n,
                              h.out + (size_t)r0 * vocab, st)))
      return stt;
  }
  FZ_CUDA(fz::launch_argmax_rows(h.out, h.m, vocab, h.head.argmax, st));
  return FZ_OK;
}

// ------------------------------------------------------------ per-row scratch

// A layer's key/value ring for one sequence: a window layer keeps its window,
// a prefill block (512) and the rollback reserve (plan.cpp:335-336), rounded
// up to whole 32-slot chunks so that a decode chunk's tensor copy never
// wraps; never more than the context.  A global layer's window is the
// trained context, so its ring is the context.
uint32_t ring_slots(uint32_t window, uint32_t context, uint32_t rollback) {
  const uint64_t ring = ((uint64_t)window + 512 + rollback + 31) / 32 * 32;
  return (uint32_t)std::min<uint64_t>(context, ring);
}

// Every layer's attention window (the trained context for global layers).
std::vector<uint32_t> layer_windows(const Shape& s) {
  std::vector<uint32_t> w(s.layers);
  for (uint32_t l = 0; l < s.layers; l++)
    w[l] = s.window == 0 || l % s.pattern == s.pattern - 1 ? s.context : s.window;
  return w;
}

// The tensor-core attention splits the keys of a block longer than this many
// 64-key tiles (1280 keys) over two CTAs, when one wave holds all its blocks
// (a window layer's blocks stay whole: 512 keys are at most 10 tiles).
constexpr uint32_t kAttnSplitTiles = 20;
static_assert(FZ_ATTENTION_WIDE_SPLIT_FLOATS == fz::kAttnSplitBlocks * 2 * fz::kAttnSplitFloats, "split scratch size");

// Its split halves: wide steps (more than 16 rows) with the tensor-core form.
uint64_t attn_split_bytes(const Shape& s, uint64_t rows) {
  if (rows <= (uint64_t)fz::kMaxTokens || !fz::attention_prefill_supported(s.heads, s.kv_heads, s.head_dim)) return 0;
  return (uint64_t)fz::kAttnSplitBlocks * 2 * fz::kAttnSplitFloats * 4;
}

// The device bytes of a batch, counted with the expressions its allocations
// use (fz_batch_create, alloc_rows): the key/value rings, and the scratch
// for `rows` token rows a step.
struct BatchBytes {
  uint64_t cache = 0, scratch = 0;
};
BatchBytes batch_bytes(const Shape& s, uint32_t S, uint32_t context, uint32_t rollback, uint32_t rows) {
  BatchBytes out;
  uint32_t splits_max = 1;
  for (uint32_t w : layer_windows(s)) {
    const uint64_t per_seq = (uint64_t)ring_slots(w, context, rollback) * s.kv_heads * s.head_dim;
    out.cache += 2 * per_seq * S * 2;
    const uint32_t keys = std::min(w, context);
    splits_max = std::max<uint32_t>({splits_max, (keys + split_keys_for(keys) - 1) / split_keys_for(keys),
                                     std::min<uint32_t>((keys + fz::kDecodeSplitKeys - 1) / fz::kDecodeSplitKeys,
                                                        fz::kDecodeMaxSplits)});
  }
  const uint64_t Q = (uint64_t)s.heads * s.head_dim, KV = (uint64_t)s.kv_heads * s.head_dim;
  const uint64_t R8 = (uint64_t)fz::kDecodeMaxRows * 8, V = s.vocab, T16 = fz::kMaxTokens;
  const uint64_t tiles = fz::select_tiles(s.vocab), table_words = 2ull * s.layers + 5ull * kMaxEdits;
  uint64_t f = R8 * s.hidden + R8 * (Q + 2 * KV) + R8 * Q + R8 * s.ffn + R8 * s.heads * fz::kDecodeFoldSplits * s.head_dim +
               R8 * s.heads * fz::kDecodeFoldSplits * 2;
  f += S * V * 4 + S * 8 + S * tiles * 64 * 8 + S * 128 * 4 + S * 16 + 64 + S * 8 + 16 + S * table_words * 4 +
       S * capture_layout(s).words * 4 + T16 * s.hidden * 4 + T16 * V * 4 + T16 * 8 + T16 * tiles * 64 * 8;
  const uint64_t M = rows, X = std::max<uint64_t>(s.hidden, Q);
  const uint64_t PM = fz::attention_prefill_supported(s.heads, s.kv_heads, s.head_dim) ? std::min<uint64_t>(M, T16) : M;
  f += M * s.hidden * 4 * 2 + M * (Q + 2 * KV) * 4 + M * Q * 4 * 2 + M * s.hidden * 4 * 2 + M * s.ffn * 4 +
       PM * s.heads * splits_max * s.head_dim * 4 + PM * s.heads * splits_max * 2 * 4 +
       attn_split_bytes(s, rows) + (uint64_t)s.layers * (1 + M * s.kv_heads) * 4 + M * 4 + M * X * 2 * 2 + M * s.ffn * 2 * 2 +
       (fz::kDecodeOSlices + fz::kDecodeDownSlices) * M * s.hidden * 4 +
       fz::decode_sync_words(s.layers, (uint32_t)M, s.kv_heads) * 4;
  out.scratch = f;
  return out;
}

// plan_residency's sizing (plan.cpp:321-419) for one batch: `fixed` bytes
// (weights, copies) plus the batch's scratch and rings must stay within the
// budget.  The cost never falls as the context or the sequences grow, so the
// largest context (or sequence count) that fits is found by bisection.
fz_status plan_batch(const Shape& s, uint64_t fixed, fz_plan* p) {
  if (p->sequences > (uint32_t)fz::kMaxTokens) return fail(FZ_ERR_ARGUMENT, "more than 16 sequences a batch");
  if (p->context > s.context) return fail(FZ_ERR_ARGUMENT, "a context past the trained context");
  const uint32_t rows = p->rows ? p->rows : 4096u;
  if (rows < fz::kMaxTokens) return fail(FZ_ERR_ARGUMENT, "fewer than 16 rows a step");
  const uint64_t slack = 1ull << 26;   // allocation granules and small per-batch buffers: 64 MiB
  const auto cost = [&](uint32_t S, uint32_t ctx) {
    const BatchBytes b = batch_bytes(s, S, ctx, p->rollback, std::max<uint32_t>(rows, S * fz::kMaxTokens));
    return fixed + slack + b.scratch + b.cache;
  };
  const uint32_t shortest = std::min<uint32_t>(512, s.context);
  uint32_t S = p->sequences ? p->sequences : 1u;
  uint32_t ctx = p->context ? p->context : shortest;
  if (cost(S, ctx) > p->budget) {
    p->total_bytes = cost(S, ctx);
    return fail(FZ_ERR_FIT, "the weights, scratch and shortest cache exceed the budget (PlanError::ExceedsBudget)");
  }
  if (!p->sequences) {
    uint32_t lo = 1, hi = fz::kMaxTokens;   // the most sequences that fit at the context
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo + 1) / 2;
      if (cost(mid, ctx) <= p->budget) lo = mid;
      else hi = mid - 1;
    }
    S = lo;
  }
  if (!p->context) {
    uint32_t lo = shortest, hi = s.context;   // the largest context that fits for S sequences
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo + 1) / 2;
      if (cost(S, mid) <= p->budget) lo = mid;
      else hi = mid - 1;
    }
    ctx = lo;
  }
  const BatchBytes b = batch_bytes(s, S, ctx, p->rollback, std::max<uint32_t>(rows, S * fz::kMaxTokens));
  p->sequences = S;
  p->context = ctx;
  p->rows = rows;
  p->scratch_bytes = b.scratch;
  p->cache_bytes = b.cache;
  p->total_bytes = cost(S, ctx);
  return FZ_OK;
}

// The model's weights on the device (every tensor's bytes in its file form,
// the repacked layout being the same size, and the RoPE turns), and its f16
// prefill copies (f16 part and remainder of every layer product).
void weight_bytes_of(const fz_model& m, uint64_t& weights, uint64_t& copies) {
  const Shape& s = m.shape;
  weights = 0;
  // Q4_0, Q8_0 and f32 tensors take their file bytes on the device; a Q4_1
  // block (20 bytes) becomes a Q4_0 block and a 4-byte correction (22).
  for (const auto& t : m.index.tensors) weights += t.bytes + (t.type == kTypeQ4_1 ? t.bytes / 10 : 0);
  weights += (uint64_t)s.layers * (s.head_dim / 2) * 4;
  const uint64_t Q = (uint64_t)s.heads * s.head_dim, KV = (uint64_t)s.kv_heads * s.head_dim;
  copies = (uint64_t)s.layers * ((Q + 2 * KV) * s.hidden + s.hidden * Q + 3ull * s.ffn * s.hidden) * 2 * 2;
}

// (Re)allocates every buffer sized by the step's rows for `rows` rows.
fz_status alloc_rows(fz_batch& b, uint32_t rows) {
  const Shape& s = b.model->shape;
  FZ_CUDA(cudaStreamSynchronize(b.model->dev->stream));
  for (auto& kv : b.graphs) cudaGraphExecDestroy(kv.second);
  b.graphs.clear();
  for (void* p : b.row_allocs) cudaFree(p);
  b.row_allocs.clear();
  for (auto& sl : b.slot)
    if (sl.ids) {
      cudaFreeHost(sl.ids);
      sl.ids = nullptr;
    }
  const uint32_t Q = s.heads * s.head_dim, KV = s.kv_heads * s.head_dim;
  const size_t M = rows, X = std::max(s.hidden, Q);
  // Attention split partials serve steps of at most 16 rows (and the decode
  // kernel's); wider steps use the tensor-core attention, which needs none.
  const size_t PM = fz::attention_prefill_supported(s.heads, s.kv_heads, s.head_dim)
                        ? std::min<size_t>(rows, (size_t)fz::kMaxTokens)
                        : M;
  b.counters_per_layer = 1 + rows * s.kv_heads;
  fz_status st;
  if ((st = b.alloc_row(&b.hidden_a, M * s.hidden * 4)) || (st = b.alloc_row(&b.hidden_b, M * s.hidden * 4)) ||
      (st = b.alloc_row(&b.qkv, M * (Q + 2 * KV) * 4)) || (st = b.alloc_row(&b.q, M * Q * 4)) ||
      (st = b.alloc_row(&b.attn, M * Q * 4)) || (st = b.alloc_row(&b.y_attn, M * s.hidden * 4)) ||
      (st = b.alloc_row(&b.y_mlp, M * s.hidden * 4)) || (st = b.alloc_row(&b.act, M * s.ffn * 4)) ||
      (st = b.alloc_row(&b.partial_o, PM * s.heads * b.splits_max * s.head_dim * 4)) ||
      (st = b.alloc_row(&b.partial_ml, PM * s.heads * b.splits_max * 2 * 4)) ||
      (st = b.alloc_row(&b.attn_split, attn_split_bytes(s, rows))) ||
      (st = b.alloc_row(&b.counters, (size_t)s.layers * b.counters_per_layer * 4)) ||
      (st = b.alloc_row(&b.dids, M * 4)) || (st = b.alloc_row(&b.x16_hi, M * X * 2)) ||
      (st = b.alloc_row(&b.x16_lo, M * X * 2)) || (st = b.alloc_row(&b.act16_hi, M * s.ffn * 2)) ||
      (st = b.alloc_row(&b.act16_lo, M * s.ffn * 2)))
    return st;
  b.dsync_words = fz::decode_sync_words(s.layers, rows, s.kv_heads);
  if ((st = b.alloc_row(&b.y_parts, (fz::kDecodeOSlices + fz::kDecodeDownSlices) * M * s.hidden * 4)) ||
      (st = b.alloc_row(&b.dsync, b.dsync_words * 4)))
    return st;
  for (auto& sl : b.slot) FZ_CUDA(cudaMallocHost(&sl.ids, M * 4));
  FZ_CUDA(cudaDeviceSynchronize());
  b.rows_cap = rows;
  return FZ_OK;
}

// ------------------------------------------------------------ the step chain

// The persistent decode kernel serves one-token steps unless
// FRIZZLE_B200_LAYERED=1 asks for the per-operation launches.
bool decode_step_enabled() {
  const char* v = std::getenv("FRIZZLE_B200_LAYERED");
  return !(v && *v && *v != '0');
}

fz_status enqueue_forward(fz_batch& b, const GraphKey& key, cudaStream_t st);

// What a capture step adds after the forward pass (capture/capture.h): each
// layer's attention weights and statistics, then its readout.  The readout
// rows of the layers before the last (the residual each leaves) go through
// the final norm and the tied head kMaxTokens at a time, and the top 64 of
// each row into the layer's slot; the last layer's readout is the top 64 of
// the step's own logits, the candidates the draw chooses from.  A step that
// asks for no logits has no last readout and no final addition: both slots
// are zeroed.
fz_status enqueue_capture(fz_batch& b, const GraphKey& key, cudaStream_t st) {
  fz_model& m = *b.model;
  const Shape& s = m.shape;
  const CaptureLayout cl = capture_layout(s);
  const bool pdl = true;
  fz::WeightsArgs w{};
  w.step = b.dstep;
  w.store = b.captures;
  w.store_stride = cl.words;
  w.layers = b.cap_layers;
  w.heads = s.heads;
  w.kv_heads = s.kv_heads;
  w.head_dim = s.head_dim;
  w.scale_log2e = (float)((double)(1.0f / std::sqrt((float)s.head_dim)) * 1.4426950408889634);
  FZ_CUDA(fz::launch_attention_weights(w, s.layers, b.S, st, pdl));
  fz::ReadoutArgs r{};
  r.store = b.captures;
  r.store_stride = cl.words;
  r.layers = b.cap_layers;
  r.n_layers = s.layers;
  r.width = s.hidden;
  r.rows = b.ro_rows;
  r.logits = b.ro_logits;
  r.vocab = s.vocab;
  r.tile_best = b.ro_tile_best;
  const uint32_t rows = b.S * (s.layers - 1);
  for (uint32_t g0 = 0; g0 < rows; g0 += fz::kMaxTokens) {
    const uint32_t n = std::min<uint32_t>(fz::kMaxTokens, rows - g0);
    FZ_CUDA(fz::launch_readout_rows(r, g0, n, st, pdl));
    FZ_CUDA(cudaMemsetAsync(b.ro_argmax, 0, (size_t)n * 8, st));
    fz::MatvecArgs h{};
    h.step = b.dstep;
    h.mat[0] = m.embd.view();
    h.m = n;
    h.seq_tokens = 1;
    h.norm.hidden_in = b.ro_rows;
    h.norm.gain = m.output_norm;
    h.norm.eps = s.eps;
    h.norm.width = s.hidden;
    h.norm.row_of_token_stride = 1;
    h.out = b.ro_logits;
    h.out_stride = s.vocab;
    h.head.argmax = b.ro_argmax;
    fz_status stt;
    if ((stt = run_head(b, h, st, pdl))) return stt;
    FZ_CUDA(fz::launch_readout_select(r, g0, n, false, st, pdl));
  }
  if (key.logits) {
    r.logits = b.logits;
    FZ_CUDA(fz::launch_readout_select(r, 0, b.S, true, st, pdl));
  } else {
    const CaptureSlot& last = cl.layer[s.layers - 1];
    FZ_CUDA(cudaMemset2DAsync(b.captures + last.mlp_added, cl.words * 4, 0, (size_t)s.hidden * 4, b.S, st));
    FZ_CUDA(cudaMemset2DAsync(b.captures + last.readout, cl.words * 4, 0, (size_t)kReadoutWords * 4, b.S, st));
  }
  return FZ_OK;
}

// Device address of a pinned host buffer (mapped into the device's address space).
template <typename T>
fz_status mapped(T* host, T** dev) {
  void* d = nullptr;
  FZ_CUDA(cudaHostGetDevicePointer(&d, const_cast<void*>(static_cast<const void*>(host)), 0));
  *dev = static_cast<T*>(d);
  return FZ_OK;
}

// The whole step: its inputs staged from the host slot by a kernel, the
// forward pass (and the capture), its records and error word published into
// the slot by a kernel.
fz_status enqueue_step(fz_batch& b, const GraphKey& key, cudaStream_t st) {
  auto& sl = b.slot[key.slot];
  fz::StageArgs sa{};
  fz_status stt;
  if ((stt = mapped<const DeviceStep>(sl.step, &sa.step_h)) || (stt = mapped<const uint32_t>(sl.seeds, &sa.seeds_h)) ||
      (stt = mapped<const uint32_t>(sl.ids, &sa.ids_h)))
    return stt;
  sa.step_d = b.dstep;
  sa.seeds_d = b.dseeds;
  sa.ids_d = b.dids;
  sa.seed_words = 2 * b.S;
  sa.id_words = key.tokens * b.S;   // (a fed step's are not read)
  sa.zero = b.dsync;                // the decode kernel's phase counters start at zero
  sa.zero_words = (uint32_t)b.dsync_words;
  FZ_CUDA(fz::launch_stage(sa, st));
  stt = enqueue_forward(b, key, st);
  if (!stt && key.capture) stt = enqueue_capture(b, key, st);
  if (stt) return stt;
  fz::PublishArgs pa{};
  pa.records_d = b.records;
  pa.record_words = 4 * b.S;
  pa.error_d = b.gemm_error;
  if ((stt = mapped(sl.records, &pa.records_h)) || (stt = mapped(sl.error, &pa.error_h))) return stt;
  FZ_CUDA(fz::launch_publish(pa, st));
  return FZ_OK;
}

fz_status enqueue_forward(fz_batch& b, const GraphKey& key, cudaStream_t st) {
  fz_model& m = *b.model;
  const Shape& s = m.shape;
  const uint32_t T = key.tokens, M = b.S * T;
  const bool pdl = true;
  const CaptureLayout cl = capture_layout(s);
  float* cap = key.capture ? b.captures : nullptr;
  const uint32_t QW = s.heads * s.head_dim;
  fz_status stt;
  {
    fz::EmbedArgs e{};
    e.step = b.dstep;
    e.table = m.embd.view();
    e.q8_codes = m.embd_q8;
    e.q8_scales = m.embd_q8_scales;
    e.ids = b.dids;
    e.records = b.records;
    e.seq_tokens = T;
    e.m = M;
    e.scale = std::sqrt((float)s.hidden);
    e.hidden = b.hidden_a;
    e.argmax = b.argmax;
    e.seqs = b.S;
    FZ_CUDA(fz::launch_embed(e, st, pdl));
  }
  if (T == 1 && decode_step_enabled() &&
      fz::decode_supported(b.S, s.hidden, s.ffn, s.heads, s.kv_heads, s.head_dim)) {
    // One token for each sequence: the whole step in one persistent kernel.
    // (the stage kernel cleared the phase counters, b.dsync)
    fz::DecodeArgs d{};
    d.step = b.dstep;
    d.layers = b.dlayers;
    d.kv_maps = b.kv_maps;
    d.n_layers = s.layers;
    d.m = b.S;
    d.hidden = s.hidden;
    d.ffn = s.ffn;
    d.heads = s.heads;
    d.kv_heads = s.kv_heads;
    d.eps = s.eps;
    d.scale_log2e = (float)((double)(1.0f / std::sqrt((float)s.head_dim)) * 1.4426950408889634);
    d.hidden_a = b.hidden_a;
    d.hidden_b = b.hidden_b;
    d.qkv = b.qkv;
    d.qkv_ll = b.qkv_ll;
    d.attn_ll = b.attn_ll;
    d.act_ll = b.act_ll;
    d.norm_ll = b.norm_ll;
    d.part_o_ll = b.part_o_ll;
    d.part_ml_ll = b.part_ml_ll;
    d.attn = b.attn;
    d.y_attn = b.y_parts;
    d.act = b.act;
    d.y_mlp = b.y_parts + (size_t)fz::kDecodeOSlices * b.S * s.hidden;
    d.partial_o = b.partial_o;
    d.partial_ml = b.partial_ml;
    d.max_splits = b.splits_max;
    d.sync = b.dsync;
    d.edit_table = key.edits ? b.edit_tables : nullptr;
    d.table_stride = b.table_words;
    d.capture = cap;
    d.capture_stride = cl.words;
    d.cap_region2 = cl.layer[0].residual;
    d.cap_block = 3ull * s.hidden + (uint64_t)s.heads * s.head_dim + 2ull * s.heads + kReadoutWords;
    d.cap_keys_local = s.window == 0 ? s.context : std::min(s.window, s.context);
    d.cap_keys_global = s.context;
    d.cap_pattern = s.pattern;
    for (uint32_t l = 0; l < s.layers; l++)  // the closed form the kernel uses
      if (cl.layer[l].keys != (s.window == 0 || l % s.pattern == s.pattern - 1 ? d.cap_keys_global
                                                                                : d.cap_keys_local))
        return fail(FZ_ERR_NOT_SUPPORTED, "capture layout outside the decode kernel's closed form");
    d.head = m.embd.view();
    d.output_norm = m.output_norm;
    // The head runs as its own streaming launch (below), not inside the step.
    d.logits = nullptr;
    d.argmax = b.argmax;
    d.error = b.gemm_error;
    if (b.trace) {
      FZ_CUDA(cudaMemsetAsync(b.trace, 0, (size_t)b.trace_ctas * b.trace_events * 8, st));
      d.trace = b.trace;
      d.trace_stride = b.trace_events;
    }
    // (a timed step is launched directly, not from a graph: plain events on
    // the stream bracket the kernel alone, a delay ahead of the first keeping
    // the stream busy while the host submits the launch)
    if (key.timed) {
      FZ_CUDA(fz::launch_delay(200000u, st));
      FZ_CUDA(cudaEventRecord(b.dk_start, st));
    }
    FZ_CUDA(fz::launch_decode(d, st));
    if (key.timed) FZ_CUDA(cudaEventRecord(b.dk_end, st));
    if (key.logits) {
      // Final norm (X plus the last down projection's K-slice partials) and the tied head.
      fz::MatvecArgs h{};
      h.step = b.dstep;
      h.mat[0] = m.embd.view();
      h.m = b.S;
      h.seq_tokens = 1;
      h.capture_stride = cl.words;
      h.norm.hidden_in = b.hidden_a;
      h.norm.y = d.y_mlp;
      h.norm.y_parts = fz::kDecodeDownSlices;
      h.norm.y_part_stride = (uint64_t)b.S * s.hidden;
      h.norm.post_gain = m.layers[s.layers - 1].post_ffw_norm;
      h.norm.gain = m.output_norm;
      h.norm.hidden_out = nullptr;
      h.norm.eps = s.eps;
      h.norm.width = s.hidden;
      h.norm.row_of_token_stride = 1;
      h.norm.capture_added = cap ? cap + cl.layer[s.layers - 1].mlp_added : nullptr;
      h.out = b.logits;
      h.out_stride = s.vocab;
      h.head.argmax = b.argmax;
      if ((stt = run_head(b, h, st, pdl))) return stt;
      fz::SelectArgs se{};
      se.step = b.dstep;
      se.logits = b.logits;
      se.vocab = s.vocab;
      se.seqs = b.S;
      se.argmax = b.argmax;
      se.seeds = b.dseeds;
      se.tile_best = b.tile_best;
      se.candidates = b.candidates;
      se.records = b.records;
      FZ_CUDA(fz::launch_select(se, st, pdl));
    }
    return FZ_OK;
  }
  if (M > (uint32_t)fz::kMaxTokens) {
    // Wide step: per-row norms into f16, the products on the tensor cores.
    __half* xlo = b.passes >= 2 ? b.x16_lo : nullptr;
    __half* alo = b.passes >= 2 ? b.act16_lo : nullptr;
    auto gemm = [&](const DevMatrix& w, const DevMatrix* up, const __half* xh, const __half* xl, float* out,
                    uint32_t stride, int epi, uint32_t layer) -> fz_status {
      fz::GemmArgs g{};
      g.step = b.dstep;
      g.w[0] = w.view();
      if (up) g.w[1] = up->view();
      g.w_hi[0] = w.f16_hi;
      g.w_lo[0] = w.f16_lo;
      if (up) {
        g.w_hi[1] = up->f16_hi;
        g.w_lo[1] = up->f16_lo;
      }
      g.m = M;
      g.x_hi = xh;
      g.x_lo = xl;
      g.exact_w = b.passes == 3 ? 1u : 0u;
      g.out = out;
      g.out_stride = stride;
      g.act_hi = b.act16_hi;
      g.act_lo = alo;
      g.edit_table = key.edits ? b.edit_tables : nullptr;
      g.table_stride = b.table_words;
      g.layer = layer;
      g.seq_tokens = T;
      g.capture_neurons = (cap && epi == fz::kGemmGated) ? cap + cl.layer[layer].neurons : nullptr;
      g.capture_stride = cl.words;
      g.error = b.gemm_error;
      FZ_CUDA(fz::launch_gemm(g, epi, st, pdl));
      return FZ_OK;
    };
    for (uint32_t l = 0; l < s.layers; l++) {
      const Layer& L = m.layers[l];
      uint32_t* lc = b.counters + (size_t)l * b.counters_per_layer;
      fz::MatvecArgs a{};
      a.step = b.dstep;
      a.m = M;
      a.seq_tokens = T;
      a.capture_stride = cl.words;
      a.norm.hidden_in = b.hidden_a;
      a.norm.y = l ? b.y_mlp : nullptr;
      a.norm.post_gain = l ? m.layers[l - 1].post_ffw_norm : nullptr;
      a.norm.gain = L.attn_norm;
      a.norm.hidden_out = b.hidden_b;
      a.norm.eps = s.eps;
      a.norm.width = s.hidden;
      a.norm.capture_residual = cap ? cap + cl.layer[l].residual : nullptr;
      a.norm.capture_added = (cap && l) ? cap + cl.layer[l - 1].mlp_added : nullptr;
      FZ_CUDA(fz::launch_norm_f16(a, b.x16_hi, xlo, st, pdl));
      if ((stt = gemm(L.qkv, nullptr, b.x16_hi, xlo, b.qkv, L.qkv.n, fz::kGemmWrite, l))) return stt;
      a.out = b.qkv;
      a.out_stride = L.qkv.n;
      a.rope.q_gain = L.q_norm;
      a.rope.k_gain = L.k_norm;
      a.rope.turns = L.turns;
      a.rope.eps = s.eps;
      a.rope.heads = s.heads;
      a.rope.kv_heads = s.kv_heads;
      a.rope.head_dim = s.head_dim;
      a.rope.key_cache = b.kc[l];
      a.rope.value_cache = b.vc[l];
      a.rope.slots = b.slots[l];
      a.rope.seq_stride = b.seq_stride[l];
      a.rope.query_out = b.q;
      a.rope.capture_query = cap ? cap + cl.layer[l].query : nullptr;
      FZ_CUDA(fz::launch_rope_rows(a, st, pdl));
      fz::AttentionArgs at{};
      at.step = b.dstep;
      at.q = b.q;
      at.key_cache = b.kc[l];
      at.value_cache = b.vc[l];
      at.seq_stride = b.seq_stride[l];
      at.slots = b.slots[l];
      at.heads = s.heads;
      at.kv_heads = s.kv_heads;
      at.head_dim = s.head_dim;
      at.window = L.window;
      at.seq_tokens = T;
      at.m = M;
      at.scale_log2e = (float)((double)(1.0f / std::sqrt((float)s.head_dim)) * 1.4426950408889634);
      at.split_keys = split_keys_for(std::min(L.window, b.context));
      at.splits = (std::min(L.window, b.context) + at.split_keys - 1) / at.split_keys;
      at.partial_o = b.partial_o;
      at.partial_ml = b.partial_ml;
      at.counters = lc + 1;
      at.out = b.attn;
      at.out_hi = b.x16_hi;
      at.out_lo = xlo;
      at.kv_maps = b.kv_maps + l;
      at.error = b.gemm_error;
      at.split_part = attn_split_bytes(s, b.rows_cap) ? b.attn_split : nullptr;
      at.split_tiles = kAttnSplitTiles;
      if (fz::attention_prefill_supported(s.heads, s.kv_heads, s.head_dim)) {
        at.out = nullptr;   // (the output projection reads the f16 halves only)
        FZ_CUDA(fz::launch_attention_tc(at, st, pdl));
      } else
        FZ_CUDA(fz::launch_attention(at, st, pdl));
      if ((stt = gemm(L.o, nullptr, b.x16_hi, xlo, b.y_attn, s.hidden, fz::kGemmWrite, l))) return stt;
      fz::MatvecArgs g = a;
      g.norm.hidden_in = b.hidden_b;
      g.norm.y = b.y_attn;
      g.norm.post_gain = L.post_attn_norm;
      g.norm.gain = L.ffn_norm;
      g.norm.hidden_out = b.hidden_a;
      g.norm.capture_residual = nullptr;
      g.norm.capture_added = cap ? cap + cl.layer[l].attn_added : nullptr;
      FZ_CUDA(fz::launch_norm_f16(g, b.x16_hi, xlo, st, pdl));
      if ((stt = gemm(L.gate, &L.up, b.x16_hi, xlo, nullptr, s.ffn, fz::kGemmGated, l))) return stt;
      if ((stt = gemm(L.down, nullptr, b.act16_hi, alo, b.y_mlp, s.hidden, fz::kGemmWrite, l))) return stt;
    }
  } else
  for (uint32_t l = 0; l < s.layers; l++) {
    const Layer& L = m.layers[l];
    uint32_t* lc = b.counters + (size_t)l * b.counters_per_layer;
    // QKV with the attention norm before it and QK-norm/RoPE/KV append after.
    fz::MatvecArgs a{};
    a.step = b.dstep;
    a.mat[0] = L.qkv.view();
    a.m = M;
    a.seq_tokens = T;
    a.capture_stride = cl.words;
    a.norm.hidden_in = b.hidden_a;
    a.norm.y = l ? b.y_mlp : nullptr;
    a.norm.post_gain = l ? m.layers[l - 1].post_ffw_norm : nullptr;
    a.norm.gain = L.attn_norm;
    a.norm.hidden_out = b.hidden_b;
    a.norm.eps = s.eps;
    a.norm.width = s.hidden;
    a.norm.row_of_token_stride = 1;
    a.norm.capture_residual = cap ? cap + cl.layer[l].residual : nullptr;
    a.norm.capture_added = (cap && l) ? cap + cl.layer[l - 1].mlp_added : nullptr;
    a.out = b.qkv;
    a.out_stride = L.qkv.n;
    a.rope.q_gain = L.q_norm;
    a.rope.k_gain = L.k_norm;
    a.rope.turns = L.turns;
    a.rope.eps = s.eps;
    a.rope.heads = s.heads;
    a.rope.kv_heads = s.kv_heads;
    a.rope.head_dim = s.head_dim;
    a.rope.key_cache = b.kc[l];
    a.rope.value_cache = b.vc[l];
    a.rope.slots = b.slots[l];
    a.rope.seq_stride = b.seq_stride[l];
    a.rope.query_out = b.q;
    a.rope.capture_query = cap ? cap + cl.layer[l].query : nullptr;
    a.counter = lc;
    if (M <= 4) {
      // The product's last CTA runs QK-norm, RoPE and the KV append.
      if ((stt = run_matvec(a, fz::kPrologueNorm, fz::kEpilogueQkv, st, pdl))) return stt;
    } else {
      // More rows: a warp a (row, head) in a launch of its own, not M x 6 heads in one CTA.
      if ((stt = run_matvec(a, fz::kPrologueNorm, fz::kEpilogueWrite, st, pdl))) return stt;
      FZ_CUDA(fz::launch_rope_rows(a, st, pdl));
    }
    // Attention.
    fz::AttentionArgs at{};
    at.step = b.dstep;
    at.q = b.q;
    at.key_cache = b.kc[l];
    at.value_cache = b.vc[l];
    at.seq_stride = b.seq_stride[l];
    at.slots = b.slots[l];
    at.heads = s.heads;
    at.kv_heads = s.kv_heads;
    at.head_dim = s.head_dim;
    at.window = L.window;
    at.seq_tokens = T;
    at.m = M;
    at.scale_log2e = (float)((double)(1.0f / std::sqrt((float)s.head_dim)) * 1.4426950408889634);
    at.split_keys = split_keys_for(std::min(L.window, b.context));
    at.splits = (std::min(L.window, b.context) + at.split_keys - 1) / at.split_keys;
    at.partial_o = b.partial_o;
    at.partial_ml = b.partial_ml;
    at.counters = lc + 1;
    at.out = b.attn;
    FZ_CUDA(fz::launch_attention(at, st, pdl));
    // Output projection.
    fz::MatvecArgs o{};
    o.step = b.dstep;
    o.mat[0] = L.o.view();
    o.m = M;
    o.seq_tokens = T;
    o.x = b.attn;
    o.out = b.y_attn;
    o.out_stride = s.hidden;
    if ((stt = run_matvec(o, fz::kPrologueInput, fz::kEpilogueWrite, st, pdl))) return stt;
    // Gate and up with the feed-forward norm before and GELU and edits after.
    fz::MatvecArgs g{};
    g.step = b.dstep;
    g.mat[0] = L.gate.view();
    g.mat[1] = L.up.view();
    g.m = M;
    g.seq_tokens = T;
    g.capture_stride = cl.words;
    g.norm.hidden_in = b.hidden_b;
    g.norm.y = b.y_attn;
    g.norm.post_gain = L.post_attn_norm;
    g.norm.gain = L.ffn_norm;
    g.norm.hidden_out = b.hidden_a;
    g.norm.eps = s.eps;
    g.norm.width = s.hidden;
    g.norm.row_of_token_stride = 1;
    g.norm.capture_added = cap ? cap + cl.layer[l].attn_added : nullptr;
    g.out = b.act;
    g.out_stride = s.ffn;
    g.edit.table = key.edits ? b.edit_tables : nullptr;
    g.edit.table_stride = b.table_words;
    g.edit.layer = l;
    g.edit.capture_neurons = cap ? cap + cl.layer[l].neurons : nullptr;
    if ((stt = run_matvec(g, fz::kPrologueNorm, fz::kEpilogueGated, st, pdl))) return stt;
    // Down projection.
    fz::MatvecArgs d{};
    d.step = b.dstep;
    d.mat[0] = L.down.view();
    d.m = M;
    d.seq_tokens = T;
    d.x = b.act;
    d.out = b.y_mlp;
    d.out_stride = s.hidden;
    if ((stt = run_matvec(d, fz::kPrologueInput, fz::kEpilogueWrite, st, pdl))) return stt;
    if (L.down_corr) FZ_CUDA(fz::launch_block_correction(b.act, M, s.ffn, L.down_corr, s.hidden, b.y_mlp, st));
  }
  (void)QW;
  if (key.logits) {
    fz::MatvecArgs h{};
    h.step = b.dstep;
    h.mat[0] = m.embd.view();
    h.m = b.S;
    h.seq_tokens = T;
    h.capture_stride = cl.words;
    h.norm.hidden_in = b.hidden_a;
    h.norm.y = b.y_mlp;
    h.norm.post_gain = m.layers[s.layers - 1].post_ffw_norm;
    h.norm.gain = m.output_norm;
    h.norm.hidden_out = nullptr;
    h.norm.eps = s.eps;
    h.norm.width = s.hidden;
    h.norm.row_of_token_stride = T;
    h.norm.row_of_token_offset = T - 1;
    h.norm.capture_added = cap ? cap + cl.layer[s.layers - 1].mlp_added : nullptr;
    h.out = b.logits;
    h.out_stride = s.vocab;
    h.head.argmax = b.argmax;
    if ((stt = run_head(b, h, st, pdl))) return stt;
    fz::SelectArgs se{};
    se.step = b.dstep;
    se.logits = b.logits;
    se.vocab = s.vocab;
    se.seqs = b.S;
    se.argmax = b.argmax;
    se.seeds = b.dseeds;
    se.tile_best = b.tile_best;
    se.candidates = b.candidates;
    se.records = b.records;
    FZ_CUDA(fz::launch_select(se, st, pdl));
  }
  return FZ_OK;
}

fz_status capture_graph(fz_batch& b, const GraphKey& key, cudaGraphExec_t* out);

// The step graph for `key`; a shape seen for the first time is captured for
// both host slots at once, so that a later step on the other slot finds its
// graph made.
fz_status graph_for(fz_batch& b, const GraphKey& key, cudaGraphExec_t* out) {
  auto it = b.graphs.find(key);
  if (it != b.graphs.end()) {
    *out = it->second;
    return FZ_OK;
  }
  GraphKey other = key;
  other.slot ^= 1u;
  cudaGraphExec_t unused = nullptr;
  fz_status st;
  if (!b.graphs.count(other) && (st = capture_graph(b, other, &unused))) return st;
  return capture_graph(b, key, out);
}

fz_status capture_graph(fz_batch& b, const GraphKey& key, cudaGraphExec_t* out) {
  cudaStream_t cs = b.model->dev->capture;
  FZ_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  fz_status st = enqueue_step(b, key, cs);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(cs, &graph);
  if (st) {
    if (graph) cudaGraphDestroy(graph);
    return st;
  }
  if (e != cudaSuccess) return fail(FZ_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return fail(FZ_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
  b.graphs[key] = exec;
  *out = exec;
  return FZ_OK;
}

bool direct_launch() {
  const char* v = std::getenv("FRIZZLE_B200_NO_GRAPH");
  return v && *v && *v != '0';
}

}  // namespace

// ================================================================== C ABI

extern "C" {

const char* fz_last_error(void) { return g_error.c_str(); }

fz_status fz_device_open(int ordinal, fz_device** out) {
  if (!out) return fail(FZ_ERR_ARGUMENT, "null output");
  int count = 0;
  FZ_CUDA(cudaGetDeviceCount(&count));
  if (ordinal < 0 || ordinal >= count) return fail(FZ_ERR_ARGUMENT, "no device " + std::to_string(ordinal));
  FZ_CUDA(cudaSetDevice(ordinal));
  cudaDeviceProp prop{};
  FZ_CUDA(cudaGetDeviceProperties(&prop, ordinal));
  if (prop.major != 10) return fail(FZ_ERR_NOT_SUPPORTED, std::string("not an sm_100 device: ") + prop.name);
  auto d = std::make_unique<fz_device>();
  d->ordinal = ordinal;
  FZ_CUDA(fz::configure_kernels());
  FZ_CUDA(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
  FZ_CUDA(cudaStreamCreateWithFlags(&d->capture, cudaStreamNonBlocking));
  *out = d.release();
  return FZ_OK;
}

fz_status fz_device_close(fz_device* d) {
  if (!d) return FZ_OK;
  cudaSetDevice(d->ordinal);
  cudaStreamSynchronize(d->stream);
  cudaStreamDestroy(d->stream);
  cudaStreamDestroy(d->capture);
  delete d;
  return FZ_OK;
}

void* fz_device_stream(fz_device* d) { return d ? (void*)d->stream : nullptr; }

uint64_t fz_model_index_needed(void) { return g_index_needed; }

fz_status fz_model_index_check(const void* head, uint64_t head_bytes, uint64_t file_bytes, fz_model_info* o) {
  if (!head || !o) return fail(FZ_ERR_ARGUMENT, "null argument");
  fz_model m;
  uint64_t needed = 0;
  std::string msg;
  const fz::GgufError e = fz::parse_gguf_index(static_cast<const uint8_t*>(head), head_bytes, m.index, needed, msg);
  if (e == fz::GgufError::Truncated) {
    g_index_needed = needed;
    return fail(FZ_ERR_TRUNCATED, msg);
  }
  if (e != fz::GgufError::Ok) return fail(FZ_ERR_INDEX, msg);
  uint64_t end = 0;
  for (auto& t : m.index.tensors) end = std::max(end, t.offset + t.bytes);   // (the parser refuses wraps)
  if (end > file_bytes || m.index.data_offset > file_bytes - end)
    return fail(FZ_ERR_INDEX, "tensor data runs past the end of the file");
  fz_status st;
  if ((st = describe(m))) return st;
  const Shape& s = m.shape;
  uint64_t bytes = 0;
  for (auto& t : m.index.tensors) bytes += t.bytes;
  *o = fz_model_info{s.layers, s.hidden, s.ffn, s.heads, s.kv_heads, s.head_dim, s.vocab, s.window, s.pattern,
                     s.context, s.eps, s.rope_global, s.rope_local, bytes};
  return FZ_OK;
}

fz_status fz_model_load_begin(fz_device* dev, const void* head, uint64_t head_bytes, uint64_t file_bytes,
                              fz_model** out) {
  if (!dev || !head || !out) return fail(FZ_ERR_ARGUMENT, "null argument");
  FZ_CUDA(cudaSetDevice(dev->ordinal));
  auto m = std::make_unique<fz_model>();
  m->dev = dev;
  m->file_bytes = file_bytes;
  uint64_t needed = 0;
  std::string msg;
  const fz::GgufError e =
      fz::parse_gguf_index(static_cast<const uint8_t*>(head), head_bytes, m->index, needed, msg);
  if (e == fz::GgufError::Truncated) {
    g_index_needed = needed;
    return fail(FZ_ERR_TRUNCATED, msg);
  }
  if (e != fz::GgufError::Ok) return fail(FZ_ERR_INDEX, msg);
  uint64_t end = 0;
  for (auto& t : m->index.tensors) end = std::max(end, t.offset + t.bytes);   // (the parser refuses wraps)
  if (end > file_bytes || m->index.data_offset > file_bytes - end)
    return fail(FZ_ERR_INDEX, "tensor data runs past the end of the file");
  fz_status st;
  if ((st = describe(*m)) || (st = place_model(*m))) return st;
  *out = m.release();
  return FZ_OK;
}

fz_status fz_model_load_write(fz_model* m, uint64_t offset, const void* chunk, uint64_t bytes) {
  if (!m || (!chunk && bytes)) return fail(FZ_ERR_ARGUMENT, "null argument");
  if (m->finished || !m->stage) return fail(FZ_ERR_STATE, "the load is finished");
  if (offset > m->file_bytes || bytes > m->file_bytes - offset)
    return fail(FZ_ERR_UPLOAD, "chunk past the end of the file");
  if (offset != m->cursor)
    return fail(FZ_ERR_UPLOAD, "chunks arrive in order: expected offset " + std::to_string(m->cursor) + ", got " +
                                   std::to_string(offset));
  FZ_CUDA(cudaSetDevice(m->dev->ordinal));
  const uint8_t* src = static_cast<const uint8_t*>(chunk);
  const uint64_t end = offset + bytes;
  uint64_t pos = offset;
  fz_status st;
  while (pos < end && m->next_sink < m->sinks.size()) {
    fz_model::Sink& k = m->sinks[m->next_sink];
    if (pos < k.begin) {   // bytes no sink reads (the header, padding)
      pos = std::min(end, k.begin);
      continue;
    }
    const uint64_t n = std::min(end, k.end) - pos;
    if (k.gain) {
      FZ_CUDA(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(k.gain) + (pos - k.begin), src + (pos - offset), n,
                              cudaMemcpyHostToDevice, m->dev->stream));
      pos += n;
    } else {
      for (uint64_t left = n; left;) {
        const uint64_t take = std::min(left, kLoadStage - m->stage_fill);
        FZ_CUDA(cudaMemcpyAsync(m->stage + m->stage_fill, src + (pos - offset), take, cudaMemcpyHostToDevice,
                                m->dev->stream));
        m->stage_fill += take;
        pos += take;
        left -= take;
        if ((st = drain_stage(*m, k))) return st;
      }
    }
    if (pos == k.end) {
      if ((st = finish_sink(*m, k))) return st;
      m->next_sink++;
    }
  }
  m->cursor = end;
  return FZ_OK;
}

fz_status fz_model_load_finish(fz_model* m) {
  if (!m) return fail(FZ_ERR_ARGUMENT, "null model");
  if (m->finished) return fail(FZ_ERR_STATE, "the load is finished");
  FZ_CUDA(cudaSetDevice(m->dev->ordinal));
  if (m->next_sink < m->sinks.size())
    return fail(FZ_ERR_UPLOAD, "tensor " + m->sinks[m->next_sink].name + " was not written");
  FZ_CUDA(cudaStreamSynchronize(m->dev->stream));
  FZ_CUDA(cudaFree(m->stage));
  m->stage = nullptr;
  if (m->stage_q4_0) FZ_CUDA(cudaFree(m->stage_q4_0));
  m->stage_q4_0 = nullptr;
  m->finished = true;
  return FZ_OK;
}

fz_status fz_model_info_get(const fz_model* m, fz_model_info* o) {
  if (!m || !o) return fail(FZ_ERR_ARGUMENT, "null argument");
  const Shape& s = m->shape;
  *o = fz_model_info{s.layers, s.hidden, s.ffn, s.heads, s.kv_heads, s.head_dim, s.vocab, s.window, s.pattern,
                     s.context, s.eps, s.rope_global, s.rope_local, m->weight_bytes};
  return FZ_OK;
}

fz_status fz_model_plan(const fz_model* m, fz_plan* p) {
  if (!m || !p) return fail(FZ_ERR_ARGUMENT, "null argument");
  if (!m->finished) return fail(FZ_ERR_STATE, "the model is not loaded");
  weight_bytes_of(*m, p->weight_bytes, p->copy_bytes);
  if (!p->budget) {
    // The device's free memory now: the weights and copies are already in place.
    FZ_CUDA(cudaSetDevice(m->dev->ordinal));
    size_t free_b = 0, total_b = 0;
    FZ_CUDA(cudaMemGetInfo(&free_b, &total_b));
    p->budget = free_b + p->weight_bytes + p->copy_bytes;
  }
  return plan_batch(m->shape, p->weight_bytes + p->copy_bytes, p);
}

fz_status fz_model_index_plan(const void* head, uint64_t head_bytes, uint64_t file_bytes, fz_plan* p) {
  if (!head || !p) return fail(FZ_ERR_ARGUMENT, "null argument");
  if (!p->budget) return fail(FZ_ERR_ARGUMENT, "a plan without a device needs a budget");
  fz_model m;
  uint64_t needed = 0;
  std::string msg;
  const fz::GgufError e = fz::parse_gguf_index(static_cast<const uint8_t*>(head), head_bytes, m.index, needed, msg);
  if (e == fz::GgufError::Truncated) {
    g_index_needed = needed;
    return fail(FZ_ERR_TRUNCATED, msg);
  }
  if (e != fz::GgufError::Ok) return fail(FZ_ERR_INDEX, msg);
  fz_status st;
  if ((st = describe(m))) return st;
  (void)file_bytes;
  weight_bytes_of(m, p->weight_bytes, p->copy_bytes);
  return plan_batch(m.shape, p->weight_bytes + p->copy_bytes, p);
}

fz_status fz_model_free(fz_model* m) {
  if (m) {
    cudaSetDevice(m->dev->ordinal);
    delete m;
  }
  return FZ_OK;
}

fz_status fz_batch_create(fz_model* m, uint32_t sequences, uint32_t context, uint32_t rollback, fz_batch** out) {
  if (!m || !out) return fail(FZ_ERR_ARGUMENT, "null argument");
  if (!m->finished) return fail(FZ_ERR_STATE, "the model is not loaded");
  if (sequences == 0 || sequences > (uint32_t)fz::kMaxTokens)
    return fail(FZ_ERR_NOT_SUPPORTED, "1 to 16 sequences a batch");
  if (context == 0 || context > m->shape.context) return fail(FZ_ERR_ARGUMENT, "context outside 1 .. trained context");
  FZ_CUDA(cudaSetDevice(m->dev->ordinal));
  const Shape& s = m->shape;
  auto b = std::make_unique<fz_batch>();
  b->model = m;
  b->S = sequences;
  b->context = context;
  b->rollback = rollback;
  const uint32_t M = sequences * fz::kMaxTokens;
  fz_status st;
  for (uint32_t l = 0; l < s.layers; l++) {
    const Layer& L = m->layers[l];
    // plan.cpp:335-336, rounded up to whole 32-slot chunks (the decode
    // kernel's tensor-map boxes never wrap).
    const uint32_t slots = ring_slots(L.window, context, rollback);
    const uint64_t per_seq = (uint64_t)slots * s.kv_heads * s.head_dim;
    uint16_t *k = nullptr, *v = nullptr;
    if ((st = b->alloc(&k, per_seq * sequences * 2)) || (st = b->alloc(&v, per_seq * sequences * 2))) return st;
    b->kc.push_back(k);
    b->vc.push_back(v);
    b->slots.push_back(slots);
    b->windows.push_back(L.window);
    b->seq_stride.push_back(per_seq);
    // The per-op attention splits its keys split_keys_for(keys) at a time; the decode
    // kernel into up to one split a CTA (kDecodeSplitKeys keys at least).
    const uint32_t keys = std::min(L.window, context);
    b->splits_max = std::max<uint32_t>({b->splits_max, (keys + split_keys_for(keys) - 1) / split_keys_for(keys),
                                        std::min<uint32_t>((keys + fz::kDecodeSplitKeys - 1) / fz::kDecodeSplitKeys,
                                                           fz::kDecodeMaxSplits)});
  }
  const CaptureLayout cl = capture_layout(s);
  {
    std::vector<fz::DecodeLayer> dl(s.layers);
    std::vector<fz::DecodeKvMaps> maps(s.layers);
    for (uint32_t l = 0; l < s.layers; l++) {
      const Layer& L = m->layers[l];
      fz::DecodeLayer& d = dl[l];
      d.qkv = L.qkv.view();
      d.o = L.o.view();
      d.gate = L.gate.view();
      d.up = L.up.view();
      d.down = L.down.view();
      d.down_corr = L.down_corr;
      d.attn_norm = L.attn_norm;
      d.q_norm = L.q_norm;
      d.k_norm = L.k_norm;
      d.post_attn_norm = L.post_attn_norm;
      d.ffn_norm = L.ffn_norm;
      d.post_ffw_norm = L.post_ffw_norm;
      d.turns = L.turns;
      d.key_cache = b->kc[l];
      d.value_cache = b->vc[l];
      d.seq_stride = b->seq_stride[l];
      d.slots = b->slots[l];
      d.window = L.window;
      if (s.head_dim == 256 && !fz::make_kv_maps(maps[l], d, s.kv_heads, sequences))
        return fail(FZ_ERR_CUDA, "cuTensorMapEncodeTiled refused the key/value cache maps");
    }
    const size_t R8 = (size_t)fz::kDecodeMaxRows * 8;   // rows x bytes a word
    if ((st = b->alloc(&b->norm_ll, R8 * s.hidden)) ||
        (st = b->alloc(&b->qkv_ll, R8 * (s.heads + 2 * s.kv_heads) * s.head_dim)) ||
        (st = b->alloc(&b->attn_ll, R8 * s.heads * s.head_dim)) || (st = b->alloc(&b->act_ll, R8 * s.ffn)) ||
        (st = b->alloc(&b->part_o_ll, R8 * s.heads * fz::kDecodeFoldSplits * s.head_dim)) ||
        (st = b->alloc(&b->part_ml_ll, R8 * s.heads * fz::kDecodeFoldSplits * 2)) ||
        (st = b->alloc(&b->dlayers, dl.size() * sizeof(fz::DecodeLayer))) ||
        (st = b->alloc(&b->kv_maps, maps.size() * sizeof(fz::DecodeKvMaps))))
      return st;
    if (fz::decode_supported(1, s.hidden, s.ffn, s.heads, s.kv_heads, s.head_dim))
      FZ_CUDA(fz::prepare_decode(s.hidden, s.ffn, s.heads, s.kv_heads));
    if (fz::attention_prefill_supported(s.heads, s.kv_heads, s.head_dim)) {
      FZ_CUDA(fz::configure_attention_tc());
    }
    FZ_CUDA(cudaMemcpy(b->dlayers, dl.data(), dl.size() * sizeof(fz::DecodeLayer), cudaMemcpyHostToDevice));
    FZ_CUDA(cudaMemcpy(b->kv_maps, maps.data(), maps.size() * sizeof(fz::DecodeKvMaps), cudaMemcpyHostToDevice));
  }
  b->table_words = 2 * s.layers + 5 * kMaxEdits;
  b->capture_floats = cl.words;
  const uint32_t tiles = fz::select_tiles(s.vocab);
  if ((st = b->alloc(&b->logits, (size_t)sequences * s.vocab * 4)) || (st = b->alloc(&b->argmax, (size_t)sequences * 8)) ||
      (st = b->alloc(&b->tile_best, (size_t)sequences * tiles * 64 * 8)) ||
      (st = b->alloc(&b->candidates, (size_t)sequences * 128 * 4)) || (st = b->alloc(&b->records, (size_t)sequences * 16)) ||
      (st = b->alloc(&b->dstep, sizeof(DeviceStep))) || (st = b->alloc(&b->dseeds, (size_t)sequences * 8)) ||
      (st = b->alloc(&b->gemm_error, 16)) ||
      (st = b->alloc(&b->edit_tables, (size_t)sequences * b->table_words * 4)) ||
      (st = b->alloc(&b->captures, (size_t)sequences * b->capture_floats * 4)) ||
      (st = b->alloc(&b->cap_layers, (size_t)s.layers * sizeof(fz::CaptureLayer))) ||
      (st = b->alloc(&b->ro_rows, (size_t)fz::kMaxTokens * s.hidden * 4)) ||
      (st = b->alloc(&b->ro_logits, (size_t)fz::kMaxTokens * s.vocab * 4)) ||
      (st = b->alloc(&b->ro_argmax, (size_t)fz::kMaxTokens * 8)) ||
      (st = b->alloc(&b->ro_tile_best, (size_t)fz::kMaxTokens * tiles * 64 * 8)) || (st = alloc_rows(*b, M)))
    return st;
  b->head_rows = std::max<uint32_t>(sequences, fz::kMaxTokens);
  if (m->embd_type == kTypeQ8_0 && (st = b->alloc(&b->head_x, (size_t)b->head_rows * s.hidden * 4))) return st;
  {
    std::vector<fz::CaptureLayer> v(s.layers);
    for (uint32_t l = 0; l < s.layers; l++) {
      v[l].key_cache = b->kc[l];
      v[l].seq_stride = b->seq_stride[l];
      v[l].slots = b->slots[l];
      v[l].keys = cl.layer[l].keys;
      v[l].residual = cl.layer[l].residual;
      v[l].query = cl.layer[l].query;
      v[l].weights = cl.layer[l].weights;
      v[l].stats = cl.layer[l].stats;
      v[l].readout = cl.layer[l].readout;
    }
    FZ_CUDA(cudaMemcpy(b->cap_layers, v.data(), v.size() * sizeof(fz::CaptureLayer), cudaMemcpyHostToDevice));
  }
  if (const char* v = std::getenv("FRIZZLE_B200_PASSES")) {
    const int p = std::atoi(v);
    b->passes = p == 1 ? 1u : p == 3 ? 3u : 2u;
  }
  b->has_edits.assign(sequences, false);
  for (auto& sl : b->slot) {
    FZ_CUDA(cudaMallocHost(&sl.step, sizeof(DeviceStep)));
    FZ_CUDA(cudaMallocHost(&sl.seeds, (size_t)sequences * 8));
    FZ_CUDA(cudaMallocHost(&sl.error, 16));
    FZ_CUDA(cudaMallocHost(&sl.records, (size_t)sequences * 16));
    FZ_CUDA(cudaEventCreateWithFlags(&sl.copied, cudaEventDisableTiming));
    FZ_CUDA(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
  }
  FZ_CUDA(cudaDeviceSynchronize());
  *out = b.release();
  return FZ_OK;
}

fz_status fz_batch_set_wait_limit(fz_batch* b, uint32_t microseconds) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  if (microseconds != 0 && (microseconds < 100 || microseconds > 10000000))
    return fail(FZ_ERR_ARGUMENT, "a wait limit outside 100 us .. 10 s");
  b->wait_us = microseconds;
  return FZ_OK;
}

fz_status fz_batch_time_decode(fz_batch* b, int enable) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  if (enable && !b->dk_start) {
    FZ_CUDA(cudaEventCreate(&b->dk_start));
    FZ_CUDA(cudaEventCreate(&b->dk_end));
  }
  b->time_decode = enable != 0;
  return FZ_OK;
}

fz_status fz_batch_decode_time(fz_batch* b, float* microseconds) {
  if (!b || !microseconds) return fail(FZ_ERR_ARGUMENT, "null argument");
  if (!b->time_decode) return fail(FZ_ERR_STATE, "decode timing is off (fz_batch_time_decode)");
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  float ms = 0.f;
  FZ_CUDA(cudaEventSynchronize(b->dk_end));
  FZ_CUDA(cudaEventElapsedTime(&ms, b->dk_start, b->dk_end));
  *microseconds = ms * 1000.f;
  return FZ_OK;
}

fz_status fz_batch_inject_stale_epoch(fz_batch* b, int enable) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  b->stale_epoch = enable ? 1u : 0u;
  return FZ_OK;
}

fz_status fz_batch_trace(fz_batch* b, int enable) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  FZ_CUDA(cudaStreamSynchronize(b->model->dev->stream));
  for (auto& kv : b->graphs) cudaGraphExecDestroy(kv.second);
  b->graphs.clear();
  if (b->trace) {
    cudaFree(b->trace);
    b->trace = nullptr;
  }
  if (!enable) return FZ_OK;
  int sms = 0;
  FZ_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, b->model->dev->ordinal));
  b->trace_ctas = (uint32_t)sms;
  b->trace_events = b->model->shape.layers * fz::kDecodeTracePhases * fz::kDecodeTraceStamps + fz::kDecodeTraceTail;
  const size_t bytes = (size_t)b->trace_ctas * b->trace_events * 8;
  FZ_CUDA(cudaMalloc(&b->trace, bytes));
  FZ_CUDA(cudaMemset(b->trace, 0, bytes));
  return FZ_OK;
}

fz_status fz_batch_read_trace(fz_batch* b, uint64_t* out, size_t count, uint32_t* ctas, uint32_t* events) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  if (!b->trace) return fail(FZ_ERR_STATE, "tracing is off (fz_batch_trace)");
  if (ctas) *ctas = b->trace_ctas;
  if (events) *events = b->trace_events;
  if (!out) return FZ_OK;
  const size_t n = (size_t)b->trace_ctas * b->trace_events;
  if (count < n) return fail(FZ_ERR_ARGUMENT, "the output holds fewer than ctas x events values");
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  FZ_CUDA(cudaStreamSynchronize(b->model->dev->stream));
  FZ_CUDA(cudaMemcpy(out, b->trace, n * 8, cudaMemcpyDeviceToHost));
  return FZ_OK;
}

fz_status fz_batch_free(fz_batch* b) {
  if (b) {
    cudaSetDevice(b->model->dev->ordinal);
    cudaStreamSynchronize(b->model->dev->stream);
    delete b;
  }
  return FZ_OK;
}

fz_status fz_batch_set_edits(fz_batch* b, uint32_t sequence, const uint32_t* words, size_t count) {
  if (!b || sequence >= b->S) return fail(FZ_ERR_ARGUMENT, "no such sequence");
  const Shape& s = b->model->shape;
  std::vector<uint32_t> table(b->table_words, 0u);
  if (words && count) {
    if (count > b->table_words || count < 2 * (size_t)s.layers)
      return fail(FZ_ERR_EDITS, "table size outside 2 x layers .. 2 x layers + 5 x 4096 words");
    for (uint32_t l = 0; l < s.layers; l++) {
      const uint64_t first = words[2 * l], n = words[2 * l + 1];
      if (n && (first < 2ull * s.layers || first + 5 * n > count))
        return fail(FZ_ERR_EDITS, "layer " + std::to_string(l) + "'s edits lie outside the table");
      for (uint64_t i = 0; i < n; i++) {
        const uint32_t* e = words + first + 5 * i;
        if (e[0] >= s.ffn) return fail(FZ_ERR_EDITS, "an edit's neuron is past the layer's width");
        if (e[1] > 2) return fail(FZ_ERR_EDITS, "an edit's kind is not Set, Scale or Zero");
        if (i && words[first + 5 * (i - 1)] > e[0])
          return fail(FZ_ERR_EDITS, "a layer's edits are not sorted by neuron (edit::table's order)");
      }
    }
    std::memcpy(table.data(), words, count * 4);
  }
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  FZ_CUDA(cudaStreamSynchronize(b->model->dev->stream));
  FZ_CUDA(cudaMemcpy(b->edit_tables + (size_t)sequence * b->table_words, table.data(), table.size() * 4,
                     cudaMemcpyHostToDevice));
  b->has_edits[sequence] = words && count;
  return FZ_OK;
}

fz_status fz_batch_step(fz_batch* b, const fz_step* step, const uint32_t* ids, const uint32_t* seeds) {
  if (!b || !step) return fail(FZ_ERR_ARGUMENT, "null argument");
  const Shape& s = b->model->shape;
  const uint32_t T = step->tokens;
  if (T < 1 || (uint64_t)T * b->S > (1u << 16)) return fail(FZ_ERR_NOT_SUPPORTED, "sequences x tokens above 65536");
  if (step->fed && T != 1) return fail(FZ_ERR_ARGUMENT, "a fed step is one token");
  if ((uint64_t)step->position + T > b->context) return fail(FZ_ERR_ARGUMENT, "the step runs past the context");
  if ((uint64_t)step->position + T > (1u << 24)) return fail(FZ_ERR_ARGUMENT, "position past 2^24 (interface.h:220)");
  if (!step->fed && !ids) return fail(FZ_ERR_ARGUMENT, "no token identifiers");
  if (!step->fed)
    for (uint32_t i = 0; i < T * b->S; i++)
      if (ids[i] >= s.vocab) return fail(FZ_ERR_ARGUMENT, "a token identifier past the vocabulary");
  if (step->logits && step->temperature > 0.f && step->top_k == 0) return fail(FZ_ERR_ARGUMENT, "top_k 0");
  if (step->capture && !capture_aligned(capture_layout(s)))
    return fail(FZ_ERR_NOT_SUPPORTED, "a capture layout whose vector slots are not 16-byte aligned");
  // The step's first position is the cache's length: a later one would read
  // keys nobody wrote, an earlier one rewinds the cache first (kv.h:36-44).
  if (step->position > b->length) return fail(FZ_ERR_ARGUMENT, "the step starts past the tokens the cache holds");
  if (step->position < b->length &&
      !fz_cache_truncate_keeps(b->windows.data(), b->slots.data(), s.layers, b->written, step->position)) {
    b->length = b->written = 0;
    return fail(FZ_ERR_ARGUMENT,
                "a rewind past the rollback reserve: the cache no longer holds the window before this position, "
                "and was emptied; prefill from position 0");
  }
  cudaStream_t st = b->model->dev->stream;
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  if (T * b->S > b->rows_cap) {
    uint32_t cap = 16;
    while (cap < T * b->S) cap <<= 1;
    fz_status gs;
    if ((gs = alloc_rows(*b, cap))) return gs;
    for (auto& x : b->slot) x.used = false;
  }
  auto& sl = b->slot[b->next_slot];
  if (sl.used) FZ_CUDA(cudaEventSynchronize(sl.copied));
  std::memcpy(sl.step, step, sizeof(DeviceStep));
  sl.step->padding[0] = b->serial++;   // a new epoch for the decode kernel's flag-in-data words
  sl.step->padding[1] = b->wait_us;    // its waits' limit, microseconds (0: default)
  sl.step->padding[2] = b->stale_epoch;
  sl.step->padding[3] = 0;
  if (!step->fed) std::memcpy(sl.ids, ids, (size_t)T * b->S * 4);
  for (uint32_t i = 0; i < b->S; i++) {
    sl.seeds[2 * i] = seeds ? seeds[2 * i] : step->seed[0];
    sl.seeds[2 * i + 1] = seeds ? seeds[2 * i + 1] : step->seed[1];
  }
  // (the step's first launch reads the slot's Step, ids and seeds from the
  // pinned host memory; its last writes the records and the error word back)
  bool edits = false;
  for (bool e : b->has_edits) edits = edits || e;
  const GraphKey key{T, step->logits ? 1u : 0u, step->capture ? 1u : 0u, edits ? 1u : 0u,
                     b->time_decode && T == 1 ? 1u : 0u, (uint32_t)b->next_slot};
  fz_status stt;
  if (direct_launch() || key.timed) {
    if ((stt = enqueue_step(*b, key, st))) return stt;
  } else {
    cudaGraphExec_t exec = nullptr;
    if ((stt = graph_for(*b, key, &exec))) return stt;
    FZ_CUDA(cudaGraphLaunch(exec, st));
  }
  FZ_CUDA(cudaEventRecord(sl.copied, st));   // the slot's inputs are read by now
  FZ_CUDA(cudaEventRecord(sl.done, st));
  sl.used = true;
  sl.pending = true;
  b->last_slot = b->next_slot;
  b->next_slot ^= 1;
  // KvCache::advance: the step's rows are written.
  b->length = step->position + T;
  b->written = std::max(b->written, b->length);
  return FZ_OK;
}

int fz_cache_truncate_keeps(const uint32_t* windows, const uint32_t* slots, uint32_t layers, uint32_t written,
                            uint32_t tokens) {
  if (tokens == 0) return 1;
  for (uint32_t l = 0; l < layers; l++) {
    // The next query, at `tokens`, reads back to tokens - window + 1; the
    // ring still holds back to written - slots.
    if (windows[l] <= 1) continue;
    const uint32_t oldest_held = written > slots[l] ? written - slots[l] : 0;
    const uint32_t oldest_read = tokens >= windows[l] ? tokens - windows[l] + 1 : 0;
    if (oldest_held > oldest_read) return 0;
  }
  return 1;
}

fz_status fz_batch_truncate(fz_batch* b, uint32_t tokens, uint32_t* kept) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  const uint32_t t = std::min(tokens, b->length);
  if (t > 0 && fz_cache_truncate_keeps(b->windows.data(), b->slots.data(), b->model->shape.layers, b->written, t)) {
    b->length = t;
  } else {
    b->length = b->written = 0;
  }
  if (kept) *kept = b->length;
  return FZ_OK;
}

fz_status fz_batch_cache_advance(fz_batch* b, uint32_t tokens) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  if ((uint64_t)b->length + tokens > b->context) return fail(FZ_ERR_ARGUMENT, "advance past the batch's context");
  b->length += tokens;
  b->written = std::max(b->written, b->length);
  return FZ_OK;
}

fz_status fz_batch_cache_state(fz_batch* b, uint32_t* length, uint32_t* written) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  if (length) *length = b->length;
  if (written) *written = b->written;
  return FZ_OK;
}

namespace {

// The waits a device error word names (the decode step's bits, or the
// tensor-core product's codes 1..5).
std::string wait_names(uint32_t code) {
  if (code < 0x100) return "a tensor-core product's pipeline wait";
  static const std::pair<uint32_t, const char*> bits[] = {
      {0x100u, "a phase's wait for another phase's output"}, {0x200u, "a wait for a weight tile"},
      {0x400u, "the copy issuer's wait for a free slot"}, {0x800u, "a copy's drain"},
      {0x1000u, "a weight tile out of sequence"}, {0x2000u, "a norm's staging"}};
  std::string out;
  for (const auto& b : bits)
    if (code & b.first) out += (out.empty() ? "" : ", ") + std::string(b.second);
  return out.empty() ? "an unnamed wait" : out;
}

// Waits for slot `sl`'s step and copies its records out.
fz_status settle(fz_batch* b, fz_batch::Slot& sl, fz_record* records) {
  cudaError_t e = cudaEventSynchronize(sl.done);
  if (e != cudaSuccess) {
    const bool lost = e == cudaErrorIllegalAddress || e == cudaErrorLaunchFailure || e == cudaErrorECCUncorrectable;
    return fail(lost ? FZ_ERR_DEVICE_LOST : FZ_ERR_CUDA, std::string("step: ") + cudaGetErrorString(e));
  }
  if (*sl.error) {
    const uint32_t code = *sl.error;
    FZ_CUDA(cudaMemsetAsync(b->gemm_error, 0, 4, b->model->dev->stream));
    sl.pending = false;
    return fail(FZ_ERR_CUDA, "a device wait gave up, the step was abandoned: " + wait_names(code) + " (code " +
                                 std::to_string(code) + ")");
  }
  if (records) std::memcpy(records, sl.records, (size_t)b->S * 16);
  sl.pending = false;
  return FZ_OK;
}

}  // namespace

fz_status fz_batch_wait(fz_batch* b, fz_record* records) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  if (b->last_slot < 0) return fail(FZ_ERR_STATE, "no step was run");
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  // The last step settles every earlier one.
  b->slot[b->last_slot ^ 1].pending = false;
  return settle(b, b->slot[b->last_slot], records);
}

fz_status fz_batch_wait_oldest(fz_batch* b, fz_record* records) {
  if (!b) return fail(FZ_ERR_ARGUMENT, "null batch");
  // With both slots pending the older is the one the next step reuses.
  const int i = b->slot[b->next_slot].pending ? b->next_slot : b->last_slot;
  if (i < 0 || !b->slot[i].pending) return fail(FZ_ERR_STATE, "no step to report");
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  return settle(b, b->slot[i], records);
}

fz_status fz_batch_read_logits(fz_batch* b, uint32_t sequence, float* out, size_t count) {
  if (!b || !out || sequence >= b->S) return fail(FZ_ERR_ARGUMENT, "bad argument");
  const uint32_t V = b->model->shape.vocab;
  if (count < V) return fail(FZ_ERR_ARGUMENT, "the output holds fewer than vocab floats");
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  FZ_CUDA(cudaStreamSynchronize(b->model->dev->stream));
  FZ_CUDA(cudaMemcpy(out, b->logits + (size_t)sequence * V, (size_t)V * 4, cudaMemcpyDeviceToHost));
  return FZ_OK;
}

size_t fz_capture_floats(const fz_model* m) { return m ? capture_layout(m->shape).words : 0; }

fz_status fz_capture_layout(const fz_model* m, uint32_t layer, fz_capture_slots* out) {
  if (!m || !out) return fail(FZ_ERR_ARGUMENT, "null model or output");
  if (!m->finished) return fail(FZ_ERR_STATE, "the model is not loaded");
  const Shape& s = m->shape;
  if (layer >= s.layers) return fail(FZ_ERR_ARGUMENT, "layer out of range");
  const CaptureLayout cl = capture_layout(s);
  if (cl.words > 0xFFFFFFFFull) return fail(FZ_ERR_NOT_SUPPORTED, "a capture store past 2^32 words");
  const CaptureSlot& k = cl.layer[layer];
  const auto slot = [](uint64_t first, uint64_t width) { return fz_capture_slot{(uint32_t)first, (uint32_t)width}; };
  out->neurons = slot(k.neurons, s.ffn);
  out->residual = slot(k.residual, s.hidden);
  out->attention_added = slot(k.attn_added, s.hidden);
  out->mlp_added = slot(k.mlp_added, s.hidden);
  out->query = slot(k.query, (uint64_t)s.heads * s.head_dim);
  out->weights = slot(k.weights, (uint64_t)s.heads * k.keys);
  out->stats = slot(k.stats, 2ull * s.heads);
  out->readout = slot(k.readout, kReadoutWords);
  out->keys = k.keys;
  out->query_heads = s.heads;
  out->window = k.window;
  out->full_attention = k.window >= s.context ? 1u : 0u;
  return FZ_OK;
}

fz_status fz_batch_read_capture(fz_batch* b, uint32_t sequence, float* out, size_t count) {
  if (!b || !out || sequence >= b->S) return fail(FZ_ERR_ARGUMENT, "bad argument");
  if (count < b->capture_floats) return fail(FZ_ERR_ARGUMENT, "the output holds fewer than fz_capture_floats floats");
  FZ_CUDA(cudaSetDevice(b->model->dev->ordinal));
  FZ_CUDA(cudaStreamSynchronize(b->model->dev->stream));
  FZ_CUDA(cudaMemcpy(out, b->captures + (size_t)sequence * b->capture_floats, b->capture_floats * 4,
                     cudaMemcpyDeviceToHost));
  return FZ_OK;
}

fz_status fz_batch_cache(fz_batch* b, uint32_t sequence, uint32_t layer, int values, void** ptr, uint32_t* slots) {
  if (!b || !ptr || sequence >= b->S || layer >= b->model->shape.layers) return fail(FZ_ERR_ARGUMENT, "bad argument");
  *ptr = (values ? b->vc[layer] : b->kc[layer]) + (size_t)sequence * b->seq_stride[layer];
  if (slots) *slots = b->slots[layer];
  return FZ_OK;
}

// ------------------------------------------------------------------ kernel level

size_t fz_q4_0_codes_bytes(uint32_t n, uint32_t k) { return fz::q4_codes_bytes(n, k); }
size_t fz_q4_0_scales_bytes(uint32_t n, uint32_t k) { return fz::q4_scales_bytes(n, k); }

static fz_status check_shape(uint32_t n, uint32_t k) {
  if (n == 0 || k == 0 || n % 16 || k % 64) return fail(FZ_ERR_ARGUMENT, "n must be a multiple of 16 and k of 64");
  return FZ_OK;
}

fz_status fz_q4_0_repack(const void* file_blocks, uint32_t n, uint32_t k, void* codes, void* scales, void* stream) {
  fz_status st;
  if ((st = check_shape(n, k))) return st;
  if (!file_blocks || !codes || !scales) return fail(FZ_ERR_ARGUMENT, "null pointer");
  FZ_CUDA(fz::launch_repack(static_cast<const uint8_t*>(file_blocks), n, k, static_cast<uint4*>(codes),
                            static_cast<uint2*>(scales), static_cast<cudaStream_t>(stream)));
  return FZ_OK;
}

fz_status fz_q4_0_rows(const void* codes, const void* scales, uint32_t n, uint32_t k, const uint32_t* rows,
                       uint32_t count, float scale, float* out, void* stream) {
  fz_status st;
  if ((st = check_shape(n, k))) return st;
  if (!codes || !scales || !rows || !out) return fail(FZ_ERR_ARGUMENT, "null pointer");
  const Q4Matrix mat{static_cast<const uint4*>(codes), static_cast<const uint2*>(scales), n, k};
  FZ_CUDA(fz::launch_dequant_rows(mat, rows, count, scale, out, static_cast<cudaStream_t>(stream)));
  return FZ_OK;
}

fz_status fz_q4_0_matvec(const void* codes, const void* scales, uint32_t n, uint32_t k, const float* x, uint32_t m,
                         float* y, void* stream) {
  fz_status st;
  if ((st = check_shape(n, k))) return st;
  if (!codes || !scales || !x || !y) return fail(FZ_ERR_ARGUMENT, "null pointer");
  if (m < 1 || m > (uint32_t)fz::kMaxTokens) return fail(FZ_ERR_ARGUMENT, "m outside 1 .. 16");
  fz::MatvecArgs a{};
  a.mat[0] = Q4Matrix{static_cast<const uint4*>(codes), static_cast<const uint2*>(scales), n, k};
  a.m = m;
  a.seq_tokens = m;
  a.x = x;
  a.out = y;
  a.out_stride = n;
  return run_matvec(a, fz::kPrologueInput, fz::kEpilogueWrite, static_cast<cudaStream_t>(stream), false);
}

fz_status fz_q4_0_gated(const void* gate_codes, const void* gate_scales, const void* up_codes, const void* up_scales,
                        uint32_t f, uint32_t k, const float* x, uint32_t m, const uint32_t* table, uint32_t layer,
                        uint32_t position, float* act, void* stream) {
  fz_status st;
  if ((st = check_shape(f, k))) return st;
  if (!gate_codes || !gate_scales || !up_codes || !up_scales || !x || !act) return fail(FZ_ERR_ARGUMENT, "null pointer");
  if (m < 1 || m > (uint32_t)fz::kMaxTokens) return fail(FZ_ERR_ARGUMENT, "m outside 1 .. 16");
  fz::MatvecArgs a{};
  a.mat[0] = Q4Matrix{static_cast<const uint4*>(gate_codes), static_cast<const uint2*>(gate_scales), f, k};
  a.mat[1] = Q4Matrix{static_cast<const uint4*>(up_codes), static_cast<const uint2*>(up_scales), f, k};
  a.m = m;
  a.seq_tokens = m;
  a.position = position;
  a.x = x;
  a.out = act;
  a.out_stride = f;
  a.edit.table = table;
  a.edit.layer = layer;
  return run_matvec(a, fz::kPrologueInput, fz::kEpilogueGated, static_cast<cudaStream_t>(stream), false);
}

fz_status fz_q4_0_head(const void* codes, const void* scales, uint32_t n, uint32_t k, const float* x, uint32_t m,
                       float* logits, unsigned long long* argmax, void* stream) {
  fz_status st;
  if ((st = check_shape(n, k))) return st;
  if (!codes || !scales || !x || !logits || !argmax) return fail(FZ_ERR_ARGUMENT, "null pointer");
  if (m < 1 || m > (uint32_t)fz::kMaxTokens) return fail(FZ_ERR_ARGUMENT, "m outside 1 .. 16");
  fz::MatvecArgs a{};
  a.mat[0] = Q4Matrix{static_cast<const uint4*>(codes), static_cast<const uint2*>(scales), n, k};
  a.m = m;
  a.seq_tokens = m;
  a.x = x;
  a.out = logits;
  a.out_stride = n;
  a.head.argmax = argmax;
  return run_matvec(a, fz::kPrologueInput, fz::kEpilogueHead, static_cast<cudaStream_t>(stream), false);
}

fz_status fz_q4_0_gemm(const void* codes, const void* scales, uint32_t n, uint32_t k, const void* x_hi, const void* x_lo,
                       uint32_t exact_weights, uint32_t m, float* y, uint32_t* error, void* stream) {
  fz_status st;
  if ((st = check_shape(n, k))) return st;
  if (!codes || !scales || !x_hi || !y || !error || m == 0) return fail(FZ_ERR_ARGUMENT, "null pointer or m = 0");
  fz::GemmArgs a{};
  a.w[0] = Q4Matrix{static_cast<const uint4*>(codes), static_cast<const uint2*>(scales), n, k};
  a.m = m;
  a.x_hi = static_cast<const __half*>(x_hi);
  a.x_lo = static_cast<const __half*>(x_lo);
  a.exact_w = exact_weights;
  a.out = y;
  a.out_stride = n;
  a.seq_tokens = m;
  a.error = error;
  FZ_CUDA(fz::launch_gemm(a, fz::kGemmWrite, static_cast<cudaStream_t>(stream), false));
  return FZ_OK;
}

fz_status fz_q4_0_to_f16(const void* codes, const void* scales, uint32_t n, uint32_t k, void* w_hi, void* w_lo,
                         void* stream) {
  fz_status st;
  if ((st = check_shape(n, k))) return st;
  if (!codes || !scales || !w_hi) return fail(FZ_ERR_ARGUMENT, "null pointer");
  const Q4Matrix w{static_cast<const uint4*>(codes), static_cast<const uint2*>(scales), n, k};
  FZ_CUDA(fz::launch_dequant_f16(w, static_cast<__half*>(w_hi), static_cast<__half*>(w_lo),
                                 static_cast<cudaStream_t>(stream)));
  return FZ_OK;
}

fz_status fz_f16_gemm(const void* w_hi, const void* w_lo, uint32_t n, uint32_t k, const void* x_hi, const void* x_lo,
                      uint32_t exact_weights, uint32_t m, float* y, uint32_t* error, void* stream) {
  fz_status st;
  if ((st = check_shape(n, k))) return st;
  if (!w_hi || (exact_weights && (!w_lo || !x_lo)) || !x_hi || !y || !error || m == 0)
    return fail(FZ_ERR_ARGUMENT, "null pointer or m = 0");
  fz::GemmArgs a{};
  a.w[0] = Q4Matrix{nullptr, nullptr, n, k};
  a.w_hi[0] = static_cast<const __half*>(w_hi);
  a.w_lo[0] = static_cast<const __half*>(w_lo);
  a.m = m;
  a.x_hi = static_cast<const __half*>(x_hi);
  a.x_lo = static_cast<const __half*>(x_lo);
  a.exact_w = exact_weights;
  a.out = y;
  a.out_stride = n;
  a.seq_tokens = m;
  a.error = error;
  FZ_CUDA(fz::launch_gemm(a, fz::kGemmWrite, static_cast<cudaStream_t>(stream), false));
  return FZ_OK;
}

fz_status fz_f16_gemm_gated(const void* gate_hi, const void* gate_lo, const void* up_hi, const void* up_lo, uint32_t f,
                            uint32_t k, const void* x_hi, const void* x_lo, uint32_t exact_weights, uint32_t m,
                            const uint32_t* table, uint32_t layer, uint32_t position, float* act, void* act_hi,
                            void* act_lo, uint32_t* error, void* stream) {
  fz_status st;
  if ((st = check_shape(f, k))) return st;
  if (!gate_hi || !up_hi || (exact_weights && (!gate_lo || !up_lo || !x_lo)) || !x_hi || !act_hi || !error || m == 0)
    return fail(FZ_ERR_ARGUMENT, "null pointer or m = 0");
  fz::GemmArgs a{};
  a.w[0] = Q4Matrix{nullptr, nullptr, f, k};
  a.w[1] = Q4Matrix{nullptr, nullptr, f, k};
  a.w_hi[0] = static_cast<const __half*>(gate_hi);
  a.w_lo[0] = static_cast<const __half*>(gate_lo);
  a.w_hi[1] = static_cast<const __half*>(up_hi);
  a.w_lo[1] = static_cast<const __half*>(up_lo);
  a.m = m;
  a.position = position;
  a.x_hi = static_cast<const __half*>(x_hi);
  a.x_lo = static_cast<const __half*>(x_lo);
  a.exact_w = exact_weights;
  a.out = act;
  a.out_stride = f;
  a.act_hi = static_cast<__half*>(act_hi);
  a.act_lo = static_cast<__half*>(act_lo);
  a.edit_table = table;
  a.layer = layer;
  a.seq_tokens = m;
  a.error = error;
  FZ_CUDA(fz::launch_gemm(a, fz::kGemmGated, static_cast<cudaStream_t>(stream), false));
  return FZ_OK;
}

fz_status fz_q4_0_gemm_gated(const void* gate_codes, const void* gate_scales, const void* up_codes,
                             const void* up_scales, uint32_t f, uint32_t k, const void* x_hi, const void* x_lo,
                             uint32_t exact_weights, uint32_t m, const uint32_t* table, uint32_t layer,
                             uint32_t position, float* act, void* act_hi, void* act_lo, uint32_t* error,
                             void* stream) {
  fz_status st;
  if ((st = check_shape(f, k))) return st;
  if (!gate_codes || !gate_scales || !up_codes || !up_scales || !x_hi || !act_hi || !error || m == 0)
    return fail(FZ_ERR_ARGUMENT, "null pointer or m = 0");
  fz::GemmArgs a{};
  a.w[0] = Q4Matrix{static_cast<const uint4*>(gate_codes), static_cast<const uint2*>(gate_scales), f, k};
  a.w[1] = Q4Matrix{static_cast<const uint4*>(up_codes), static_cast<const uint2*>(up_scales), f, k};
  a.m = m;
  a.position = position;
  a.x_hi = static_cast<const __half*>(x_hi);
  a.x_lo = static_cast<const __half*>(x_lo);
  a.exact_w = exact_weights;
  a.out = act;
  a.out_stride = f;
  a.act_hi = static_cast<__half*>(act_hi);
  a.act_lo = static_cast<__half*>(act_lo);
  a.edit_table = table;
  a.layer = layer;
  a.seq_tokens = m;
  a.error = error;
  FZ_CUDA(fz::launch_gemm(a, fz::kGemmGated, static_cast<cudaStream_t>(stream), false));
  return FZ_OK;
}

fz_status fz_split_f16(const float* x, size_t n, void* hi, void* lo, void* stream) {
  if (!x || !hi) return fail(FZ_ERR_ARGUMENT, "null pointer");
  FZ_CUDA(fz::launch_split_f16(x, n, static_cast<__half*>(hi), static_cast<__half*>(lo), static_cast<cudaStream_t>(stream)));
  return FZ_OK;
}

uint32_t fz_attention_splits(uint32_t window, uint32_t position, uint32_t rows) {
  const uint64_t keys = std::min<uint64_t>(window, (uint64_t)position + rows);
  return (uint32_t)((keys + kSplitKeys - 1) / kSplitKeys);
}

fz_status fz_attention(const float* q, const void* key_cache, const void* value_cache, uint32_t slots, uint32_t heads,
                       uint32_t kv_heads, uint32_t head_dim, uint32_t window, uint32_t position, uint32_t rows,
                       float* partial_o, float* partial_ml, uint32_t* counters, float* out, void* stream) {
  if (!q || !key_cache || !value_cache || !out) return fail(FZ_ERR_ARGUMENT, "null pointer");
  if (head_dim != 256) return fail(FZ_ERR_NOT_SUPPORTED, "head dimension other than 256");
  if (kv_heads == 0 || heads % kv_heads) return fail(FZ_ERR_ARGUMENT, "heads must be a multiple of kv_heads");
  const uint32_t group = heads / kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8)
    return fail(FZ_ERR_ARGUMENT, "heads per KV head must be 1, 2, 4 or 8");
  if (rows == 0 || window == 0 || slots == 0) return fail(FZ_ERR_ARGUMENT, "rows, window and slots must be nonzero");
  if ((uint64_t)position + rows > (1u << 24)) return fail(FZ_ERR_ARGUMENT, "position past 2^24");
  const uint32_t splits = fz_attention_splits(window, position, rows);
  if (splits > 1 && (!partial_o || !partial_ml || !counters))
    return fail(FZ_ERR_ARGUMENT, "more than one split needs partial and counter scratch");
  fz::AttentionArgs at{};
  at.step = nullptr;
  at.position = position;
  at.q = q;
  at.key_cache = static_cast<const uint16_t*>(key_cache);
  at.value_cache = static_cast<const uint16_t*>(value_cache);
  at.seq_stride = 0;
  at.slots = slots;
  at.heads = heads;
  at.kv_heads = kv_heads;
  at.head_dim = head_dim;
  at.window = window;
  at.seq_tokens = rows;
  at.m = rows;
  at.scale_log2e = (float)((double)(1.0f / std::sqrt((float)head_dim)) * 1.4426950408889634);
  at.split_keys = kSplitKeys;
  at.splits = splits;
  at.partial_o = partial_o;
  at.partial_ml = partial_ml;
  at.counters = counters;
  at.out = out;
  FZ_CUDA(fz::launch_attention(at, static_cast<cudaStream_t>(stream), false));
  return FZ_OK;
}

fz_status fz_attention_wide(const float* q, const void* key_cache, const void* value_cache, uint32_t slots,
                            uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t window, uint32_t position,
                            uint32_t rows, void* maps, float* split_part, uint32_t* counters, float* out,
                            uint32_t* error, void* stream) {
  if (!q || !key_cache || !value_cache || !out || !maps) return fail(FZ_ERR_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(maps) & 63u) return fail(FZ_ERR_ARGUMENT, "maps not 64-byte aligned");
  if ((reinterpret_cast<uintptr_t>(key_cache) | reinterpret_cast<uintptr_t>(value_cache)) & 15u)
    return fail(FZ_ERR_ARGUMENT, "caches not 16-byte aligned");
  if (!fz::attention_prefill_supported(heads, kv_heads, head_dim))
    return fail(FZ_ERR_ARGUMENT, "head dimension 256 and 1, 2, 4 or 8 heads per KV head only");
  if (rows == 0 || window == 0 || slots == 0) return fail(FZ_ERR_ARGUMENT, "rows, window and slots must be nonzero");
  if (slots % 32) return fail(FZ_ERR_ARGUMENT, "slots must be a multiple of 32 (whole key tiles)");
  if ((uint64_t)position + rows > (1u << 24)) return fail(FZ_ERR_ARGUMENT, "position past 2^24");
  if (split_part && !counters) return fail(FZ_ERR_ARGUMENT, "split scratch needs its counters");
  fz::DecodeLayer d{};
  d.key_cache = static_cast<uint16_t*>(const_cast<void*>(key_cache));
  d.value_cache = static_cast<uint16_t*>(const_cast<void*>(value_cache));
  d.slots = slots;
  d.seq_stride = (uint64_t)slots * kv_heads * head_dim;
  fz::DecodeKvMaps host{};
  if (!fz::make_kv_maps(host, d, kv_heads, 1)) return fail(FZ_ERR_CUDA, "cache tensor maps refused");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  FZ_CUDA(fz::configure_attention_tc());
  // (from pageable memory: the copy has taken `host` when the call returns)
  FZ_CUDA(cudaMemcpyAsync(maps, &host, sizeof(host), cudaMemcpyHostToDevice, st));
  fz::AttentionArgs at{};
  at.position = position;
  at.q = q;
  at.key_cache = d.key_cache;
  at.value_cache = d.value_cache;
  at.slots = slots;
  at.heads = heads;
  at.kv_heads = kv_heads;
  at.head_dim = head_dim;
  at.window = window;
  at.seq_tokens = rows;
  at.m = rows;
  at.scale_log2e = (float)((double)(1.0f / std::sqrt((float)head_dim)) * 1.4426950408889634);
  at.counters = counters;
  at.out = out;
  at.kv_maps = maps;
  at.error = error;
  at.split_part = split_part;
  at.split_tiles = split_part ? kAttnSplitTiles : 0u;
  FZ_CUDA(fz::launch_attention_tc(at, st, false));
  return FZ_OK;
}

}  // extern "C"
