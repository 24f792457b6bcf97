// fz_attention_static: the attention entry point for callers that cannot
// allocate device memory.
//
// Some hosts of this library own no allocator on the device: a runtime that
// hands out only pre-registered buffers, a process whose memory pool is fixed
// before it loads plugins, or a caller that must not call cudaMalloc because
// it is recording a sequence of work that has to stay free of allocation and
// synchronisation.  fz_attention needs scratch for the partial results of
// key splits; this variant keeps that scratch in a static device array that
// every GPU loading the library holds until the process exits, so the caller
// passes only its inputs and outputs.
#include <mutex>

#include "frizzle_b200.h"
#include "kernels.cuh"
#include "last_error.h"

namespace {

constexpr uint32_t kStaticPartials = FZ_ATTENTION_STATIC_MAX_PARTIALS;  // rows x heads x splits
constexpr uint32_t kStaticCounters = FZ_ATTENTION_STATIC_MAX_COUNTERS;  // rows x kv_heads
constexpr uint32_t kHeadDim = 256;
constexpr uint32_t kSplitKeys = 512;

// The scratch: partial outputs, their (max, sum) pairs, and the split
// counters.  2 MiB + 16 KiB + 512 B on every device that loads the library.
struct StaticScratch {
  float partial_o[kStaticPartials * kHeadDim];
  float partial_ml[kStaticPartials * 2];
  uint32_t counters[kStaticCounters];
};
static __device__ __align__(256) StaticScratch g_scratch;

// Device addresses of g_scratch, one per device, looked up once with that
// device current.  In host code `g_scratch` names a host-side stand-in, so its
// address must never reach a kernel.
std::mutex g_mu;
StaticScratch* g_address[64] = {};

fz_status refuse(fz_status s, const char* why) {
  fz::set_last_error(why);
  return s;
}

}  // namespace

extern "C" fz_status fz_attention_static(const float* q, const void* key_cache, const void* value_cache, uint32_t slots,
                                         uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t window,
                                         uint32_t position, uint32_t rows, float* out, void* stream) {
  if (!q || !key_cache || !value_cache || !out) return refuse(FZ_ERR_ARGUMENT, "null pointer");
  if (head_dim != kHeadDim) return refuse(FZ_ERR_NOT_SUPPORTED, "head dimension other than 256");
  if (kv_heads == 0 || heads % kv_heads || heads / kv_heads > 8) return refuse(FZ_ERR_ARGUMENT, "heads per KV head 1..8");
  if (rows == 0 || window == 0 || slots == 0) return refuse(FZ_ERR_ARGUMENT, "rows, window and slots must be nonzero");
  if ((uint64_t)position + rows > (1u << 24)) return refuse(FZ_ERR_ARGUMENT, "position past 2^24");
  const uint64_t keys = (uint64_t)window < (uint64_t)position + rows ? window : (uint64_t)position + rows;
  const uint64_t splits = (keys + kSplitKeys - 1) / kSplitKeys;
  if ((uint64_t)rows * heads * splits > kStaticPartials)
    return refuse(FZ_ERR_ARGUMENT,
                  "rows x heads x key splits exceeds the static scratch (FZ_ATTENTION_STATIC_MAX_PARTIALS); "
                  "use fz_attention with caller scratch");
  if ((uint64_t)rows * kv_heads > kStaticCounters)
    return refuse(FZ_ERR_ARGUMENT, "rows x kv_heads exceeds FZ_ATTENTION_STATIC_MAX_COUNTERS");

  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess || device < 0 || device >= 64) return refuse(FZ_ERR_CUDA, "cudaGetDevice failed");
  StaticScratch* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_address[device]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_scratch);
      if (e != cudaSuccess || !p) {
        (void)cudaGetLastError();
        return refuse(FZ_ERR_CUDA, "cudaGetSymbolAddress of the static attention scratch failed");
      }
      g_address[device] = static_cast<StaticScratch*>(p);
    }
    scratch = g_address[device];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The split counters must start at zero; the previous call left them at
  // zero, but a call that never finished might not have.
  e = cudaMemsetAsync(scratch->counters, 0, (size_t)rows * kv_heads * sizeof(uint32_t), s);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return refuse(FZ_ERR_CUDA, "clearing the static split counters failed");
  }
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
  at.scale_log2e = (float)((double)(1.0f / sqrtf((float)head_dim)) * 1.4426950408889634);
  at.split_keys = kSplitKeys;
  at.splits = (uint32_t)splits;
  at.partial_o = scratch->partial_o;
  at.partial_ml = scratch->partial_ml;
  at.counters = scratch->counters;
  at.out = out;
  e = fz::launch_attention(at, s, false);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return refuse(FZ_ERR_CUDA, cudaGetErrorString(e));
  }
  return FZ_OK;
}
