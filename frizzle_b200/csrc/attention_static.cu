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
#include <cuda.h>
#include <cudaTypedefs.h>

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

// Device addresses of g_scratch, one per CUDA context, looked up once with
// that context current.  In host code `g_scratch` names a host-side stand-in,
// so its address must never reach a kernel.  The key is the context's unique
// ID (cuCtxGetId), not the device ordinal: a non-primary context on the same
// device, or the primary context made again after cudaDeviceReset, loads the
// module afresh at another address, and IDs are never reused in a process.
struct ContextAddress {
  unsigned long long context_id;
  StaticScratch* address;
};
constexpr int kContexts = 64;
std::mutex g_mu;
ContextAddress g_address[kContexts] = {};
int g_next = 0;

PFN_cuCtxGetCurrent_v4000 g_get_current = nullptr;
PFN_cuCtxGetId_v12000 g_get_id = nullptr;
std::once_flag g_once;

// The current context's ID, or false when the driver cannot say.
bool current_context_id(unsigned long long& id) {
  std::call_once(g_once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  CUcontext ctx = nullptr;
  return g_get_current && g_get_id && g_get_current(&ctx) == CUDA_SUCCESS && ctx && g_get_id(ctx, &id) == CUDA_SUCCESS;
}

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
  if (kv_heads == 0 || heads % kv_heads) return refuse(FZ_ERR_ARGUMENT, "heads must be a multiple of kv_heads");
  const uint32_t group = heads / kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8)
    return refuse(FZ_ERR_ARGUMENT, "heads per KV head must be 1, 2, 4 or 8");
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

  // The array's address in the current context: looked up on the first call
  // in that context (cudaGetSymbolAddress also makes the runtime's context
  // current on a thread that has none), then cached under the context's ID.
  cudaError_t e = cudaSuccess;
  unsigned long long ctx = 0;
  if (!current_context_id(ctx)) {
    // No context is current on this thread yet: a runtime call makes the
    // current device's primary context current.
    void* p = nullptr;
    (void)cudaGetSymbolAddress(&p, g_scratch);
    (void)cudaGetLastError();
    if (!current_context_id(ctx)) return refuse(FZ_ERR_CUDA, "cannot identify the current CUDA context");
  }
  StaticScratch* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    for (const ContextAddress& c : g_address)
      if (c.address && c.context_id == ctx) scratch = c.address;
    if (!scratch) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_scratch);
      if (e != cudaSuccess || !p) {
        (void)cudaGetLastError();
        return refuse(FZ_ERR_CUDA, "cudaGetSymbolAddress of the static attention scratch failed");
      }
      scratch = static_cast<StaticScratch*>(p);
      g_address[g_next] = ContextAddress{ctx, scratch};
      g_next = (g_next + 1) % kContexts;
    }
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
