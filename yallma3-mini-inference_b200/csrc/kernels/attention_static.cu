// yl_fused_attention_static: the single-token split attention of
// yl_fused_attention with its split partials in a fixed, file-scope device
// array instead of a per-call workspace, so the call allocates nothing.
//
// Who needs it: callers that cannot call cudaMalloc / cudaMallocAsync on the
// path that runs attention -- for example an engine whose memory manager owns
// all device memory up front, or a latency-critical loop that must not hit
// the allocator's implicit synchronization or its out-of-memory failures.
//
// The array belongs to this library's module: every GPU that loads the
// library holds it (YL_ATTN_STATIC_BYTES) until the process exits. All calls
// share it and it keeps the last call's contents.
#include <mutex>
#include <string>

#include "../host/common.h"
#include "kernels.h"

namespace {

// One slot of (max, sum, head_size values) per (query head, key split).
constexpr size_t kStaticBytes = 1u << 20;  // YL_ATTN_STATIC_BYTES
static __device__ __align__(256) float g_attn_scratch[kStaticBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Host code must not pass g_attn_scratch itself to a kernel: on the host it
// names a stand-in, not the device address. Resolve the device address once
// per device, with that device current.
int scratch_for_current_device(float** out) {
  int dev = 0;
  YL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return yl::fail(YL_ERR_UNSUPPORTED, "device index beyond the static table");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || p == nullptr)
      return yl::fail(YL_ERR_CUDA, std::string("cudaGetSymbolAddress(static attention scratch): ") +
                                       cudaGetErrorString(e));
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return YL_OK;
}

}  // namespace

extern "C" int yl_fused_attention_static(float* output, const float* sq, const float* key_cache,
                                         const float* value_cache, uint64_t seq_len, uint64_t batch, uint64_t n_heads,
                                         uint64_t n_kv_heads, uint64_t head_size, uint32_t start_pos, uint64_t kv_dim,
                                         float attn_scale, void* stream) {
  if (!output || !sq || !key_cache || !value_cache) return yl::fail(YL_ERR_ARG, "null pointer");
  if (batch == 0) return yl::fail(YL_ERR_ARG, "empty batch");
  if (head_size != 64 && head_size != 128) return yl::fail(YL_ERR_UNSUPPORTED, "head_size must be 64 or 128");
  if (n_kv_heads == 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > 8)
    return yl::fail(YL_ERR_UNSUPPORTED, "n_heads must be a multiple (at most 8x) of n_kv_heads");
  if (kv_dim < n_kv_heads * head_size) return yl::fail(YL_ERR_ARG, "kv_dim smaller than n_kv_heads * head_size");
  if ((uint64_t)start_pos + batch > seq_len) return yl::fail(YL_ERR_RANGE, "start_pos + batch exceeds seq_len");
  if (((uintptr_t)key_cache | (uintptr_t)value_cache) % 16 || kv_dim % 4)
    return yl::fail(YL_ERR_ARG, "caches must be 16-byte aligned");
  // same split count as yl_fused_attention, so both give the same result
  int dev = 0, sms = 148;
  YL_CUDA_TRY(cudaGetDevice(&dev));
  YL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  uint64_t ns = 1;
  if (batch == 1) {
    ns = (2 * (uint64_t)sms + n_kv_heads - 1) / n_kv_heads;
    ns = ns < 64 ? ns : 64;
    ns = ns < seq_len ? ns : seq_len;
    ns = ns > 0 ? ns : 1;
  }
  const uint64_t need = n_heads * ns * (head_size + 2) * sizeof(float);
  if (ns > 1 && need > kStaticBytes)
    return yl::fail(YL_ERR_UNSUPPORTED, "attention needs " + std::to_string(need) +
                                            " bytes of split scratch; the static area holds " +
                                            std::to_string(kStaticBytes));
  float* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  yl::k::AttnArgs a{};
  a.q = sq;
  a.kcache = key_cache;
  a.vcache = value_cache;
  a.ntok = (uint32_t)batch;
  a.n_heads = (uint32_t)n_heads;
  a.n_kv_heads = (uint32_t)n_kv_heads;
  a.head_size = (uint32_t)head_size;
  a.kv_dim = (uint32_t)kv_dim;
  a.pos0 = start_pos;
  a.scale = attn_scale;
  a.n_splits = (uint32_t)ns;
  // Every partial slot the merge reads is written by the same call first, so
  // nothing in the array needs clearing between calls.
  a.part = scratch;
  a.out = output;
  yl::k::LaunchCfg lc;
  lc.stream = (cudaStream_t)stream;
  cudaError_t e = yl::k::attention(a, lc);
  if (e != cudaSuccess) return yl::fail(YL_ERR_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
  return YL_OK;
}
