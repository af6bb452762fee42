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
#include <string>

#include "../host/common.h"
#include "kernels.h"

namespace {

// The weights row of every (query row, head): batch * n_heads rows of
// seq_len floats (attention_scratch_floats).
constexpr size_t kStaticBytes = YL_ATTN_STATIC_BYTES;
static_assert(kStaticBytes % 256 == 0, "the static partials area is a whole number of 256-byte lines");
static __device__ __align__(256) float g_attn_scratch[kStaticBytes / sizeof(float)];

// Host code must not pass g_attn_scratch itself to a kernel: on the host it
// names a stand-in, not the device address. The device address is resolved
// on every call with the caller's device current (cudaGetSymbolAddress does
// not allocate), so a call made after cudaDeviceReset, which reloads the
// module at a new address, still gets the live array. The first call on a
// device also loads the module there, which is why it should come before
// any stream capture.
int scratch_for_current_device(float** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
  if (e != cudaSuccess || p == nullptr)
    return yl::fail(YL_ERR_CUDA, std::string("cudaGetSymbolAddress(static attention scratch): ") +
                                     cudaGetErrorString(e));
  *out = static_cast<float*>(p);
  return YL_OK;
}

}  // namespace

extern "C" int yl_fused_attention_static(float* output, const float* sq, const float* key_cache,
                                         const float* value_cache, uint64_t seq_len, uint64_t batch, uint64_t n_heads,
                                         uint64_t n_kv_heads, uint64_t head_size, uint32_t start_pos, uint64_t kv_dim,
                                         float attn_scale, void* stream) {
  int rc = yl::check_attention_args(output, sq, key_cache, value_cache, seq_len, batch, n_heads, n_kv_heads,
                                    head_size, start_pos, kv_dim);
  if (rc) return rc;
  // the same kernel and scratch layout as yl_fused_attention, so both give
  // the same result
  const uint64_t need =
      yl::k::attention_scratch_floats((uint32_t)batch, (uint32_t)n_heads, start_pos) * sizeof(float);
  if (need > kStaticBytes)
    return yl::fail(YL_ERR_UNSUPPORTED, "attention needs " + std::to_string(need) +
                                            " bytes of scratch; the static area holds " +
                                            std::to_string(kStaticBytes));
  float* scratch = nullptr;
  if ((rc = scratch_for_current_device(&scratch))) return rc;
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
  a.n_splits = 1;
  // Every weight the kernel reads is written by the same call first, so
  // nothing in the array needs clearing between calls.
  a.part = scratch;
  a.out = output;
  yl::k::LaunchCfg lc;
  lc.stream = (cudaStream_t)stream;
  cudaError_t e = yl::k::attention(a, lc);
  if (e != cudaSuccess) return yl::fail(YL_ERR_CUDA, std::string("attention launch: ") + cudaGetErrorString(e));
  return YL_OK;
}
