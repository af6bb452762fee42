// Tensor-parallel exchange steps over NVLink peer memory (Megatron split of
// the reference's forward.rs:154-279 across ranks): the row-parallel wo and
// down projections produce per-rank partial sums that are all-reduced and
// added to the replicated residual stream; the vocabulary-parallel lm_head
// publishes per-rank winners that are combined into the greedy id.
//
// One-shot protocol per exchange site: after the producing kernel completed
// (programmatic-launch wait), thread r of CTA 0 stores the step's epoch into
// rank r's flag[site][me] with release semantics at system scope; every CTA
// then waits (bounded) until its own flag[site][*] all reach the epoch and
// reads the peers' data directly over NVLink. Partials alternate between two
// buffers (even / odd sites), which a rank can only overwrite after every
// peer has signalled the site in between, i.e. finished reading.
#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {
using namespace yl::dev;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Signals this rank's arrival at the site to every rank (CTA 0), then waits
// until all ranks arrived. Returns false (error flag set) on timeout.
__device__ bool tp_sync(const TpArgs& t, uint32_t e) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x < t.world) {
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(t.base[threadIdx.x] + t.flags_off) + t.site * t.world + t.rank;
    st_release_sys(f, e);
  }
  if (threadIdx.x < t.world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(t.base[t.rank] + t.flags_off) + t.site * t.world + threadIdx.x;
    const uint64_t t0 = clock64();
    uint32_t it = 0;
    // wrap-safe: epochs increase by one per step
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if ((++it & 255u) == 0 && (uint64_t)(clock64() - t0) > 4000000000ull) {
        if (t.err) atomicExch(t.err, ERR_WAIT_TIMEOUT);
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(256) tp_allreduce_add_kernel(TpArgs t, uint64_t part_off, uint32_t n, float* x) {
  grid_dep_launch();
  grid_dep_wait();
  const uint32_t e = *t.epoch + 1;
  if (!tp_sync(t, e)) return;
  const float* p[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) p[r] = reinterpret_cast<const float*>(t.base[r < (int)t.world ? r : 0] + part_off);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float v[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) v[r] = r < (int)t.world ? __ldcv(p[r] + i) : 0.0f;
    float s = v[0];
#pragma unroll
    for (int r = 1; r < 8; ++r)
      if (r < (int)t.world) s = __fadd_rn(s, v[r]);
    x[i] = __fadd_rn(x[i], s);
  }
}

__global__ void __launch_bounds__(256) tp_argmax_kernel(TpArgs t, uint64_t lm_off, uint64_t logit_off, uint32_t vl,
                                                       float* logits, uint32_t* hist, StepState* state, uint32_t* epoch,
                                                       uint32_t* pepoch) {
  grid_dep_launch();
  grid_dep_wait();
  const uint32_t e = *t.epoch + 1;
  if (!tp_sync(t, e)) return;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu, nan0 = 0;
    if (lane < (int)t.world) {
      const uint32_t* slot = reinterpret_cast<const uint32_t*>(t.base[lane] + lm_off);
      bv = __uint_as_float(__ldcv(slot));
      bi = __ldcv(slot + 1);
      nan0 = lane == 0 ? __ldcv(slot + 2) : 0u;
      if (bi == 0xFFFFFFFFu) bv = -INFINITY;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {  // max value, lowest index among equals (sampler.rs:67-79)
      const float ov = __shfl_xor_sync(FULL, bv, o);
      const uint32_t oi = __shfl_xor_sync(FULL, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    nan0 = __shfl_sync(FULL, nan0, 0);
    if (lane == 0) {
      uint32_t res = bi == 0xFFFFFFFFu ? 0u : bi;
      if (nan0) res = 0;  // a NaN first logit is never beaten
      hist[state ? state->steps : 0] = res;
      if (state) {
        state->next = (int32_t)res;
        state->token = (int32_t)res;
        state->pos += 1;
        state->steps += 1;
      }
    }
  }
  if (logits) {
    for (uint32_t r = 0; r < t.world; ++r) {
      const float* src = reinterpret_cast<const float*>(t.base[r] + logit_off);
      for (uint32_t i = threadIdx.x; i < vl; i += blockDim.x) logits[(uint64_t)r * vl + i] = __ldcv(src + i);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *epoch = e;  // the step's collectives are done
    if (pepoch) *pepoch += 1;
  }
}

cudaError_t tp_allreduce_add(const TpArgs& t, uint64_t part_off, uint32_t n, float* x, const LaunchCfg& lc) {
  if (t.world < 2 || t.world > 8 || t.rank >= t.world) return cudaErrorInvalidValue;
  const uint32_t grid = std::min<uint32_t>(32u, (n + 255) / 256);
  return launch_kernel(tp_allreduce_add_kernel, dim3(grid), dim3(256), 0, lc, t, part_off, n, x);
}

cudaError_t tp_argmax(const TpArgs& t, uint64_t lm_off, uint64_t logit_off, uint32_t vl, float* logits,
                      uint32_t* hist, StepState* state, uint32_t* epoch, uint32_t* pepoch, const LaunchCfg& lc) {
  if (t.world < 2 || t.world > 8 || t.rank >= t.world) return cudaErrorInvalidValue;
  return launch_kernel(tp_argmax_kernel, dim3(1), dim3(256), 0, lc, t, lm_off, logit_off, vl, logits, hist, state,
                       epoch, pepoch);
}

}  // namespace k
}  // namespace yl
