// Activation-side kernels: the bit-exact Q8_0 quantizer, fused RMSNorm +
// quantize, embedding gather and the greedy argmax.
#include <float.h>

#include <algorithm>

#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {
using namespace yl::dev;

// quantization.rs:29-52, one warp per 32-element block.
__global__ void __launch_bounds__(256) quantize_q8_kernel(const float* __restrict__ x, int8_t* __restrict__ q,
                                                          float* __restrict__ s, uint64_t nblocks) {
  grid_dep_launch();
  grid_dep_wait();
  const uint64_t b = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= nblocks) return;
  float sc;
  const int8_t v = quant_q8_lane(x[b * 32 + lane], &sc);
  q[b * 32 + lane] = v;
  if (lane == 0) s[b] = sc;
}

cudaError_t quantize_q8(const float* x, int8_t* q, float* s, uint64_t nblocks, const LaunchCfg& lc) {
  if (nblocks == 0) return cudaSuccess;
  return launch_kernel(quantize_q8_kernel, dim3((unsigned)((nblocks + 7) / 8)), dim3(256), 0, lc, x, q, s, nblocks);
}

// util.rs:389-426: ss = sum x^2; ss /= n; ss += eps; ss = 1/sqrt(ss);
// y = w * (ss * x); then the Q8_0 quantizer on y (forward.rs:155-160). Every
// step is the reference's sequence of IEEE f32 operations, the sum of squares
// in its 8-lane order, so y and its Q8_0 blocks are bit-identical. CTA
// (sx, t) stages row t in shared memory, lanes 0..7 of warp 0 walk its eight
// addition chains (every CTA of the row computes the same factor), then the
// CTA's warps normalize and quantize its share sx of the row's 32-blocks: a
// few rows still fill the GPU, and no warp quantizes more than a few blocks.
__global__ void __launch_bounds__(256) rmsnorm_quant_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            uint32_t ntok, uint32_t dim, float eps,
                                                            int8_t* __restrict__ q, float* __restrict__ s,
                                                            float* __restrict__ y) {
  extern __shared__ __align__(16) float rq_stage[];  // [dim]
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float rf;
  const uint32_t t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xr = x + (uint64_t)t * dim;
  for (uint32_t i = threadIdx.x * 4; i < dim; i += 256 * 4)
    *reinterpret_cast<float4*>(rq_stage + i) = *reinterpret_cast<const float4*>(xr + i);
  __syncthreads();
  if (warp == 0) {
    const float r = rms_factor_smem8(rq_stage, dim, eps, lane);
    if (lane == 0) rf = r;
  }
  __syncthreads();
  const uint32_t nb = dim / 32;
  const uint32_t b0 = (uint32_t)((uint64_t)nb * blockIdx.x / gridDim.x);
  const uint32_t b1 = (uint32_t)((uint64_t)nb * (blockIdx.x + 1) / gridDim.x);
  for (uint32_t b = b0 + warp; b < b1; b += 8) {
    const uint32_t k = b * 32 + lane;
    const float yv = __fmul_rn(w[k], __fmul_rn(rf, rq_stage[k]));
    if (y) y[(uint64_t)t * dim + k] = yv;
    if (q) {
      float sc;
      const int8_t qv = quant_q8_lane(yv, &sc);
      q[(uint64_t)t * dim + k] = qv;
      if (lane == 0) s[(uint64_t)t * nb + b] = sc;
    }
  }
}

cudaError_t rmsnorm_quant(const float* x, const float* w, uint32_t ntok, uint32_t dim, float eps, int8_t* q,
                          float* s, float* y, const LaunchCfg& lc) {
  if (ntok == 0) return cudaSuccess;
  if (dim % 32 || ntok > 65535u) return cudaErrorInvalidValue;
  const uint32_t smem = dim * 4;
  if (smem > 227u * 1024u) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(rmsnorm_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // shares of a row: enough CTAs for the SMs when the rows are few, one warp
  // pass (8 blocks) per share at least
  const uint32_t nb = dim / 32, sms = lc.grid ? lc.grid : 148u;
  uint32_t split = (2 * sms + ntok - 1) / ntok;
  split = std::max<uint32_t>(1u, std::min<uint32_t>(split, (nb + 7) / 8));
  return launch_kernel(rmsnorm_quant_kernel, dim3(split, ntok), dim3(256), smem, lc, x, w, ntok, dim, eps, q, s,
                       y);
}

// Embedding gather: x[t][k] = value of row tokens[t], q * scale rounded once
// as the reference's dequantized table holds it (an int8 times an f16 scale
// is exact in f32; f32 scales come from lm.rs files and requantized
// safetensors), zeros for ids >= vocab (base_transformer.rs:148-158).
__global__ void __launch_bounds__(256) embed_kernel(int fmt, const uint8_t* __restrict__ wq,
                                                    const uint8_t* __restrict__ ws, uint32_t row_bytes,
                                                    uint32_t scale_row_bytes, bool sf16, uint32_t dim,
                                                    uint32_t vocab, const uint32_t* __restrict__ tokens,
                                                    const StepState* state,
                                                    float* __restrict__ x) {
  grid_dep_launch();
  grid_dep_wait();
  const uint32_t t = blockIdx.y;
  const uint32_t k = blockIdx.x * 256 + threadIdx.x;
  if (k >= dim) return;
  const uint32_t id = state ? (uint32_t)state->token : tokens[t];
  float v = 0.0f;
  if (id < vocab) {
    const uint8_t* row = wq + (uint64_t)id * row_bytes;
    if (fmt == FMT_F16) {
      v = __half2float(reinterpret_cast<const __half*>(row)[k]);
    } else {
      const uint8_t* srow = ws + (uint64_t)id * scale_row_bytes;
      const float sc = sf16 ? __half2float(reinterpret_cast<const __half*>(srow)[k / 32])
                            : reinterpret_cast<const float*>(srow)[k / 32];
      int qv;
      if (fmt == FMT_Q8) {
        qv = (int8_t)row[k];
      } else {
        const uint32_t j = k & 31;
        const uint8_t byte = row[(k / 32) * 16 + (j & 15)];
        qv = (int)(j < 16 ? (byte & 0xF) : (byte >> 4)) - 8;
      }
      v = __fmul_rn((float)qv, sc);
    }
  }
  x[(uint64_t)t * dim + k] = v;
}

cudaError_t embed(int fmt, const uint8_t* wq, const uint8_t* ws, uint32_t row_bytes, uint32_t scale_row_bytes,
                  bool sf16, uint32_t dim, uint32_t vocab, const uint32_t* tokens, const StepState* state, uint32_t ntok,
                  float* x, const LaunchCfg& lc) {
  if (ntok == 0) return cudaSuccess;
  return launch_kernel(embed_kernel, dim3((dim + 255) / 256, ntok), dim3(256), 0, lc, fmt, wq, ws, row_bytes,
                       scale_row_bytes, sf16, dim, vocab, tokens, state, x);
}

// sampler.rs:67-79: index of the first strictly-greatest value. NaNs never
// win; if logits[0] is NaN the reference returns 0 (nothing compares greater).
__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, uint32_t n,
                                                      uint32_t* __restrict__ out, StepState* state) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  for (uint32_t i = threadIdx.x; i < n; i += 1024) {
    const float v = logits[i];
    if (v == v && better(v, i, bv, bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(FULL, bv, o);
    const uint32_t oi = __shfl_xor_sync(FULL, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bv = sv[lane];
    bi = si[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(FULL, bv, o);
      const uint32_t oi = __shfl_xor_sync(FULL, bi, o);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) {
      uint32_t r = bi == 0xFFFFFFFFu ? 0u : bi;
      if (logits[0] != logits[0]) r = 0;
      if (out) out[state ? state->steps : 0] = r;
      if (state) {
        state->next = (int32_t)r;
        state->token = (int32_t)r;
        state->pos += 1;
        state->steps += 1;
      }
    }
  }
}

cudaError_t argmax(const float* logits, uint32_t n, uint32_t* out, StepState* state, const LaunchCfg& lc) {
  return launch_kernel(argmax_kernel, dim3(1), dim3(1024), 0, lc, logits, n, out, state);
}

// The token and position travel as launch arguments, so back-to-back calls
// that enqueue without synchronizing each start from their own values.
__global__ void set_step_state_kernel(StepState* state, int32_t pos, int32_t token) {
  grid_dep_wait();
  state->pos = pos;
  state->token = token;
  state->next = 0;
  state->steps = 0;
}

cudaError_t set_step_state(StepState* state, int32_t pos, int32_t token, const LaunchCfg& lc) {
  return launch_kernel(set_step_state_kernel, dim3(1), dim3(1), 0, lc, state, pos, token);
}

}  // namespace k
}  // namespace yl
