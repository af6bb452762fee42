// RoPE + KV-cache write and causal GQA attention over the f32 KV cache.
#include <float.h>

#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {
using namespace yl::dev;

// The reference's separately rounded rotation (util.rs:683-690, :620-632).
__device__ __forceinline__ void rotate(float v0, float v1, float2 f, float& r0, float& r1) {
  r0 = __fsub_rn(__fmul_rn(v0, f.x), __fmul_rn(v1, f.y));
  r1 = __fadd_rn(__fmul_rn(v0, f.y), __fmul_rn(v1, f.x));
}
// Pair p of a head: (2p, 2p+1) for rope_gguf (util.rs:653-718), (p, p+hd/2)
// for rope (util.rs:589-635).
__device__ __forceinline__ void pair_index(int mode, uint32_t p, uint32_t half, uint32_t& i0, uint32_t& i1) {
  i0 = mode == 0 ? 2 * p : p;
  i1 = mode == 0 ? 2 * p + 1 : p + half;
}

// RoPE with (cos, sin) precomputed per (position, pair) on the host by the
// same formula, plus the K/V cache write, for ntok tokens (prefill path).
__global__ void __launch_bounds__(256) rope_kv_kernel(const float* __restrict__ qkv, uint32_t n_heads,
                                                      uint32_t n_kv_heads, uint32_t hd, int mode,
                                                      const float2* __restrict__ cs, const StepState* state,
                                                      uint32_t pos0, float* __restrict__ q_out,
                                                      float* __restrict__ kcache, float* __restrict__ vcache) {
  grid_dep_launch();
  grid_dep_wait();
  const uint32_t t = blockIdx.x;
  const uint32_t pos = (state ? (uint32_t)state->pos : pos0) + t;
  const uint32_t att = n_heads * hd, kvd = n_kv_heads * hd, half = hd / 2;
  const float* row = qkv + (uint64_t)t * (att + 2 * kvd);
  const float2* c = cs + (uint64_t)pos * half;
  const uint32_t npairs = (n_heads + n_kv_heads) * half;
  for (uint32_t i = threadIdx.x; i < npairs; i += blockDim.x) {
    const uint32_t h = i / half, p = i % half;
    uint32_t i0, i1;
    pair_index(mode, p, half, i0, i1);
    const float* src = row + h * hd;  // q heads then k heads are contiguous
    float r0, r1;
    rotate(src[i0], src[i1], c[p], r0, r1);
    float* dst = h < n_heads ? q_out + (uint64_t)t * att + h * hd : kcache + (uint64_t)pos * kvd + (h - n_heads) * hd;
    dst[i0] = r0;
    dst[i1] = r1;
  }
  for (uint32_t i = threadIdx.x; i < kvd; i += blockDim.x) vcache[(uint64_t)pos * kvd + i] = row[att + kvd + i];
}

cudaError_t rope_kv(const float* qkv, uint32_t ntok, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_size,
                    int rope_mode, const float2* cs, uint32_t ctx_len, const StepState* state, uint32_t pos0,
                    float* q_out, float* kcache, float* vcache, const LaunchCfg& lc) {
  (void)ctx_len;
  if (ntok == 0) return cudaSuccess;
  return launch_kernel(rope_kv_kernel, dim3(ntok), dim3(256), 0, lc, qkv, n_heads, n_kv_heads, head_size, rope_mode,
                       cs, state, pos0, q_out, kcache, vcache);
}

constexpr int AT_THREADS = 128;
constexpr int AT_TILE = 64;
constexpr int AT_MAXKV = 8;  // max query heads per KV head

template <int HD>
struct AttnSmem {
  float qs[AT_MAXKV][HD];
  float ps[AT_MAXKV][AT_TILE];
  float os[AT_MAXKV][HD];
  float ms[AT_MAXKV], ls[AT_MAXKV], cr[AT_MAXKV];
};

// Online-softmax attention of the kv_mul query heads in sm.qs over keys
// [p_begin, p_end) of one KV head: s = (q.k)*scale (forward.rs:328-346),
// exp(s - max), o = sum p*V (forward.rs:368-399), kept unnormalized in
// (sm.ms, sm.ls, sm.os). The kv_mul heads share every K/V row read.
template <int HD>
__device__ __forceinline__ void attn_tiles(AttnSmem<HD>& sm, const float* kc, const float* vc, uint32_t kv_dim,
                                           uint32_t kvh, uint32_t kv_mul, float scale, uint32_t p_begin,
                                           uint32_t p_end) {
  constexpr int E = HD / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t p0 = p_begin; p0 < p_end; p0 += AT_TILE) {
    const uint32_t tn = min((uint32_t)AT_TILE, p_end - p0);
    for (uint32_t pp = warp; pp < tn; pp += AT_THREADS / 32) {
      const float* kr = kc + (uint64_t)(p0 + pp) * kv_dim + kvh * HD + lane * E;
      float kv[E];
      if (E == 4) {
        const float4 v = *reinterpret_cast<const float4*>(kr);
        kv[0] = v.x; kv[1] = v.y; kv[2] = v.z; kv[3] = v.w;
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) kv[e] = kr[e];
      }
      for (uint32_t hh = 0; hh < kv_mul; ++hh) {
        float s = 0.0f;
#pragma unroll
        for (int e = 0; e < E; ++e) s = fmaf(sm.qs[hh][lane * E + e], kv[e], s);
        s = warp_sum(s);
        if (lane == 0) sm.ps[hh][pp] = __fmul_rn(s, scale);
      }
    }
    __syncthreads();
    for (uint32_t hh = warp; hh < kv_mul; hh += AT_THREADS / 32) {
      float mx = -INFINITY;
      for (uint32_t pp = lane; pp < tn; pp += 32) mx = fmaxf(mx, sm.ps[hh][pp]);
      mx = warp_max(mx);
      const float m_old = sm.ms[hh];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.0f;
      for (uint32_t pp = lane; pp < tn; pp += 32) {
        const float e = expf(sm.ps[hh][pp] - m_new);
        sm.ps[hh][pp] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float c = expf(m_old - m_new);
        sm.cr[hh] = c;
        sm.ls[hh] = sm.ls[hh] * c + sum;
        sm.ms[hh] = m_new;
      }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < kv_mul * HD; i += AT_THREADS) {
      const uint32_t hh = i / HD, d = i % HD;
      float o = sm.os[hh][d] * sm.cr[hh];
      const float* vr = vc + (uint64_t)p0 * kv_dim + kvh * HD + d;
      for (uint32_t pp = 0; pp < tn; ++pp) o = fmaf(sm.ps[hh][pp], vr[(uint64_t)pp * kv_dim], o);
      sm.os[hh][d] = o;
    }
    __syncthreads();
  }
}

// Writes one finished head: f32 and/or Q8_0 blocks (forward.rs:191 quantizes
// the attention output; head_size is a multiple of 32, so a head's blocks
// never straddle heads).
template <int HD>
__device__ __forceinline__ void attn_emit(float* out, int8_t* q8, float* s8, uint64_t base, const float* o_head) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int b = warp; b < HD / 32; b += AT_THREADS / 32) {
    const float v = o_head[b * 32 + lane];
    const uint64_t k = base + b * 32 + lane;
    if (out) out[k] = v;
    if (q8) {
      float sc;
      const int8_t qv = quant_q8_lane(v, &sc);
      q8[k] = qv;
      if (lane == 0) s8[k / 32] = sc;
    }
  }
}

// Prefill / general path. One CTA: KV head blockIdx.x, query token
// blockIdx.y, key split blockIdx.z (q already rotated, cache already written).
template <int HD>
__global__ void __launch_bounds__(AT_THREADS) attn_kernel(AttnArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ AttnSmem<HD> sm;
  const uint32_t kvh = blockIdx.x, t = blockIdx.y, sp = blockIdx.z;
  const uint32_t kv_mul = a.n_heads / a.n_kv_heads;
  const uint32_t pos0 = a.state ? (uint32_t)a.state->pos : a.pos0;
  const uint32_t nvis = pos0 + t + 1;  // causal: keys 0..abs_pos
  const uint32_t chunk = (nvis + a.n_splits - 1) / a.n_splits;
  const uint32_t p_begin = min(nvis, sp * chunk), p_end = min(nvis, p_begin + chunk);
  const uint32_t att = a.n_heads * HD;
  for (uint32_t i = threadIdx.x; i < kv_mul * HD; i += AT_THREADS) {
    const uint32_t hh = i / HD, d = i % HD;
    sm.qs[hh][d] = a.q[(uint64_t)t * att + (kvh * kv_mul + hh) * HD + d];
    sm.os[hh][d] = 0.0f;
  }
  if (threadIdx.x < kv_mul) {
    sm.ms[threadIdx.x] = -INFINITY;
    sm.ls[threadIdx.x] = 0.0f;
  }
  __syncthreads();
  attn_tiles<HD>(sm, a.kcache, a.vcache, a.kv_dim, kvh, kv_mul, a.scale, p_begin, p_end);
  if (a.n_splits == 1) {
    for (uint32_t hh = 0; hh < kv_mul; ++hh) {
      const float inv = sm.ls[hh] > 0.0f ? 1.0f / sm.ls[hh] : 0.0f;
      for (uint32_t d = threadIdx.x; d < HD; d += AT_THREADS) sm.os[hh][d] *= inv;
      __syncthreads();
      attn_emit<HD>(a.out, a.q8, a.s8, (uint64_t)t * att + (kvh * kv_mul + hh) * HD, sm.os[hh]);
      __syncthreads();
    }
  } else {
    for (uint32_t i = threadIdx.x; i < kv_mul * (HD + 2); i += AT_THREADS) {
      const uint32_t hh = i / (HD + 2), j = i % (HD + 2);
      const uint32_t h = kvh * kv_mul + hh;
      float* dst = a.part + (((uint64_t)t * a.n_heads + h) * a.n_splits + sp) * (HD + 2);
      dst[j] = j == 0 ? sm.ms[hh] : (j == 1 ? sm.ls[hh] : sm.os[hh][j - 2]);
    }
  }
}

// Merges the split partials of one (token, head) and emits the output.
template <int HD>
__global__ void __launch_bounds__(AT_THREADS) attn_combine_kernel(AttnArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float o[HD];
  __shared__ float wgt[64];
  __shared__ float inv_l;
  const uint32_t h = blockIdx.x, t = blockIdx.y;
  const float* base = a.part + ((uint64_t)t * a.n_heads + h) * a.n_splits * (HD + 2);
  if (threadIdx.x < 32) {
    float M = -INFINITY;
    for (uint32_t s = threadIdx.x; s < a.n_splits; s += 32) M = fmaxf(M, base[s * (HD + 2)]);
    M = warp_max(M);
    float L = 0.0f;
    for (uint32_t s = threadIdx.x; s < a.n_splits; s += 32) {
      const float m = base[s * (HD + 2)];
      const float w = m == -INFINITY ? 0.0f : expf(m - M);
      wgt[s] = w;
      L += base[s * (HD + 2) + 1] * w;
    }
    L = warp_sum(L);
    if (threadIdx.x == 0) inv_l = L > 0.0f ? 1.0f / L : 0.0f;
  }
  __syncthreads();
  for (uint32_t d = threadIdx.x; d < HD; d += AT_THREADS) {
    float acc = 0.0f;
    for (uint32_t s0 = 0; s0 < a.n_splits; s0 += 8) {  // 8 independent loads in flight
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = s0 + j < a.n_splits ? base[(s0 + j) * (HD + 2) + 2 + d] : 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (s0 + j < a.n_splits) acc = fmaf(v[j], wgt[s0 + j], acc);
    }
    o[d] = acc * inv_l;
  }
  __syncthreads();
  attn_emit<HD>(a.out, a.q8, a.s8, (uint64_t)t * a.n_heads * HD + h * HD, o);
}

cudaError_t attention(const AttnArgs& a, const LaunchCfg& lc) {
  if (a.ntok == 0) return cudaSuccess;
  const uint32_t kv_mul = a.n_heads / a.n_kv_heads;
  if (kv_mul > AT_MAXKV || a.n_splits == 0 || a.n_splits > 64) return cudaErrorInvalidValue;
  dim3 g(a.n_kv_heads, a.ntok, a.n_splits);
  cudaError_t e;
  if (a.head_size == 64) e = launch_kernel(attn_kernel<64>, g, dim3(AT_THREADS), 0, lc, a);
  else if (a.head_size == 128) e = launch_kernel(attn_kernel<128>, g, dim3(AT_THREADS), 0, lc, a);
  else return cudaErrorInvalidValue;
  if (e != cudaSuccess || a.n_splits == 1) return e;
  dim3 gc(a.n_heads, a.ntok);
  if (a.head_size == 64) return launch_kernel(attn_combine_kernel<64>, gc, dim3(AT_THREADS), 0, lc, a);
  return launch_kernel(attn_combine_kernel<128>, gc, dim3(AT_THREADS), 0, lc, a);
}

// Batch-1 decode: one CTA per (KV head, key split). RoPE of q and of the new
// key, the K/V-cache write of position `pos` (by the split that covers it),
// the split attention, and the merge + Q8_0 quantization of the output by the
// last CTA of each KV head to finish (arrival counter, reset by that CTA).
template <int HD>
__global__ void __launch_bounds__(AT_THREADS) attn_decode_kernel(AttnDecodeArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ AttnSmem<HD> sm;
  __shared__ float wgt[64];
  __shared__ int is_last;
  const uint32_t kvh = blockIdx.x, sp = blockIdx.y;
  const uint32_t kv_mul = a.n_heads / a.n_kv_heads;
  const uint32_t pos = a.state ? (uint32_t)a.state->pos : a.pos0;
  const uint32_t nvis = pos + 1;
  const uint32_t chunk = (nvis + a.n_splits - 1) / a.n_splits;
  const uint32_t p_begin = min(nvis, sp * chunk), p_end = min(nvis, p_begin + chunk);
  const uint32_t att = a.n_heads * HD, half = HD / 2;
  const float2* c = a.cs + (uint64_t)pos * half;
  for (uint32_t i = threadIdx.x; i < kv_mul * half; i += AT_THREADS) {
    const uint32_t hh = i / half, p = i % half;
    uint32_t i0, i1;
    pair_index(a.rope_mode, p, half, i0, i1);
    const float* src = a.qkv + (kvh * kv_mul + hh) * HD;
    float r0, r1;
    rotate(src[i0], src[i1], c[p], r0, r1);
    sm.qs[hh][i0] = r0;
    sm.qs[hh][i1] = r1;
  }
  for (uint32_t i = threadIdx.x; i < kv_mul * HD; i += AT_THREADS) sm.os[i / HD][i % HD] = 0.0f;
  if (threadIdx.x < kv_mul) {
    sm.ms[threadIdx.x] = -INFINITY;
    sm.ls[threadIdx.x] = 0.0f;
  }
  if (p_begin <= pos && pos < p_end) {  // this split owns the new position
    const float* ksrc = a.qkv + att + kvh * HD;
    const float* vsrc = a.qkv + att + a.kv_dim + kvh * HD;
    float* kdst = a.kcache + (uint64_t)pos * a.kv_dim + kvh * HD;
    float* vdst = a.vcache + (uint64_t)pos * a.kv_dim + kvh * HD;
    for (uint32_t p = threadIdx.x; p < half; p += AT_THREADS) {
      uint32_t i0, i1;
      pair_index(a.rope_mode, p, half, i0, i1);
      float r0, r1;
      rotate(ksrc[i0], ksrc[i1], c[p], r0, r1);
      kdst[i0] = r0;
      kdst[i1] = r1;
    }
    for (uint32_t d = threadIdx.x; d < HD; d += AT_THREADS) vdst[d] = vsrc[d];
  }
  __syncthreads();  // q in smem; this CTA's cache writes visible to its threads
  attn_tiles<HD>(sm, a.kcache, a.vcache, a.kv_dim, kvh, kv_mul, a.scale, p_begin, p_end);
  for (uint32_t i = threadIdx.x; i < kv_mul * (HD + 2); i += AT_THREADS) {
    const uint32_t hh = i / (HD + 2), j = i % (HD + 2);
    const uint32_t h = kvh * kv_mul + hh;
    float* dst = a.part + ((uint64_t)h * a.n_splits + sp) * (HD + 2);
    dst[j] = j == 0 ? sm.ms[hh] : (j == 1 ? sm.ls[hh] : sm.os[hh][j - 2]);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(a.count + kvh, 1u) == a.n_splits - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (uint32_t hh = 0; hh < kv_mul; ++hh) {
    const uint32_t h = kvh * kv_mul + hh;
    const float* base = a.part + (uint64_t)h * a.n_splits * (HD + 2);
    if (threadIdx.x < 32) {
      float M = -INFINITY;
      for (uint32_t s = threadIdx.x; s < a.n_splits; s += 32) M = fmaxf(M, __ldcg(base + s * (HD + 2)));
      M = warp_max(M);
      float L = 0.0f;
      for (uint32_t s = threadIdx.x; s < a.n_splits; s += 32) {
        const float m = __ldcg(base + s * (HD + 2));
        const float w = m == -INFINITY ? 0.0f : expf(m - M);
        wgt[s] = w;
        L += __ldcg(base + s * (HD + 2) + 1) * w;
      }
      L = warp_sum(L);
      if (threadIdx.x == 0) sm.ls[0] = L > 0.0f ? 1.0f / L : 0.0f;
    }
    __syncthreads();
    for (uint32_t d = threadIdx.x; d < HD; d += AT_THREADS) {
      float acc = 0.0f;
      for (uint32_t s0 = 0; s0 < a.n_splits; s0 += 8) {  // 8 independent L2 loads in flight
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = s0 + j < a.n_splits ? __ldcg(base + (s0 + j) * (HD + 2) + 2 + d) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (s0 + j < a.n_splits) acc = fmaf(v[j], wgt[s0 + j], acc);
      }
      sm.os[0][d] = acc * sm.ls[0];
    }
    __syncthreads();
    attn_emit<HD>(a.out, a.q8, a.s8, (uint64_t)h * HD, sm.os[0]);
    __syncthreads();
  }
  if (threadIdx.x == 0) a.count[kvh] = 0u;
}

cudaError_t attention_decode(const AttnDecodeArgs& a, const LaunchCfg& lc) {
  const uint32_t kv_mul = a.n_heads / a.n_kv_heads;
  if (kv_mul > AT_MAXKV || a.n_splits == 0 || a.n_splits > 64) return cudaErrorInvalidValue;
  dim3 g(a.n_kv_heads, a.n_splits);
  if (a.head_size == 64) return launch_kernel(attn_decode_kernel<64>, g, dim3(AT_THREADS), 0, lc, a);
  if (a.head_size == 128) return launch_kernel(attn_decode_kernel<128>, g, dim3(AT_THREADS), 0, lc, a);
  return cudaErrorInvalidValue;
}

}  // namespace k
}  // namespace yl
