// RoPE + KV-cache write and causal GQA attention over the f32 KV cache.
#include <float.h>

#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {
using namespace yl::dev;

// util.rs:653-718 (`rope_gguf`: pairs 2p, 2p+1) or util.rs:589-635 (`rope`:
// pairs p, p+hd/2), with (cos, sin) precomputed per (position, pair) on the
// host by the same formula. The rotation is the reference's separately
// rounded v0*c - v1*s, v0*s + v1*c. V rows are copied into the cache.
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
    const uint32_t i0 = mode == 0 ? 2 * p : p, i1 = mode == 0 ? 2 * p + 1 : p + half;
    const float2 f = c[p];
    const float* src = row + h * hd;  // q heads then k heads are contiguous
    const float v0 = src[i0], v1 = src[i1];
    const float r0 = __fsub_rn(__fmul_rn(v0, f.x), __fmul_rn(v1, f.y));
    const float r1 = __fadd_rn(__fmul_rn(v0, f.y), __fmul_rn(v1, f.x));
    if (h < n_heads) {
      float* dq = q_out + (uint64_t)t * att + h * hd;
      dq[i0] = r0;
      dq[i1] = r1;
    } else {
      float* dk = kcache + (uint64_t)pos * kvd + (h - n_heads) * hd;
      dk[i0] = r0;
      dk[i1] = r1;
    }
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

// Writes the finished head outputs: f32 and/or Q8_0 blocks (forward.rs:191
// quantizes the attention output; head_size is a multiple of 32, so the blocks
// of one head never straddle heads).
template <int HD>
__device__ __forceinline__ void attn_emit(const AttnArgs& a, uint32_t t, uint32_t h, const float* o_head) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t att = a.n_heads * HD;
  for (int b = warp; b < HD / 32; b += AT_THREADS / 32) {
    const float v = o_head[b * 32 + lane];
    const uint64_t k = (uint64_t)t * att + h * HD + b * 32 + lane;
    if (a.out) a.out[k] = v;
    if (a.q8) {
      float sc;
      const int8_t qv = quant_q8_lane(v, &sc);
      a.q8[k] = qv;
      if (lane == 0) a.s8[k / 32] = sc;
    }
  }
}

// One CTA: KV head blockIdx.x, query token blockIdx.y, key split blockIdx.z.
// Flash-decoding style online softmax over tiles of AT_TILE positions; the
// kv_mul query heads sharing the KV head reuse every K/V row read.
template <int HD>
__global__ void __launch_bounds__(AT_THREADS) attn_kernel(AttnArgs a) {
  grid_dep_launch();
  grid_dep_wait();
  constexpr int E = HD / 32;  // elements per lane of a K row
  __shared__ float qs[AT_MAXKV][HD];
  __shared__ float ps[AT_MAXKV][AT_TILE];
  __shared__ float os[AT_MAXKV][HD];
  __shared__ float ms[AT_MAXKV], ls[AT_MAXKV], cr[AT_MAXKV];
  const uint32_t kvh = blockIdx.x, t = blockIdx.y, sp = blockIdx.z;
  const uint32_t kv_mul = a.n_heads / a.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t pos0 = a.state ? (uint32_t)a.state->pos : a.pos0;
  const uint32_t nvis = pos0 + t + 1;  // causal: keys 0..abs_pos
  const uint32_t chunk = (nvis + a.n_splits - 1) / a.n_splits;
  const uint32_t p_begin = min(nvis, sp * chunk), p_end = min(nvis, p_begin + chunk);
  const uint32_t att = a.n_heads * HD;

  for (uint32_t i = threadIdx.x; i < kv_mul * HD; i += AT_THREADS) {
    const uint32_t hh = i / HD, d = i % HD;
    qs[hh][d] = a.q[(uint64_t)t * att + (kvh * kv_mul + hh) * HD + d];
    os[hh][d] = 0.0f;
  }
  if (threadIdx.x < kv_mul) {
    ms[threadIdx.x] = -INFINITY;
    ls[threadIdx.x] = 0.0f;
  }
  __syncthreads();

  for (uint32_t p0 = p_begin; p0 < p_end; p0 += AT_TILE) {
    const uint32_t tn = min((uint32_t)AT_TILE, p_end - p0);
    // scores: s = (q . k) * scale (forward.rs:328-346)
    for (uint32_t pp = warp; pp < tn; pp += AT_THREADS / 32) {
      const float* kr = a.kcache + (uint64_t)(p0 + pp) * a.kv_dim + kvh * HD + lane * E;
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
        for (int e = 0; e < E; ++e) s = fmaf(qs[hh][lane * E + e], kv[e], s);
        s = warp_sum(s);
        if (lane == 0) ps[hh][pp] = __fmul_rn(s, a.scale);
      }
    }
    __syncthreads();
    // online softmax update per query head
    for (uint32_t hh = warp; hh < kv_mul; hh += AT_THREADS / 32) {
      float mx = -INFINITY;
      for (uint32_t pp = lane; pp < tn; pp += 32) mx = fmaxf(mx, ps[hh][pp]);
      mx = warp_max(mx);
      const float m_old = ms[hh];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.0f;
      for (uint32_t pp = lane; pp < tn; pp += 32) {
        const float e = expf(ps[hh][pp] - m_new);
        ps[hh][pp] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float c = expf(m_old - m_new);
        cr[hh] = c;
        ls[hh] = ls[hh] * c + sum;
        ms[hh] = m_new;
      }
    }
    __syncthreads();
    // o = o * corr + sum_p p * V[p] (forward.rs:368-399)
    for (uint32_t i = threadIdx.x; i < kv_mul * HD; i += AT_THREADS) {
      const uint32_t hh = i / HD, d = i % HD;
      float o = os[hh][d] * cr[hh];
      const float* vr = a.vcache + (uint64_t)p0 * a.kv_dim + kvh * HD + d;
      for (uint32_t pp = 0; pp < tn; ++pp) o = fmaf(ps[hh][pp], vr[(uint64_t)pp * a.kv_dim], o);
      os[hh][d] = o;
    }
    __syncthreads();
  }

  if (a.n_splits == 1) {
    for (uint32_t hh = 0; hh < kv_mul; ++hh) {
      const float inv = ls[hh] > 0.0f ? 1.0f / ls[hh] : 0.0f;
      for (uint32_t d = threadIdx.x; d < HD; d += AT_THREADS) os[hh][d] *= inv;
      __syncthreads();
      attn_emit<HD>(a, t, kvh * kv_mul + hh, os[hh]);
      __syncthreads();
    }
  } else {
    for (uint32_t i = threadIdx.x; i < kv_mul * (HD + 2); i += AT_THREADS) {
      const uint32_t hh = i / (HD + 2), j = i % (HD + 2);
      const uint32_t h = kvh * kv_mul + hh;
      float* dst = a.part + (((uint64_t)t * a.n_heads + h) * a.n_splits + sp) * (HD + 2);
      dst[j] = j == 0 ? ms[hh] : (j == 1 ? ls[hh] : os[hh][j - 2]);
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
    for (uint32_t s = 0; s < a.n_splits; ++s) acc = fmaf(base[s * (HD + 2) + 2 + d], wgt[s], acc);
    o[d] = acc * inv_l;
  }
  __syncthreads();
  attn_emit<HD>(a, t, h, o);
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

}  // namespace k
}  // namespace yl
