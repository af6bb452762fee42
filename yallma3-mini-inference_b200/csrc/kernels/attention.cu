// RoPE + KV-cache write and causal GQA attention over the f32 KV cache.
#include <cooperative_groups.h>
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
  if (a.n_splits == 1 && a.ntok >= 32 && attention_prefill_ok(a)) return attention_prefill(a, lc);
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

// ---------------------------------------------------------------------------
// Batch-1 decode, built for latency (the KV bytes of one decode step are a few
// MB; the cost is the dependent chain). One cluster of n_splits CTAs per KV
// head; CTA `rank` of the cluster takes the rank-th slice of the keys:
//  * the slice's K and V rows are fetched with cp.async in one round trip
//    (before the wait on the preceding kernel when early_kv is set), while q
//    (and, in the CTA owning position `pos`, the new key and value rows) is
//    read from the fused projection output and rotated (RoPE);
//  * the owner writes the new K/V rows to the cache and into its tile;
//  * each warp runs attention over its positions in registers (see the
//    kernel), the CTA combines its eight warp partials;
//  * every CTA pushes its (max, sum, unnormalized output) partial of each
//    32-block of the KV head's output into the CTA that merges that block
//    (distributed shared memory); after one cluster barrier each CTA merges
//    and quantizes its blocks from its own shared memory.
namespace cg = cooperative_groups;
constexpr int AD_TILE = 64;      // positions per shared-memory tile
constexpr int AD_THREADS = 256;
constexpr int AD_MAXCS = 16;     // largest cluster (non-portable size)
constexpr int AD_MAXSLOT = 4;    // output 32-blocks a CTA merges: kv_mul*HD/32/cs <= 8*128/32/8

template <int HD>
struct AdLayout {
  static constexpr int ROW = HD + 4;             // padded row (floats): 16-byte aligned
  static constexpr int KS = 0;
  static constexpr int VS = KS + AD_TILE * ROW;
  static constexpr int WO = KS;                             // [8 warps][AT_MAXKV][HD] warp partials (after the tiles)
  static constexpr int QS = VS + AD_TILE * ROW;             // [AT_MAXKV][HD] rotated q
  static constexpr int NK = QS + AT_MAXKV * HD;             // owner: new key (rotated) and value rows [2][HD]
  static constexpr int WS = NK + 2 * HD;                    // [8][AT_MAXKV] warp max, then [8][AT_MAXKV] warp sum
  static constexpr int RECV = WS + 2 * 8 * AT_MAXKV;        // [AD_MAXSLOT][AD_MAXCS][34] pushed block partials
  static constexpr int TOTAL = RECV + AD_MAXSLOT * AD_MAXCS * 34;
  static_assert(8 * AT_MAXKV * HD <= 2 * AD_TILE * ROW, "warp partials fit the tile area");
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// At most 96 registers a thread: then an attention CTA (8 warps) and a
// matvec CTA (9 warps, 96 registers) fit one SM together, two plus three
// warps per sub-partition within its 16K registers, so the next projection's
// CTAs become resident and stream their weights while attention runs.
//
// Per CTA: warp w takes the positions w, w+8, ... of each key tile; lane j
// holds dims [j*E, j*E+E) of q, k, v and of its running output for all KVM
// heads, so a position costs one k and one v load per lane, a butterfly
// per head for the score, and an online-softmax update in registers
// (forward.rs:328-399). The eight warp partials are combined once per CTA.
template <int HD, int KVM>
__global__ void __maxnreg__(96) attn_decode_kernel(AttnDecodeArgs a) {
  using Lo = AdLayout<HD>;
  constexpr int E = HD / 32;
  extern __shared__ __align__(16) float sm[];
  cg::cluster_group cluster = cg::this_cluster();
  float* Ks = sm + Lo::KS;
  float* Vs = sm + Lo::VS;
  float* qs = sm + Lo::QS;
  float* nk = sm + Lo::NK;
  float* wo = sm + Lo::WO;
  float* wm = sm + Lo::WS;
  float* wl = wm + 8 * AT_MAXKV;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t cs = a.n_splits;
  const uint32_t rank = cluster.block_rank();
  const uint32_t kvh = blockIdx.x / cs;
  constexpr uint32_t kv_mul = KVM;
  uint64_t* const trace = (kTrace && a.trace) ? a.trace + (uint64_t)blockIdx.x * 8 : nullptr;
  uint64_t ts[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // timeline stamps, stored at the end
  if (trace && tid == 0) ts[0] = globaltimer();
  grid_dep_launch();
  if (!a.early_kv) grid_dep_wait();
  const uint32_t pos = a.state ? (uint32_t)a.state->pos : a.pos0;
  const uint32_t nvis = pos + 1;
  const uint32_t chunk = (nvis + cs - 1) / cs;
  const uint32_t p_begin = min(nvis, rank * chunk), p_end = min(nvis, p_begin + chunk);
  const uint32_t att = a.n_heads * HD, half = HD / 2;
  const bool owner = p_begin <= pos && pos < p_end;
  const float* kbase = a.kcache + kvh * HD;
  const float* vbase = a.vcache + kvh * HD;

  auto issue_tile = [&](uint32_t base, uint32_t n) {
    for (uint32_t i = tid; i < n * (HD / 4); i += AD_THREADS) {
      const uint32_t r = i / (HD / 4), c4 = i % (HD / 4);
      if (base + r == pos) continue;  // the new row is placed from nk
      cp_async16(Ks + r * Lo::ROW + 4 * c4, kbase + (uint64_t)(base + r) * a.kv_dim + 4 * c4);
      cp_async16(Vs + r * Lo::ROW + 4 * c4, vbase + (uint64_t)(base + r) * a.kv_dim + 4 * c4);
    }
  };
  uint32_t t0 = p_begin, tn = min((uint32_t)AD_TILE, p_end - p_begin);
  if (tn) issue_tile(t0, tn);
  if (a.early_kv) grid_dep_wait();
  if (trace && tid == 0) ts[1] = globaltimer();

  // rotated q of the KVM query heads, and (owner) the new key and value rows,
  // all from the fused projection output in one round of loads
  const float2* c = a.cs + (uint64_t)pos * half;
  for (uint32_t i = tid; i < (kv_mul + (owner ? 1u : 0u)) * half; i += AD_THREADS) {
    const uint32_t hh = i / half, p = i % half;
    uint32_t i0, i1;
    pair_index(a.rope_mode, p, half, i0, i1);
    const float* src = hh < kv_mul ? a.qkv + (kvh * kv_mul + hh) * HD : a.qkv + att + kvh * HD;
    float r0, r1;
    rotate(src[i0], src[i1], c[p], r0, r1);
    float* dst = hh < kv_mul ? qs + hh * HD : nk;
    dst[i0] = r0;
    dst[i1] = r1;
  }
  if (owner) {
    for (uint32_t d = tid; d < HD; d += AD_THREADS) nk[HD + d] = a.qkv[att + a.kv_dim + kvh * HD + d];
  }
  __syncthreads();
  float qr[KVM][E], acc[KVM][E], m[KVM], l[KVM];
#pragma unroll
  for (int h = 0; h < KVM; ++h) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      qr[h][e] = qs[h * HD + lane * E + e];
      acc[h][e] = 0.0f;
    }
    m[h] = -INFINITY;
    l[h] = 0.0f;
  }
  if (trace && tid == 0) ts[4] = globaltimer();

  const uint32_t ntiles = (p_end - p_begin + AD_TILE - 1) / AD_TILE;
  for (uint32_t ti = 0; ti < ntiles; ++ti) {
    t0 = p_begin + ti * AD_TILE;
    tn = min((uint32_t)AD_TILE, p_end - t0);
    if (ti > 0) issue_tile(t0, tn);
    if (owner && pos >= t0 && pos < t0 + tn) {
      const uint32_t r = pos - t0;
      for (uint32_t d = tid; d < HD; d += AD_THREADS) {
        Ks[r * Lo::ROW + d] = nk[d];
        Vs[r * Lo::ROW + d] = nk[HD + d];
      }
    }
    cp_async_wait_all();
    __syncthreads();
    if (trace && tid == 0 && ti == 0) ts[5] = globaltimer();
    // two positions per step (p0 and p0 + 8): their loads, dots and
    // butterflies interleave, and one softmax update absorbs both. The
    // exponentials use the hardware exp2 (__expf): a few ulp on weights in
    // [0, 1], far inside the logit tolerance, and one instruction instead of
    // a range-reduced sequence on this latency-bound chain.
    for (uint32_t p0 = warp; p0 < tn; p0 += 2 * (AD_THREADS / 32)) {
      const uint32_t p1 = p0 + AD_THREADS / 32;
      const bool two = p1 < tn;  // warp-uniform
      float k0[E], v0[E], k1[E], v1[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        k0[e] = Ks[p0 * Lo::ROW + lane * E + e];
        v0[e] = Vs[p0 * Lo::ROW + lane * E + e];
        k1[e] = two ? Ks[p1 * Lo::ROW + lane * E + e] : 0.0f;
        v1[e] = two ? Vs[p1 * Lo::ROW + lane * E + e] : 0.0f;
      }
      float s0[KVM], s1[KVM];
#pragma unroll
      for (int h = 0; h < KVM; ++h) {
        float t0v = 0.0f, t1v = 0.0f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          t0v = fmaf(qr[h][e], k0[e], t0v);
          t1v = fmaf(qr[h][e], k1[e], t1v);
        }
        s0[h] = t0v;
        s1[h] = t1v;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int h = 0; h < KVM; ++h) {
          s0[h] += __shfl_xor_sync(FULL, s0[h], o);
          s1[h] += __shfl_xor_sync(FULL, s1[h], o);
        }
#pragma unroll
      for (int h = 0; h < KVM; ++h) {
        const float a0 = __fmul_rn(s0[h], a.scale);  // (q.k) * scale (forward.rs:328-346)
        const float a1 = two ? __fmul_rn(s1[h], a.scale) : -INFINITY;
        const float mn = fmaxf(m[h], fmaxf(a0, a1));
        const float cf = __expf(m[h] - mn);  // 0 while m is -inf
        const float e0 = __expf(a0 - mn);
        const float e1 = two ? __expf(a1 - mn) : 0.0f;
        l[h] = fmaf(l[h], cf, e0 + e1);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[h][e] = fmaf(acc[h][e], cf, fmaf(e0, v0[e], e1 * v1[e]));
        m[h] = mn;
      }
    }
    __syncthreads();  // the tile area is reloaded or reused below
  }
  // warp partials -> CTA partial (unnormalized, with its max and sum)
#pragma unroll
  for (int h = 0; h < KVM; ++h) {
#pragma unroll
    for (int e = 0; e < E; ++e) wo[(warp * AT_MAXKV + h) * HD + lane * E + e] = acc[h][e];
    if (lane == 0) {
      wm[warp * AT_MAXKV + h] = m[h];
      wl[warp * AT_MAXKV + h] = l[h];
    }
  }
  __syncthreads();
  if (trace && tid == 0) ts[6] = globaltimer();
  // The KV head's kv_mul*HD outputs form 32-blocks; block b is merged by CTA
  // b % cs. Each CTA pushes its partial of every block, with the head's max
  // and sum, into the merging CTA's shared memory (distributed shared
  // memory); one cluster barrier later every CTA merges its blocks locally.
  float* recv = sm + Lo::RECV;  // [AD_MAXSLOT][AD_MAXCS][34]: 32 outputs, max, sum
  for (uint32_t i = tid; i < kv_mul * HD; i += AD_THREADS) {
    const uint32_t hh = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w * AT_MAXKV + hh]);
    float O = 0.0f, Lsum = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float mw = wm[w * AT_MAXKV + hh];
      const float wgt = mw == -INFINITY ? 0.0f : __expf(mw - M);
      O = fmaf(wo[(w * AT_MAXKV + hh) * HD + d], wgt, O);
      Lsum = fmaf(wl[w * AT_MAXKV + hh], wgt, Lsum);
    }
    const uint32_t b = i / 32, j = i % 32;
    float* dst = cluster.map_shared_rank(recv, b % cs) + ((b / cs) * AD_MAXCS + rank) * 34;
    dst[j] = O;
    if (j == 0) {
      dst[32] = M;
      dst[33] = Lsum;
    }
  }
  cluster.sync();  // release the pushes / acquire the peers' pushes
  if (trace && tid == 0) ts[2] = globaltimer();
  const uint32_t nblk = kv_mul * HD / 32;
  for (uint32_t b = rank + cs * warp; b < nblk; b += cs * (AD_THREADS / 32)) {
    const float* src = recv + (b / cs) * AD_MAXCS * 34;
    float M = -INFINITY;
    for (uint32_t r = 0; r < cs; ++r) M = fmaxf(M, src[r * 34 + 32]);
    float L = 0.0f, accv = 0.0f;
    for (uint32_t r = 0; r < cs; ++r) {
      const float mr = src[r * 34 + 32];
      const float w = mr == -INFINITY ? 0.0f : __expf(mr - M);
      L = fmaf(src[r * 34 + 33], w, L);
      accv = fmaf(src[r * 34 + lane], w, accv);
    }
    const float v = L > 0.0f ? __fdiv_rn(accv, L) : 0.0f;
    const uint64_t k = (uint64_t)kvh * kv_mul * HD + b * 32 + lane;
    if (a.out) a.out[k] = v;
    if (a.q8) {
      float sc;
      const int8_t qv = quant_q8_lane(v, &sc);
      a.q8[k] = qv;
      if (lane == 0) a.s8[k / 32] = sc;
    }
  }
  // The new rows go to the cache last: a global store before the cluster
  // barrier would make every CTA's release wait for its acknowledgement.
  if (owner) {
    float* kdst = a.kcache + (uint64_t)pos * a.kv_dim + kvh * HD;
    float* vdst = a.vcache + (uint64_t)pos * a.kv_dim + kvh * HD;
    for (uint32_t d = tid; d < HD; d += AD_THREADS) {
      kdst[d] = nk[d];
      vdst[d] = nk[HD + d];
    }
  }
  if (trace && tid == 0) {
    ts[3] = globaltimer();
    for (int i = 0; i < 8; ++i) trace[i] = ts[i];
  }
}

template <int HD, int KVM>
static cudaError_t decode_config(uint32_t n_kv_heads, uint32_t cs, cudaStream_t st, bool pdl, cudaLaunchConfig_t& cfg,
                                 cudaLaunchAttribute (&attr)[2]) {
  const uint32_t smem = AdLayout<HD>::TOTAL * sizeof(float);
  cudaError_t e =
      cudaFuncSetAttribute(attn_decode_kernel<HD, KVM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_decode_kernel<HD, KVM>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  cfg = {};
  cfg.gridDim = dim3(n_kv_heads * cs);
  cfg.blockDim = dim3(AD_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaSuccess;
}

template <int HD>
static uint32_t decode_splits_hd(uint32_t n_kv_heads) {
  for (uint32_t cs : {16u, 8u}) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    int n = 0;
    cudaError_t e = decode_config<HD, 4>(n_kv_heads, cs, nullptr, false, cfg, attr);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel<HD, 4>, &cfg);
    if (e != cudaSuccess) (void)cudaGetLastError();
    if (e == cudaSuccess && n >= (int)n_kv_heads) return cs;
  }
  return 8;
}

uint32_t attention_decode_splits(uint32_t n_kv_heads, uint32_t head_size) {
  return head_size == 64 ? decode_splits_hd<64>(n_kv_heads) : decode_splits_hd<128>(n_kv_heads);
}

template <int HD, int KVM>
static cudaError_t launch_decode(const AttnDecodeArgs& a, const LaunchCfg& lc) {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[2];
  cudaError_t e = decode_config<HD, KVM>(a.n_kv_heads, a.n_splits, lc.stream, lc.pdl, cfg, attr);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel<HD, KVM>, a);
}

template <int HD>
static cudaError_t launch_decode_hd(const AttnDecodeArgs& a, const LaunchCfg& lc, uint32_t kv_mul) {
  switch (kv_mul) {
    case 1: return launch_decode<HD, 1>(a, lc);
    case 2: return launch_decode<HD, 2>(a, lc);
    case 3: return launch_decode<HD, 3>(a, lc);
    case 4: return launch_decode<HD, 4>(a, lc);
    case 5: return launch_decode<HD, 5>(a, lc);
    case 6: return launch_decode<HD, 6>(a, lc);
    case 7: return launch_decode<HD, 7>(a, lc);
    case 8: return launch_decode<HD, 8>(a, lc);
  }
  return cudaErrorInvalidValue;
}

cudaError_t attention_decode(const AttnDecodeArgs& a, const LaunchCfg& lc) {
  const uint32_t kv_mul = a.n_kv_heads ? a.n_heads / a.n_kv_heads : 0;
  if (kv_mul == 0 || kv_mul > AT_MAXKV || a.n_splits == 0 || a.n_splits > AD_MAXCS) return cudaErrorInvalidValue;
  if (a.kv_dim % 4 || ((uintptr_t)a.kcache | (uintptr_t)a.vcache) % 16) return cudaErrorInvalidValue;
  if (a.head_size == 64) return launch_decode_hd<64>(a, lc, kv_mul);
  if (a.head_size == 128) return launch_decode_hd<128>(a, lc, kv_mul);
  return cudaErrorInvalidValue;
}

}  // namespace k
}  // namespace yl
