// RoPE + KV-cache write and causal GQA attention over the f32 KV cache.
//
// Attention reproduces forward.rs:299-400 operation for operation, so its
// output is bit-identical to the reference's (the model is chaotic enough
// that any other rounding would eventually change a greedy token):
//   score[t2] = dot8(q, k[t2]) * scale     eight lane accumulators, lane l
//                                          taking q[8s+l]*k[8s+l] in order,
//                                          folded ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7))
//   max      = max(-1e10, scores)          order-free
//   e[t2]    = exp(score[t2] - max)        the correctly rounded exp (yl_expf)
//   sum      = ((0 + e[0]) + e[1]) + ...   one chain in position order
//   p[t2]    = e[t2] * (sum > 0 ? 1/sum : 0)
//   out[d]   = reduce(lanes), lane l summing p[8c+l]*v[8c+l][d] over
//              c < seq_len/8 in order, then + p*v for the seq_len % 8 tail
// Masked positions (t2 > the query's position) have e = 0 and p = 0 and add
// exactly nothing, so they are skipped; the lane / tail split still follows
// the batch's seq_len. The sequential sum and the P.V lanes are what the
// kernels' latency is built around: every chain runs in one thread, and the
// work around them is spread over the CTA (or the cluster, for decode).
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

constexpr int AT_MAXKV = 8;  // max query heads per KV head

// wide::f32x8::reduce_add as the oracle restates it.
__device__ __forceinline__ float reduce_add8(float l0, float l1, float l2, float l3, float l4, float l5, float l6,
                                             float l7) {
  const float a0 = __fadd_rn(l0, l4), a1 = __fadd_rn(l1, l5), a2 = __fadd_rn(l2, l6), a3 = __fadd_rn(l3, l7);
  return __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
}

// dot8 of forward.rs:332-343 over HD floats (both 16-byte aligned).
template <int HD>
__device__ __forceinline__ float dot8_exact(const float* q, const float* k) {
  float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f, l3 = 0.0f, l4 = 0.0f, l5 = 0.0f, l6 = 0.0f, l7 = 0.0f;
#pragma unroll
  for (int s = 0; s < HD / 8; ++s) {
    const float4 qa = *reinterpret_cast<const float4*>(q + 8 * s);
    const float4 qb = *reinterpret_cast<const float4*>(q + 8 * s + 4);
    const float4 ka = *reinterpret_cast<const float4*>(k + 8 * s);
    const float4 kb = *reinterpret_cast<const float4*>(k + 8 * s + 4);
    l0 = __fadd_rn(l0, __fmul_rn(qa.x, ka.x));
    l1 = __fadd_rn(l1, __fmul_rn(qa.y, ka.y));
    l2 = __fadd_rn(l2, __fmul_rn(qa.z, ka.z));
    l3 = __fadd_rn(l3, __fmul_rn(qa.w, ka.w));
    l4 = __fadd_rn(l4, __fmul_rn(qb.x, kb.x));
    l5 = __fadd_rn(l5, __fmul_rn(qb.y, kb.y));
    l6 = __fadd_rn(l6, __fmul_rn(qb.z, kb.z));
    l7 = __fadd_rn(l7, __fmul_rn(qb.w, kb.w));
  }
  return reduce_add8(l0, l1, l2, l3, l4, l5, l6, l7);
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// General attention (any batch): one CTA per (query head, block of AE_QB
// query rows); the rows share every K and V tile.
constexpr int AE_QB = 16;
constexpr int AE_TILE = 64;
constexpr int AE_THREADS = 256;

constexpr int AE_ECH = 256;  // positions of exp weights staged per chunk

template <int HD>
struct AeSmem {
  float q[AE_QB][HD];
  union {
    float kv[AE_TILE][HD + 4];   // K tile, then V tile, then the output rows
    float ebuf[AE_QB][AE_ECH];   // exp weights of one chunk (softmax sums)
  };
  float w[AE_QB][AE_TILE];    // the tile's weights p
  float wmax[AE_THREADS / 32][4];
  float mx[AE_QB], inv[AE_QB];
};

template <int HD>
__global__ void __launch_bounds__(AE_THREADS) attn_exact_kernel(AttnArgs a) {
  extern __shared__ __align__(16) uint8_t ae_raw[];
  AeSmem<HD>& sm = *reinterpret_cast<AeSmem<HD>*>(ae_raw);
  grid_dep_launch();
  grid_dep_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t qh = blockIdx.x, kv_mul = a.n_heads / a.n_kv_heads, kvh = qh / kv_mul;
  const uint32_t pos0 = a.state ? (uint32_t)a.state->pos : a.pos0;
  const uint32_t r0 = blockIdx.y * AE_QB, nr = min((uint32_t)AE_QB, a.ntok - r0);
  const uint32_t seq = pos0 + a.ntok;           // the batch's seq_len
  const uint32_t nvis = pos0 + r0 + nr;         // keys any row of this CTA sees
  const uint32_t att = a.n_heads * HD;
  const float* kb = a.kcache + kvh * HD;
  const float* vb = a.vcache + kvh * HD;
  const uint64_t sstride = attention_scratch_stride(a.ntok, pos0);
  auto wrow = [&](uint32_t r) { return a.part + ((uint64_t)(r0 + r) * a.n_heads + qh) * sstride; };

  for (uint32_t i = tid; i < nr * HD / 4; i += AE_THREADS) {
    const uint32_t r = i / (HD / 4), c = i % (HD / 4);
    reinterpret_cast<float4*>(sm.q[r])[c] = reinterpret_cast<const float4*>(a.q + (uint64_t)(r0 + r) * att + qh * HD)[c];
  }
  // ---- scores, running maxima (rows tid/64 + 4m, m = 0..3) ----
  float rmax[4] = {-1e10f, -1e10f, -1e10f, -1e10f};
  for (uint32_t t0 = 0; t0 < nvis; t0 += AE_TILE) {
    const uint32_t tn = min((uint32_t)AE_TILE, nvis - t0);
    __syncthreads();  // the tile area is free
    for (uint32_t i = tid; i < tn * (HD / 4); i += AE_THREADS) {
      const uint32_t j = i / (HD / 4), c = i % (HD / 4);
      cp_async16(&sm.kv[j][4 * c], kb + (uint64_t)(t0 + j) * a.kv_dim + 4 * c);
    }
    cp_async_wait_all();
    __syncthreads();
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t r = tid / AE_TILE + 4 * m, j = tid % AE_TILE;
      const uint32_t t2 = t0 + j;
      if (r < nr && j < tn && t2 <= pos0 + r0 + r) {
        const float s = __fmul_rn(dot8_exact<HD>(sm.q[r], sm.kv[j]), a.scale);
        wrow(r)[t2] = s;
        rmax[m] = fmaxf(rmax[m], s);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float v = warp_max(rmax[m]);
    if (lane == 0) sm.wmax[warp][m] = v;
  }
  __syncthreads();
  if (tid < AE_QB) {  // row r's maxima sit in warps 2(r%4), 2(r%4)+1, slot r/4
    const uint32_t r = tid;
    sm.mx[r] = fmaxf(sm.wmax[2 * (r % 4)][r / 4], sm.wmax[2 * (r % 4) + 1][r / 4]);
  }
  __syncthreads();
  // ---- e = exp(s - max), chunk by chunk into shared memory (and back into
  // the scratch for the P.V pass); thread r extends row r's sum ----
  float rsum = 0.0f;
  for (uint32_t c0 = 0; c0 < nvis; c0 += AE_ECH) {
    const uint32_t cn = min((uint32_t)AE_ECH, nvis - c0);
    for (uint32_t i = tid; i < nr * cn; i += AE_THREADS) {
      const uint32_t r = i / cn, j = i % cn, t2 = c0 + j;
      float e = 0.0f;
      if (t2 <= pos0 + r0 + r) {
        e = yl_expf(__fsub_rn(wrow(r)[t2], sm.mx[r]));
        wrow(r)[t2] = e;
      }
      sm.ebuf[r][j] = e;  // masked: 0, which leaves the sum as it is
    }
    __syncthreads();
    if (tid < (int)nr) {
      const uint32_t n = min(cn, pos0 + r0 + tid + 1 > c0 ? pos0 + r0 + tid + 1 - c0 : 0u);
      const float* eb = sm.ebuf[tid];
      uint32_t j = 0;
      for (; j + 16 <= n; j += 16) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] = eb[j + u];
#pragma unroll
        for (int u = 0; u < 16; ++u) rsum = __fadd_rn(rsum, v[u]);
      }
      for (; j < n; ++j) rsum = __fadd_rn(rsum, eb[j]);
    }
    __syncthreads();  // ebuf is rewritten by the next chunk
  }
  if (tid < (int)nr) sm.inv[tid] = rsum > 0.0f ? __fdiv_rn(1.0f, rsum) : 0.0f;
  __syncthreads();
  // ---- P.V: thread (row tid/16, dims (tid%16)*DPT + j), eight lanes each ----
  constexpr int DPT = HD / 16;
  const uint32_t r = tid / 16, g = tid % 16;
  const uint32_t lim = min(seq / 8 * 8, pos0 + r0 + r + 1);  // lane-range keys of this row
  float acc[DPT][8];
#pragma unroll
  for (int j = 0; j < DPT; ++j)
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[j][l] = 0.0f;
  const uint32_t lane_end = min(seq / 8 * 8, nvis);
  for (uint32_t t0 = 0; t0 < lane_end; t0 += AE_TILE) {
    const uint32_t tn = min((uint32_t)AE_TILE, lane_end - t0);
    __syncthreads();
    for (uint32_t i = tid; i < tn * (HD / 4); i += AE_THREADS) {
      const uint32_t j = i / (HD / 4), c = i % (HD / 4);
      cp_async16(&sm.kv[j][4 * c], vb + (uint64_t)(t0 + j) * a.kv_dim + 4 * c);
    }
    for (uint32_t i = tid; i < AE_QB * AE_TILE; i += AE_THREADS) {
      const uint32_t rr = i / AE_TILE, j = i % AE_TILE;
      const uint32_t t2 = t0 + j;
      sm.w[rr][j] = (rr < nr && j < tn && t2 <= pos0 + r0 + rr) ? __fmul_rn(__ldcg(wrow(rr) + t2), sm.inv[rr]) : 0.0f;
    }
    cp_async_wait_all();
    __syncthreads();
    if (r < nr) {
      for (uint32_t j0 = 0; j0 < tn; j0 += 8) {  // t0 and tn are multiples of 8: key t0+j0+l is lane l
#pragma unroll
        for (int l = 0; l < 8; ++l) {
          const uint32_t t2 = t0 + j0 + l;
          if (t2 >= lim) break;
          const float p = sm.w[r][j0 + l];
          const float* vr = &sm.kv[j0 + l][g * DPT];
#pragma unroll
          for (int j = 0; j < DPT; ++j) acc[j][l] = __fadd_rn(acc[j][l], __fmul_rn(p, vr[j]));
        }
      }
    }
  }
  __syncthreads();  // the tile area now holds the output rows
  if (r < nr) {
    const uint32_t pr = pos0 + r0 + r;
    const float inv = sm.inv[r];
    const float* w = wrow(r);
#pragma unroll
    for (int j = 0; j < DPT; ++j) {
      float o = reduce_add8(acc[j][0], acc[j][1], acc[j][2], acc[j][3], acc[j][4], acc[j][5], acc[j][6], acc[j][7]);
      const uint32_t d = g * DPT + j;
      for (uint32_t t2 = seq / 8 * 8; t2 <= pr; ++t2)  // the seq_len % 8 tail, in order
        o = __fadd_rn(o, __fmul_rn(__fmul_rn(__ldcg(w + t2), inv), vb[(uint64_t)t2 * a.kv_dim + d]));
      sm.kv[r][d] = o;
    }
  }
  __syncthreads();
  for (uint32_t i = warp; i < nr * (HD / 32); i += AE_THREADS / 32) {
    const uint32_t rr = i / (HD / 32), b = i % (HD / 32);
    const float v = sm.kv[rr][b * 32 + lane];
    const uint64_t k = (uint64_t)(r0 + rr) * att + qh * HD + b * 32 + lane;
    if (a.out) a.out[k] = v;
    if (a.q8) {
      float sc;
      const int8_t q = quant_q8_lane(v, &sc);
      a.q8[k] = q;
      if (lane == 0) a.s8[k / 32] = sc;
    }
  }
}

cudaError_t attention(const AttnArgs& a, const LaunchCfg& lc) {
  if (a.ntok == 0) return cudaSuccess;
  const uint32_t kv_mul = a.n_kv_heads ? a.n_heads / a.n_kv_heads : 0;
  if (kv_mul == 0 || kv_mul > AT_MAXKV || !a.part) return cudaErrorInvalidValue;
  if (a.kv_dim % 4 || ((uintptr_t)a.kcache | (uintptr_t)a.vcache | (uintptr_t)a.q) % 16) return cudaErrorInvalidValue;
  const dim3 g(a.n_heads, (a.ntok + AE_QB - 1) / AE_QB);
  if (a.head_size == 64) {
    const uint32_t smem = sizeof(AeSmem<64>);
    cudaError_t e = cudaFuncSetAttribute(attn_exact_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return launch_kernel(attn_exact_kernel<64>, g, dim3(AE_THREADS), smem, lc, a);
  }
  if (a.head_size == 128) {
    const uint32_t smem = sizeof(AeSmem<128>);
    cudaError_t e = cudaFuncSetAttribute(attn_exact_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return launch_kernel(attn_exact_kernel<128>, g, dim3(AE_THREADS), smem, lc, a);
  }
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// Batch-1 decode with RoPE and the KV-cache write fused in. One cluster of cs
// CTAs per KV head:
//  1. CTA `rank` takes the rank-th slice of the positions 0..pos: its K rows
//     are fetched with cp.async (before the wait on the preceding kernel when
//     early_kv is set: they were written by earlier steps), q of the KVM
//     query heads is rotated, and the owner of `pos` rotates the new key and
//     writes the new K/V rows; then the slice's scores go to sc and the
//     slice's maxima to shared memory;
//  2. (cluster barrier) every CTA takes the head maxima from its peers'
//     shared memory and turns its slice's scores into exp(s - max);
//  3. (cluster barrier) the KV head's KVM*HD outputs are 32-blocks; CTA rank
//     takes blocks rank, rank + cs, ...: one thread per block walks the
//     softmax sum chain, then warp l runs lane l of the P.V sums for the
//     block's 32 dimensions, warp 0 folds the lanes, adds the tail and
//     quantizes the block.
namespace cg = cooperative_groups;
constexpr int AD_TILE = 64;      // positions per shared-memory K tile
constexpr int AD_THREADS = 256;
constexpr int AD_MAXCS = 16;     // largest cluster (non-portable size)
constexpr int AD_MAXSLOT = 4;    // output 32-blocks one CTA takes: KVM*HD/32/cs <= 8*128/32/8

constexpr int AD_ECH = 2048;     // positions of exp weights staged per chunk (per block)
constexpr int AD_VROWS = 512;    // V rows (32 dims each) fetched into shared memory at entry, per CTA

template <int HD>
struct AdSmem {
  union {
    float ks[AD_TILE][HD + 4];        // phase 1: the slice's K tile
    float ebuf[AD_MAXSLOT][AD_ECH];   // phase 3: exp weights of a chunk, per output block
  };
  float vbuf[AD_VROWS * 32];       // V columns of the CTA's output blocks, first rows
  float qs[AT_MAXKV][HD];
  float nk[HD];                   // owner: the new key, rotated
  float wred[AD_THREADS / 32][AD_MAXSLOT];
  float gmax[AD_MAXSLOT];
  float sum[AD_MAXSLOT];
  float lanes[8][32];             // P.V lane partials of one block
};

template <int HD, int KVM>
__global__ void __launch_bounds__(AD_THREADS) attn_decode_kernel(const __grid_constant__ AttnDecodeArgs a) {
  extern __shared__ __align__(16) uint8_t ad_raw[];
  AdSmem<HD>& sm = *reinterpret_cast<AdSmem<HD>*>(ad_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t cs = a.n_splits;
  const uint32_t rank = cluster.block_rank();
  const uint32_t kvh = blockIdx.x / cs;
  // this CTA's sequence: the single one, or grid row y of a batched launch
  const uint32_t sq = a.nseq ? blockIdx.y : 0u;
  float* const kcache = a.nseq ? a.kseq[sq] : a.kcache;
  float* const vcache = a.nseq ? a.vseq[sq] : a.vcache;
  const float* const qkv = a.qkv + (uint64_t)sq * a.qkv_stride;
  const uint64_t orow = (uint64_t)sq * a.n_heads * HD;
  float* const outp = a.out ? a.out + orow : nullptr;
  int8_t* const q8p = a.q8 ? a.q8 + orow : nullptr;
  float* const s8p = a.q8 ? a.s8 + orow / 32 : nullptr;
  uint64_t* const trace = (kTrace && a.trace && blockIdx.y == 0) ? a.trace + (uint64_t)blockIdx.x * 8 : nullptr;
  uint64_t ts[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // timeline stamps, stored at the end
  if (trace && tid == 0) ts[0] = globaltimer();
  grid_dep_launch();
  if (tid == 0) l2_prefetch_next(a.pf, blockIdx.x, gridDim.x);
  if (!a.early_kv) grid_dep_wait();
  const uint32_t pos = a.nseq ? a.pseq[sq] : a.state ? (uint32_t)a.state->pos : a.pos0;
  const uint32_t nvis = pos + 1;
  const uint32_t chunk = (nvis + cs - 1) / cs;
  const uint32_t p_begin = min(nvis, rank * chunk), p_end = min(nvis, p_begin + chunk);
  const uint32_t att = a.n_heads * HD, half = HD / 2;
  const bool owner = p_begin <= pos && pos < p_end;
  const float* kbase = kcache + kvh * HD;
  const float* vbase = vcache + kvh * HD;
  float* const sc0 = a.sc + (uint64_t)sq * a.sc_seq_stride + (uint64_t)kvh * KVM * a.sc_stride;  // this KV head's query heads

  auto issue_tile = [&](uint32_t base, uint32_t n) {
    for (uint32_t i = tid; i < n * (HD / 4); i += AD_THREADS) {
      const uint32_t r = i / (HD / 4), c4 = i % (HD / 4);
      if (base + r == pos) continue;  // the new row is placed from nk
      cp_async16(&sm.ks[r][4 * c4], kbase + (uint64_t)(base + r) * a.kv_dim + 4 * c4);
    }
  };
  uint32_t t0 = p_begin, tn = min((uint32_t)AD_TILE, p_end - p_begin);
  if (tn) issue_tile(t0, tn);
  cp_async_commit();
  constexpr uint32_t BPH = HD / 32;  // 32-blocks per head
  const uint32_t nblk = KVM * BPH;
  const uint32_t nmine = rank < nblk ? (nblk - rank + cs - 1) / cs : 0;
  const uint32_t vrows = nmine ? min(nvis, (uint32_t)AD_VROWS / nmine) : 0;
  if (a.early_kv) grid_dep_wait();
  if (trace && tid == 0) ts[1] = globaltimer();

  // rotated q of the KVM query heads and (owner) the new key; the owner also
  // writes the new K/V rows to the cache, visible to the peers after the
  // first cluster barrier
  const float2* c = a.cs + (uint64_t)pos * half;
  for (uint32_t i = tid; i < (KVM + (owner ? 1u : 0u)) * half; i += AD_THREADS) {
    const uint32_t hh = i / half, p = i % half;
    uint32_t i0, i1;
    pair_index(a.rope_mode, p, half, i0, i1);
    const float* src = hh < KVM ? qkv + (kvh * KVM + hh) * HD : qkv + att + kvh * HD;
    float r0, r1;
    rotate(src[i0], src[i1], c[p], r0, r1);
    float* dst = hh < KVM ? sm.qs[hh] : sm.nk;
    dst[i0] = r0;
    dst[i1] = r1;
    if (hh == KVM) {
      float* kd = kcache + (uint64_t)pos * a.kv_dim + kvh * HD;
      kd[i0] = r0;
      kd[i1] = r1;
    }
  }
  if (owner)
    for (uint32_t d = tid; d < HD; d += AD_THREADS)
      vcache[(uint64_t)pos * a.kv_dim + kvh * HD + d] = qkv[att + a.kv_dim + kvh * HD + d];
  if (trace && tid == 0) ts[4] = globaltimer();

  // ---- 1. scores of the slice: thread (head tid/64 + 4m, key tid%64) ----
  const uint32_t ntiles = (p_end - p_begin + AD_TILE - 1) / AD_TILE;
  for (uint32_t ti = 0; ti < ntiles; ++ti) {
    t0 = p_begin + ti * AD_TILE;
    tn = min((uint32_t)AD_TILE, p_end - t0);
    if (ti > 0) {
      __syncthreads();  // the previous tile is consumed
      issue_tile(t0, tn);
      cp_async_commit();
    }
    cp_async_wait_group<0>();
    __syncthreads();  // rotated q / nk and the tile are in place
    if (owner && pos >= t0 && pos < t0 + tn)
      for (uint32_t d = tid; d < HD; d += AD_THREADS) sm.ks[pos - t0][d] = sm.nk[d];
    __syncthreads();
    if (trace && tid == 0 && ti == 0) ts[5] = globaltimer();
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const uint32_t hh = tid / AD_TILE + 4 * m, j = tid % AD_TILE;
      if (hh < KVM && j < tn) sc0[(uint64_t)hh * a.sc_stride + t0 + j] = __fmul_rn(dot8_exact<HD>(sm.qs[hh], sm.ks[j]), a.scale);
    }
  }
  if (trace && tid == 0) ts[6] = globaltimer();
  // The V columns of this CTA's output blocks (blocks rank, rank + cs, ...,
  // 32 dimensions each), first `vrows` positions, into shared memory: they
  // do not depend on this step's scores, and rows below pos were written by
  // earlier steps (issued here, they land while the cluster syncs and the
  // softmax sums run). Row pos (the new value row) is placed from qkv later.
  for (uint32_t i = 0; i < nmine; ++i) {
    const uint32_t d0 = ((rank + i * cs) % BPH) * 32;
    float* vb = sm.vbuf + i * vrows * 32;
    for (uint32_t e = tid; e < vrows * 8; e += AD_THREADS) {
      const uint32_t r = e / 8, c4 = e % 8;
      if (r == pos) continue;
      cp_async16(vb + r * 32 + 4 * c4, vbase + (uint64_t)r * a.kv_dim + d0 + 4 * c4);
    }
  }
  cp_async_commit();
  cluster.sync();  // every slice's scores and the new cache rows are visible to the cluster
  if (trace && tid == 0) ts[2] = globaltimer();

  // ---- 2. the CTA's output blocks: block b = rank + i*cs, head b / BPH ----
  auto head_of = [&](uint32_t i) { return (rank + i * cs) / BPH; };
  // max(-1e10, scores), e = exp(s - max) and the sums of each block's head.
  // Rows that fit one chunk are read once into shared memory; longer rows
  // take a pass for the max, then chunk by chunk exp and sums (the scores in
  // sc are only read: the CTAs sharing a head each keep their own weights).
  const uint32_t nchunk = (nvis + AD_ECH - 1) / AD_ECH;
  auto fill_chunk = [&](uint32_t c0, uint32_t cn) {
    for (uint32_t i = 0; i < nmine; ++i) {
      const float* w = sc0 + (uint64_t)head_of(i) * a.sc_stride + c0;
      for (uint32_t j = tid; j < cn; j += AD_THREADS) sm.ebuf[i][j] = yl_expf(__fsub_rn(__ldcg(w + j), sm.gmax[i]));
    }
  };
  {
    float m[AD_MAXSLOT];
#pragma unroll
    for (int i = 0; i < AD_MAXSLOT; ++i) {
      m[i] = -1e10f;
      if ((uint32_t)i < nmine) {
        const float* w = sc0 + (uint64_t)head_of(i) * a.sc_stride;
        for (uint32_t t2 = tid; t2 < nvis; t2 += AD_THREADS) {
          const float v = __ldcg(w + t2);
          if (nchunk == 1) sm.ebuf[i][t2] = v;
          m[i] = fmaxf(m[i], v);
        }
      }
      m[i] = warp_max(m[i]);
      if (lane == 0) sm.wred[warp][i] = m[i];
    }
    __syncthreads();
    if (tid < AD_MAXSLOT) {
      float g = -1e10f;
      for (int w = 0; w < AD_THREADS / 32; ++w) g = fmaxf(g, sm.wred[w][tid]);
      sm.gmax[tid] = g;
      sm.sum[tid] = 0.0f;
    }
    __syncthreads();
  }
  for (uint32_t c = 0; c < nchunk; ++c) {
    const uint32_t c0 = c * AD_ECH, cn = min((uint32_t)AD_ECH, nvis - c0);
    if (nchunk == 1) {
      for (uint32_t i = 0; i < nmine; ++i)
        for (uint32_t j = tid; j < cn; j += AD_THREADS) sm.ebuf[i][j] = yl_expf(__fsub_rn(sm.ebuf[i][j], sm.gmax[i]));
    } else {
      fill_chunk(c0, cn);
    }
    __syncthreads();
    if (lane == 0 && (uint32_t)warp < nmine) {
      const float* eb = sm.ebuf[warp];
      float s = sm.sum[warp];
      uint32_t j = 0;
      if (cn >= 16) {  // software-pipelined: the next 16 weights load while these 16 add
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const float4*>(eb + 4 * u);
        for (j = 16; j + 16 <= cn; j += 16) {
          float4 nv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) nv[u] = *reinterpret_cast<const float4*>(eb + j + 4 * u);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            s = __fadd_rn(s, v[u].x);
            s = __fadd_rn(s, v[u].y);
            s = __fadd_rn(s, v[u].z);
            s = __fadd_rn(s, v[u].w);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) v[u] = nv[u];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          s = __fadd_rn(s, v[u].x);
          s = __fadd_rn(s, v[u].y);
          s = __fadd_rn(s, v[u].z);
          s = __fadd_rn(s, v[u].w);
        }
      }
      for (; j < cn; ++j) s = __fadd_rn(s, eb[j]);
      sm.sum[warp] = s;
    }
    __syncthreads();  // ebuf is rewritten by the next chunk (or read below)
  }
  if (trace && tid == 0) ts[7] = globaltimer();
  // the staged V columns have landed; the new value row goes in from qkv
  cp_async_wait_group<0>();
  if (pos < vrows)
    for (uint32_t i = 0; i < nmine; ++i)
      if (tid < 32)
        sm.vbuf[(i * vrows + pos) * 32 + tid] =
            qkv[att + a.kv_dim + kvh * HD + ((rank + i * cs) % BPH) * 32 + tid];
  __syncthreads();
  // P.V: warp l runs lane l of the sums (positions l, l + 8, ...) for every
  // block of the CTA, chunk by chunk (a single chunk is still in ebuf); the
  // lane chains carry over chunk boundaries, which are multiples of 8
  const uint32_t nsimd8 = nvis / 8 * 8;
  float inv[AD_MAXSLOT], acc[AD_MAXSLOT];
#pragma unroll
  for (int i = 0; i < AD_MAXSLOT; ++i) {
    inv[i] = sm.sum[i] > 0.0f ? __fdiv_rn(1.0f, sm.sum[i]) : 0.0f;
    acc[i] = 0.0f;
  }
  for (uint32_t c = 0; c < nchunk; ++c) {
    const uint32_t c0 = c * AD_ECH, cn = min((uint32_t)AD_ECH, nvis - c0);
    if (nchunk > 1) {
      __syncthreads();
      fill_chunk(c0, cn);
      __syncthreads();
    }
    const uint32_t cend = min(c0 + cn, nsimd8);
#pragma unroll
    for (int i = 0; i < AD_MAXSLOT; ++i) {
      if ((uint32_t)i >= nmine) break;
      const uint32_t b = rank + i * cs, d = (b % BPH) * 32 + lane;
      const float* vcol = vbase + d;
      const float* eb = sm.ebuf[i] - c0;
      const float* vs = sm.vbuf + i * vrows * 32 + lane;
      float s = acc[i];
      uint32_t t2 = c0 + warp;
      const uint32_t send = min(cend, vrows);  // rows below send are in shared memory
      for (; t2 + 64 <= send; t2 += 64) {
        float vv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) vv[u] = vs[(t2 + 8 * u) * 32];
#pragma unroll
        for (int u = 0; u < 8; ++u) s = __fadd_rn(s, __fmul_rn(__fmul_rn(eb[t2 + 8 * u], inv[i]), vv[u]));
      }
      for (; t2 < send; t2 += 8) s = __fadd_rn(s, __fmul_rn(__fmul_rn(eb[t2], inv[i]), vs[t2 * 32]));
      for (; t2 < cend; t2 += 128) {  // rows past the staged ones: sixteen positions' loads in flight
        float vv[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
          vv[u] = t2 + 8 * u < cend ? __ldcg(vcol + (uint64_t)(t2 + 8 * u) * a.kv_dim) : 0.0f;  // row pos: the owner's write
#pragma unroll
        for (int u = 0; u < 16; ++u)
          if (t2 + 8 * u < cend) s = __fadd_rn(s, __fmul_rn(__fmul_rn(eb[t2 + 8 * u], inv[i]), vv[u]));
      }
      acc[i] = s;
    }
  }
  // fold the lanes, add the tail (positions nsimd8..pos, in the last chunk)
  for (uint32_t i = 0; i < nmine; ++i) {
    const uint32_t b = rank + i * cs, hh = b / BPH, d = (b % BPH) * 32 + lane;
    sm.lanes[warp][lane] = acc[i];
    __syncthreads();
    if (warp == 0) {
      float o = reduce_add8(sm.lanes[0][lane], sm.lanes[1][lane], sm.lanes[2][lane], sm.lanes[3][lane],
                            sm.lanes[4][lane], sm.lanes[5][lane], sm.lanes[6][lane], sm.lanes[7][lane]);
      const uint32_t c0 = (nchunk - 1) * AD_ECH;
      float vt[8];  // the tail's (at most 7) V values, loaded ahead of the chain
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t tt = nsimd8 + u;
        vt[u] = tt >= nvis ? 0.0f
                           : tt < vrows ? sm.vbuf[(i * vrows + tt) * 32 + lane]
                                        : __ldcg(vbase + d + (uint64_t)tt * a.kv_dim);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (nsimd8 + u < nvis) o = __fadd_rn(o, __fmul_rn(__fmul_rn(sm.ebuf[i][nsimd8 + u - c0], inv[i]), vt[u]));
      const uint64_t k = (uint64_t)(kvh * KVM + hh) * HD + d;
      if (outp) outp[k] = o;
      if (q8p) {
        float scl;
        const int8_t qv = quant_q8_lane(o, &scl);
        q8p[k] = qv;
        if (lane == 0) s8p[k / 32] = scl;
      }
    }
    __syncthreads();  // lanes[] is rewritten by the next block
  }
  if (trace && tid == 0) {
    ts[3] = globaltimer();
    for (int i = 0; i < 8; ++i) trace[i] = ts[i];
  }
}

template <int HD, int KVM>
static cudaError_t decode_config(uint32_t n_kv_heads, uint32_t cs, cudaStream_t st, bool pdl, cudaLaunchConfig_t& cfg,
                                 cudaLaunchAttribute (&attr)[2], uint32_t nseq = 0) {
  const uint32_t smem = sizeof(AdSmem<HD>);
  cudaError_t e =
      cudaFuncSetAttribute(attn_decode_kernel<HD, KVM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_decode_kernel<HD, KVM>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  cfg = {};
  cfg.gridDim = dim3(n_kv_heads * cs, nseq ? nseq : 1u);
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
  cudaError_t e = decode_config<HD, KVM>(a.n_kv_heads, a.n_splits, lc.stream, lc.pdl, cfg, attr, a.nseq);
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
  if (kv_mul * a.head_size / 32 > a.n_splits * AD_MAXSLOT) return cudaErrorInvalidValue;
  if (a.kv_dim % 4 || (uintptr_t)a.sc % 16 || a.sc_stride % 4 || !a.sc || a.nseq > YL_MAX_BATCH)
    return cudaErrorInvalidValue;
  if (a.nseq == 0 && ((uintptr_t)a.kcache | (uintptr_t)a.vcache) % 16) return cudaErrorInvalidValue;
  for (uint32_t i = 0; i < a.nseq; ++i)
    if (!a.kseq[i] || !a.vseq[i] || ((uintptr_t)a.kseq[i] | (uintptr_t)a.vseq[i]) % 16) return cudaErrorInvalidValue;
  if (a.nseq && (a.qkv_stride % 4 || a.sc_seq_stride % 4 || a.sc_seq_stride < (uint64_t)a.n_heads * a.sc_stride))
    return cudaErrorInvalidValue;
  if (a.head_size == 64) return launch_decode_hd<64>(a, lc, kv_mul);
  if (a.head_size == 128) return launch_decode_hd<128>(a, lc, kv_mul);
  return cudaErrorInvalidValue;
}

}  // namespace k
}  // namespace yl
