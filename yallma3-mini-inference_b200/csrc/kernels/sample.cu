// Device sampler: Sampler::sample of the reference (sampler.rs:117-180) on a
// logits row that stays in HBM, so generation needs no logits copy to the
// host. Same arithmetic in the same order:
//   * temperature 0: sample_argmax (first index of the maximum, :67-79);
//   * else logits[q] /= T, softmax (max, exp(x - max), the sum in index
//     order, x /= sum; :28-39), then
//       top_p outside (0, 1): sample_mult, the cdf in index order (:93-104);
//       else sample_topp (:117-155): entries with p >= cutoff are written in
//       index order to the front of the sampler's persistent (prob, index)
//       array, the WHOLE array is sorted stably by descending prob (entries
//       past the kept count are the previous calls' leftovers, as in the
//       reference), the cumulative sum runs until it exceeds top_p, and the
//       draw r = rand * cumulative is located in the same prefix sums.
// The additions the reference chains (softmax sum, cumulative and cdf sums)
// run as one sequential chain on one thread, with the loads issued ahead:
// every prefix sum equals the reference's bit for bit. `exp` is the correctly
// rounded yl_expf of the forward pass.
#include <cub/device/device_radix_sort.cuh>

#include "device.cuh"
#include "expf_exact.h"
#include "kernels.h"

namespace yl {
namespace k {

namespace {

constexpr int SMP_THREADS = 512;
constexpr int SMP_ITEMS = 4;  // values per thread in the grid-wide passes
constexpr uint32_t SMP_TILE = SMP_THREADS * SMP_ITEMS;

__device__ __forceinline__ bool smp_better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// logits /= T and per-tile maxima (f32::max ignores NaN)
__global__ void __launch_bounds__(SMP_THREADS) smp_scale_max(SampleArgs a) {
  __shared__ float red[SMP_THREADS / 32];
  const uint32_t base = blockIdx.x * SMP_TILE;
  float m = -INFINITY;
#pragma unroll
  for (int u = 0; u < SMP_ITEMS; ++u) {
    const uint32_t q = base + u * SMP_THREADS + threadIdx.x;
    if (q < a.V) {
      const float x = __fdiv_rn(a.logits[q], a.temperature);
      a.logits[q] = x;
      m = fmaxf(m, x);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = red[0];
    for (int w = 1; w < SMP_THREADS / 32; ++w) b = fmaxf(b, red[w]);
    a.tile_val[blockIdx.x] = b;
  }
}

__device__ __forceinline__ float smp_global_max(const SampleArgs& a) {
  __shared__ float gm;
  if (threadIdx.x < 32) {
    float m = -INFINITY;
    for (uint32_t t = threadIdx.x; t < a.ntiles; t += 32) m = fmaxf(m, a.tile_val[t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (threadIdx.x == 0) gm = m;
  }
  __syncthreads();
  return gm;
}

// e = exp(x - max)
__global__ void __launch_bounds__(SMP_THREADS) smp_exp(SampleArgs a) {
  const float m = smp_global_max(a);
  const uint32_t base = blockIdx.x * SMP_TILE;
#pragma unroll
  for (int u = 0; u < SMP_ITEMS; ++u) {
    const uint32_t q = base + u * SMP_THREADS + threadIdx.x;
    if (q < a.V) a.logits[q] = yl_expf(__fsub_rn(a.logits[q], m));
  }
}

// The chain s = ((0 + v0) + v1) + ... over v[0, n), walked by thread 0 of a
// block of SMP_THREADS threads: the block stages the values through shared
// memory in tiles of SMP_CT (double-buffered, every thread loading the next
// tile while thread 0 adds the current one), and thread 0 keeps the next 32
// values in registers ahead of its dependent additions, so the chain runs at
// the latency of the additions rather than of global loads. With PRE every
// partial sum is stored to pre[]. The values are >= 0, so the partial sums
// never decrease: the first index whose sum exceeds `stop_above` lies in the
// first group of 32 whose last sum does, which is walked again (the same
// additions from the same start) to find it. Every thread returns the final
// (or stopping) sum; *stopped (thread 0's) is that index, or 0xFFFFFFFF.
constexpr uint32_t SMP_CT = 4096;

template <bool PRE>
__device__ float smp_chain_block(const float* v, uint32_t n, float* pre, float stop_above, uint32_t* stopped) {
  __shared__ __align__(16) float tile[2][SMP_CT];
  __shared__ uint32_t s_stop;
  __shared__ float s_sum;
  const uint32_t tid = threadIdx.x, nt = (n + SMP_CT - 1) / SMP_CT;
  for (uint32_t i = tid; i < SMP_CT && i < n; i += SMP_THREADS) tile[0][i] = __ldcg(v + i);
  if (tid == 0) s_stop = 0xFFFFFFFFu;
  __syncthreads();
  float s = 0.0f;
  for (uint32_t t = 0; t < nt; ++t) {
    const uint32_t base = t * SMP_CT;
    if (t + 1 < nt)
      for (uint32_t i = tid; i < SMP_CT && base + SMP_CT + i < n; i += SMP_THREADS)
        tile[(t + 1) & 1][i] = __ldcg(v + base + SMP_CT + i);
    if (tid == 0) {
      const float* tv = tile[t & 1];
      const uint32_t m = n - base < SMP_CT ? n - base : SMP_CT;
      float cur[32], nxt[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) cur[u] = (uint32_t)u < m ? tv[u] : 0.0f;
      for (uint32_t i0 = 0; i0 < m; i0 += 32) {
#pragma unroll
        for (int u = 0; u < 32; ++u) nxt[u] = i0 + 32 + u < m ? tv[i0 + 32 + u] : 0.0f;
        const float start = s;
        const uint32_t k = m - i0 < 32u ? m - i0 : 32u;
        if (k == 32u) {
#pragma unroll
          for (int u = 0; u < 32; ++u) {
            s = __fadd_rn(s, cur[u]);
            if (PRE) pre[base + i0 + u] = s;
          }
        } else {  // the tail (from shared memory: no dynamic register index)
          for (uint32_t u = 0; u < k; ++u) {
            s = __fadd_rn(s, tv[i0 + u]);
            if (PRE) pre[base + i0 + u] = s;
          }
        }
        if (s > stop_above) {
          float r = start;
          for (uint32_t u = 0; u < k; ++u) {
            r = __fadd_rn(r, tv[i0 + u]);
            if (r > stop_above) {
              s_stop = base + i0 + u;
              break;
            }
          }
          s = r;
          break;
        }
#pragma unroll
        for (int u = 0; u < 32; ++u) cur[u] = nxt[u];
      }
      s_sum = s;
    }
    __syncthreads();  // the next tile is staged; thread 0 is done with this one
    if (s_stop != 0xFFFFFFFFu) break;
  }
  *stopped = s_stop;
  return s_sum;
}

// the softmax denominator, summed in index order (the reference's f32 Sum)
__global__ void __launch_bounds__(SMP_THREADS) smp_sum(SampleArgs a) {
  uint32_t dummy;
  const float sum = smp_chain_block<false>(a.logits, a.V, nullptr, INFINITY, &dummy);
  if (threadIdx.x == 0) a.misc[0] = sum;
}

// p = e / sum; top-p: per-tile count of entries with p >= cutoff
__global__ void __launch_bounds__(SMP_THREADS) smp_norm(SampleArgs a) {
  __shared__ uint32_t cnt[SMP_THREADS / 32];
  const float sum = a.misc[0];
  const uint32_t base = blockIdx.x * SMP_TILE;
  uint32_t c = 0;
#pragma unroll
  for (int u = 0; u < SMP_ITEMS; ++u) {
    const uint32_t q = base + u * SMP_THREADS + threadIdx.x;
    if (q < a.V) {
      const float p = __fdiv_rn(a.logits[q], sum);
      a.logits[q] = p;
      c += p >= a.cutoff ? 1u : 0u;
    }
  }
  if (!a.topp) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
  if ((threadIdx.x & 31) == 0) cnt[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int w = 0; w < SMP_THREADS / 32; ++w) t += cnt[w];
    a.tile_cnt[blockIdx.x] = t;
  }
}

// Kept entries (p >= cutoff) to the front of the persistent array, in index
// order: tile offset = sum of the earlier tiles' counts, rank inside the tile
// by a block-wide scan over (item, thread) in index order.
__global__ void __launch_bounds__(SMP_THREADS) smp_compact(SampleArgs a) {
  __shared__ uint32_t wsum[SMP_THREADS / 32];
  __shared__ uint32_t tile_off;
  if (threadIdx.x < 32) {
    uint32_t s = 0;
    for (uint32_t t = threadIdx.x; t < blockIdx.x; t += 32) s += a.tile_cnt[t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (threadIdx.x == 0) tile_off = s;
  }
  const uint32_t base = blockIdx.x * SMP_TILE;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t run = 0;  // kept entries of this tile before the current item row
  __syncthreads();
#pragma unroll
  for (int u = 0; u < SMP_ITEMS; ++u) {
    const uint32_t q = base + u * SMP_THREADS + threadIdx.x;
    const float p = q < a.V ? a.logits[q] : 0.0f;
    const bool keep = q < a.V && p >= a.cutoff;
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, keep);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    uint32_t before = 0, row = 0;
    for (int w = 0; w < SMP_THREADS / 32; ++w) {
      const uint32_t x = wsum[w];
      if (w < warp) before += x;
      row += x;
    }
    if (keep) {
      const uint32_t pos = tile_off + run + before + __popc(bal & ((1u << lane) - 1u));
      a.sprob[pos] = p;
      a.sidx[pos] = q;
    }
    run += row;
    __syncthreads();  // wsum is rewritten for the next item row
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) a.misc[1] = __uint_as_float(tile_off + run);
}

// The cumulative chain over the sorted entries, then the draw, located by
// warp 0 in the same prefix sums (the reference's cdf loop over 0..=last adds
// the same values in the same order from 0).
__global__ void __launch_bounds__(SMP_THREADS) smp_topp_pick(SampleArgs a) {
  const int lane = threadIdx.x & 31;
  const uint32_t n0 = __float_as_uint(a.misc[1]);
  if (n0 == 0) {  // the reference underflows n0 - 1 (a panic)
    if (threadIdx.x == 0) {
      if (a.err) atomicExch(a.err, dev::ERR_BAD_ARG);
      *a.out = 0u;
    }
    return;
  }
  uint32_t stop;
  const float cum = smp_chain_block<true>(a.sprob, n0, a.prefix, a.top_p, &stop);
  if (threadIdx.x >= 32) return;
  __threadfence_block();  // thread 0's prefix stores, before warp 0 reads them
  const uint32_t last = stop == 0xFFFFFFFFu ? n0 - 1 : stop;
  const float r = __fmul_rn(a.rand, cum);
  for (uint32_t i0 = 0; i0 <= last; i0 += 32) {
    const uint32_t i = i0 + lane;
    const bool hit = i <= last && r < __ldcg(a.prefix + i);
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, hit);
    if (bal) {
      if (lane == 0) *a.out = a.sidx[i0 + __ffs(bal) - 1];
      return;
    }
  }
  if (lane == 0) *a.out = a.sidx[last];
}

// sample_mult: first index whose cdf (index order) exceeds rand
__global__ void __launch_bounds__(SMP_THREADS) smp_mult_pick(SampleArgs a) {
  uint32_t stop;
  // rand < cdf  <=>  cdf > rand
  smp_chain_block<false>(a.logits, a.V, nullptr, a.rand, &stop);
  if (threadIdx.x == 0) *a.out = stop == 0xFFFFFFFFu ? a.V - 1 : stop;
}

// sample_argmax: lowest index among the maxima; a NaN first value is never
// beaten, any other NaN never wins
__global__ void __launch_bounds__(SMP_THREADS) smp_argmax(SampleArgs a) {
  __shared__ float sv[SMP_THREADS / 32];
  __shared__ uint32_t si[SMP_THREADS / 32];
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  for (uint32_t q = threadIdx.x; q < a.V; q += SMP_THREADS) {
    const float v = a.logits[q];
    if (smp_better(v, q, bv, bi)) { bv = v; bi = q; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
    if (smp_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < SMP_THREADS / 32; ++w)
      if (smp_better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    const float l0 = a.logits[0];
    uint32_t res = bi == 0xFFFFFFFFu ? 0u : bi;
    if (l0 != l0) res = 0u;
    *a.out = res;
  }
}

}  // namespace

uint32_t sample_tiles(uint32_t V) { return (V + SMP_TILE - 1) / SMP_TILE; }

size_t sample_sort_temp_bytes(uint32_t V) {
  size_t bytes = 0;
  cub::DoubleBuffer<float> k(nullptr, nullptr);
  cub::DoubleBuffer<uint32_t> v(nullptr, nullptr);
  cub::DeviceRadixSort::SortPairsDescending(nullptr, bytes, k, v, (int)V);
  return bytes;
}

cudaError_t sample(SampleArgs& a, int* cur, const LaunchCfg& lc) {
  if (a.V == 0 || a.ntiles != sample_tiles(a.V)) return cudaErrorInvalidValue;
  cudaStream_t st = lc.stream;
  if (a.temperature == 0.0f) {
    smp_argmax<<<1, SMP_THREADS, 0, st>>>(a);
    return cudaGetLastError();
  }
  smp_scale_max<<<a.ntiles, SMP_THREADS, 0, st>>>(a);
  smp_exp<<<a.ntiles, SMP_THREADS, 0, st>>>(a);
  smp_sum<<<1, SMP_THREADS, 0, st>>>(a);
  smp_norm<<<a.ntiles, SMP_THREADS, 0, st>>>(a);
  if (!a.topp) {
    smp_mult_pick<<<1, SMP_THREADS, 0, st>>>(a);
    return cudaGetLastError();
  }
  SampleArgs b = a;
  b.sprob = a.sbuf_prob[*cur];
  b.sidx = a.sbuf_idx[*cur];
  smp_compact<<<a.ntiles, SMP_THREADS, 0, st>>>(b);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // stable radix sort of the whole persistent array by descending prob
  cub::DoubleBuffer<float> keys(a.sbuf_prob[*cur], a.sbuf_prob[*cur ^ 1]);
  cub::DoubleBuffer<uint32_t> vals(a.sbuf_idx[*cur], a.sbuf_idx[*cur ^ 1]);
  size_t bytes = a.sort_temp_bytes;
  e = cub::DeviceRadixSort::SortPairsDescending(a.sort_temp, bytes, keys, vals, (int)a.V, 0, 32, st);
  if (e != cudaSuccess) return e;
  *cur = keys.selector == 0 ? *cur : *cur ^ 1;
  if (keys.Current() != a.sbuf_prob[*cur] || vals.Current() != a.sbuf_idx[*cur]) return cudaErrorUnknown;
  b.sprob = a.sbuf_prob[*cur];
  b.sidx = a.sbuf_idx[*cur];
  smp_topp_pick<<<1, SMP_THREADS, 0, st>>>(b);
  return cudaGetLastError();
}

}  // namespace k
}  // namespace yl
