// Decode matvec for one token with Q8_0 weights (f16 or f32 scales) and int8
// activations, the per-token hot loop of forward.rs:148-254:
//   out[r] = ((0 + t_0) + t_1) + ... ,  t_g = ((f32)isum(r, g) * ws[r][g]) * xs[g]
// with isum the exact int32 dot of 32-element block g (weight_type.rs:122-226,
// the sequential `+=` over groups at :190-201), so every output equals the
// reference's bit for bit.
//
// Layout of the work (B200):
//  * a CTA owns a contiguous range of 8-row groups; one warp processes a
//    group with 4 lanes per row, lane (r, j) computing the whole int32 dot of
//    block 4s + j of row r in step s (two 16-byte weight loads, two broadcast
//    activation loads, eight dp4a), so a row's chain of block terms lives in
//    ONE register of lane (r, 0), which adds the four terms of a step in block
//    order after three shuffles (no fold warp, no term staging);
//  * a stage is one group x one K-chunk (8 rows x up to 1 KB): one 3-D TMA box
//    of chunks x 8 rows x 128 bytes with 128-byte swizzle (lane r reads 16-byte
//    chunk m of its row at chunk m ^ r, so the lanes' loads are conflict-free)
//    plus one 2-D box of the group's scales for the chunk;
//  * the ring (up to 16 stages) is split into one sub-ring per consumer warp:
//    a slot only ever carries stages of one warp, in that warp's order, so
//    every mbarrier wait is exactly one phase after the previous use of the
//    slot and the parity cannot alias (with slots shared between warps, a warp
//    could pass a wait on a phase another warp's earlier stage has not yet
//    completed);
//  * one producer thread issues the stages (K-chunk outer, group inner; group
//    g belongs to warp g % 8) with L2 evict-first hints, from before the wait
//    on the previous kernel (programmatic dependent launch).
// Prologues: PRO_LOAD (stage int8 activations), PRO_NORM (RMSNorm in the
// reference's 8-lane order + Q8_0 quantization). Epilogues: store, residual
// add, SwiGLU on interleaved (gate, up) rows with Q8_0 quantization of h.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {

namespace {

using namespace yl::dev;

constexpr int M2_NCW = 8;                       // consumer warps
constexpr int M2_THREADS = 32 * (M2_NCW + 1);   // + one producer warp
constexpr int M2_MAXT = 8;                      // groups per consumer warp at most
constexpr int M2_MAXS = 16;                     // ring stages at most

struct M2Layout {
  uint32_t bar, red, x, xs, stg, ring, sring, sq_bytes, ss_bytes, total;
};

// Shared memory: barriers, broadcast slots, the activation row (int8 + f32
// scales), the RMSNorm staging row, then the ring: `stages` quant tiles of
// sq_bytes (1024-byte aligned, for the 128-byte swizzle) followed by the
// stages' scale tiles of ss_bytes. sbytes: scale bytes of one row for one
// K-chunk.
__host__ __device__ inline M2Layout m2_layout(uint32_t K, uint32_t kc, uint32_t sbytes, int stages, bool norm) {
  M2Layout L;
  L.bar = 0;    // full[16], empty[16]
  L.red = 256;  // broadcast slots
  uint32_t off = 512;
  L.x = off;
  off = (off + K + 15u) & ~15u;
  L.xs = off;
  off = (off + K / 32 * 4 + 15u) & ~15u;
  L.stg = off;
  if (norm) off += K * 4;
  off = (off + 1023u) & ~1023u;
  L.ring = off;
  L.sq_bytes = kc / 128 * 1024;              // kc/128 tiles of 8 rows x 128 bytes
  L.ss_bytes = (8 * sbytes + 127u) & ~127u;  // scale tiles land 128-byte aligned
  L.sring = (uint32_t)stages * L.sq_bytes;   // from the aligned ring start
  // + 1 KB of slack: the ring starts at the first 1024-byte aligned shared
  // address at or after `ring`
  L.total = off + (uint32_t)stages * (L.sq_bytes + L.ss_bytes) + 1024u;
  return L;
}

// 3-D tiled TMA load of this GPU's memory (no multicast)
__device__ __forceinline__ void tma_3d_hint(void* dst, const CUtensorMap* map, uint32_t x, uint32_t y, uint32_t z,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// 2-D tiled TMA load of this GPU's memory (no multicast)
__device__ __forceinline__ void tma_2d_hint(void* dst, const CUtensorMap* map, uint32_t x, uint32_t y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

template <bool SF16, int EPI, int PRO>
__global__ void __launch_bounds__(M2_THREADS, 2)
    mv2_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap ms, const Mv2Args a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t K = a.K, kc = a.kc, nkc = K / kc, nb = K / 32;
  const int S = a.stages;
  constexpr uint32_t ssz = SF16 ? 2u : 4u;
  const uint32_t sbytes = kc / 32 * ssz;
  const M2Layout L = m2_layout(K, kc, sbytes, S, PRO == PRO_NORM);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar);
  uint64_t* empty = full + M2_MAXS;
  const uint32_t sbase = smem_u32(smem);
  uint8_t* const ring = smem + (((sbase + L.ring + 1023u) & ~1023u) - sbase);
  uint8_t* const sring = ring + L.sring;
  const uint32_t NG = (a.rows + 7u) / 8u;
  const uint32_t g0 = (uint32_t)((uint64_t)NG * blockIdx.x / gridDim.x);
  const uint32_t g1 = (uint32_t)((uint64_t)NG * (blockIdx.x + 1) / gridDim.x);
  const uint32_t ng = g1 - g0;
  const uint32_t A = ng < (uint32_t)M2_NCW ? ng : (uint32_t)M2_NCW;  // warps that own groups
  const uint32_t Sw = A ? (uint32_t)S / A : 0u;                       // sub-ring slots per warp
  if (S < 1 || S > M2_MAXS || ng > (uint32_t)(M2_NCW * M2_MAXT) || (ng && Sw < 1)) {  // never planned
    if (threadIdx.x == 0 && a.err) atomicExch(a.err, ERR_BAD_ARG);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  grid_dep_launch();

  if (warp == M2_NCW) {
    // ---------------- producer ----------------
    if (lane == 0 && ng > 0) {
      const uint64_t pol = l2_evict_first_policy();
      // per-warp position in its sub-ring (slot, phase) and stages issued
      uint32_t kslot[M2_NCW], kph[M2_NCW], kw[M2_NCW];
#pragma unroll
      for (int w = 0; w < M2_NCW; ++w) kslot[w] = kph[w] = kw[w] = 0;
      const uint32_t nchunk = kc / 128;
      bool ok = true;
      for (uint32_t c = 0; c < nkc && ok; ++c) {
        for (uint32_t gi = 0; gi < ng; ++gi) {
          const uint32_t w = gi & (M2_NCW - 1);
          const uint32_t slot = w * Sw + kslot[w];
          if (!mbar_wait(&empty[slot], kph[w] ^ 1u, a.err)) {
            ok = false;
            break;
          }
          const uint32_t row = (g0 + gi) * 8u;
          mbar_arrive_expect_tx(&full[slot], L.sq_bytes + 8u * sbytes);
          tma_3d_hint(ring + slot * L.sq_bytes, &mq, 0u, row, c * nchunk, &full[slot], pol);
          tma_2d_hint(sring + slot * L.ss_bytes, &ms, c * sbytes, row, &full[slot], pol);
          ++kw[w];
          if (++kslot[w] == Sw) {
            kslot[w] = 0;
            kph[w] ^= 1u;
          }
        }
      }
      // Drain: no copy may still target this CTA's shared memory at exit. The
      // last stage issued on each slot of each warp's sub-ring is waited on
      // with its own parity (no later phase exists on that slot); in a
      // healthy run every stage was consumed and this returns at once.
      for (uint32_t w = 0; w < A; ++w) {
        const uint32_t n = kw[w];
        for (uint32_t s2 = 0; s2 < Sw && s2 < n; ++s2) {
          const uint32_t kl = n - 1 - ((n - 1 - s2) % Sw);
          mbar_wait(&full[w * Sw + kl % Sw], (kl / Sw) & 1u, a.err, 100000000ull);
        }
      }
    }
    grid_dep_wait();  // every thread of the grid waits before exit (keeps PDL chains transitive)
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp, ctid = cw * 32 + lane;
  float* red = reinterpret_cast<float*>(smem + L.red);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + L.x);
  float* xsm = reinterpret_cast<float*>(smem + L.xs);
  if (PRO == PRO_NORM) {
    grid_dep_wait();
    float* stg = reinterpret_cast<float*>(smem + L.stg);
    for (uint32_t i = ctid * 4; i < K; i += M2_NCW * 32 * 4)
      *reinterpret_cast<float4*>(stg + i) = *reinterpret_cast<const float4*>(a.xres + i);
    named_bar_sync(1, M2_NCW * 32);
    if (cw == 0) {
      const float r = rms_factor_smem8(stg, K, a.eps, lane);  // util.rs:389-426 order
      if (lane == 0) red[0] = r;
    }
    named_bar_sync(1, M2_NCW * 32);
    const float r = red[0];
    for (uint32_t b = cw; b < nb; b += M2_NCW) {  // quantization.rs:29-52, one block per warp pass
      const uint32_t k = b * 32 + lane;
      const float y = __fmul_rn(a.norm_w[k], __fmul_rn(r, stg[k]));
      float sc;
      xq[k] = quant_q8_lane(y, &sc);
      if (lane == 0) xsm[b] = sc;
    }
  } else {
    grid_dep_wait();
    for (uint32_t i = ctid; i < K / 16; i += M2_NCW * 32)
      reinterpret_cast<int4*>(xq)[i] = reinterpret_cast<const int4*>(a.xq)[i];
    for (uint32_t i = ctid; i < nb; i += M2_NCW * 32) xsm[i] = a.xs[i];
  }
  named_bar_sync(1, M2_NCW * 32);

  const int r = lane >> 2, j = lane & 3;
  uint32_t my_slot = 0, my_ph = 0;  // position in this warp's sub-ring
  float chain[M2_MAXT];
#pragma unroll
  for (int t = 0; t < M2_MAXT; ++t) chain[t] = 0.0f;
  bool dead = false;
  for (uint32_t c = 0; c < nkc && !dead; ++c) {
#pragma unroll
    for (int t = 0; t < M2_MAXT; ++t) {
      const uint32_t gi = (uint32_t)cw + M2_NCW * (uint32_t)t;
      if (gi >= ng) break;  // warp-uniform
      const uint32_t slot = (uint32_t)cw * Sw + my_slot, ph = my_ph;
      if (++my_slot == Sw) {
        my_slot = 0;
        my_ph ^= 1u;
      }
      // warp-uniform wait: lane 0 polls, the outcome is broadcast, and the
      // warp barrier orders the lanes' reads after the observed completion
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&full[slot], ph, a.err) ? 1 : 0;
      ok = __shfl_sync(FULL, ok, 0);
      __syncwarp();
      if (!ok) {
        dead = true;
        break;
      }
      const uint8_t* st = ring + slot * L.sq_bytes;
      const uint8_t* srow = sring + slot * L.ss_bytes + (uint32_t)r * sbytes;
      float ch = chain[t];
      const uint32_t kb0 = c * (kc / 32);
      for (uint32_t s = 0; s < kc / 128; ++s) {
        const uint8_t* line = st + s * 1024u + (uint32_t)r * 128u;
        const int4 w0 = *reinterpret_cast<const int4*>(line + ((uint32_t)((2 * j) ^ r) << 4));
        const int4 w1 = *reinterpret_cast<const int4*>(line + ((uint32_t)((2 * j + 1) ^ r) << 4));
        const uint32_t kb = kb0 + s * 4u + (uint32_t)j;
        const int4 x0 = *reinterpret_cast<const int4*>(xq + kb * 32u);
        const int4 x1 = *reinterpret_cast<const int4*>(xq + kb * 32u + 16u);
        int d = dp4a(w0.x, x0.x, 0);
        d = dp4a(w0.y, x0.y, d);
        d = dp4a(w0.z, x0.z, d);
        d = dp4a(w0.w, x0.w, d);
        d = dp4a(w1.x, x1.x, d);
        d = dp4a(w1.y, x1.y, d);
        d = dp4a(w1.z, x1.z, d);
        d = dp4a(w1.w, x1.w, d);
        const uint32_t si = s * 4u + (uint32_t)j;
        const float ws = SF16 ? __half2float(reinterpret_cast<const __half*>(srow)[si])
                              : reinterpret_cast<const float*>(srow)[si];
        // block term ((f32)isum * ws) * xs (|isum| < 2^24: the conversion is exact)
        const float p = __fmul_rn(__fmul_rn((float)d, ws), xsm[kb]);
        const float p1 = __shfl_down_sync(FULL, p, 1);
        const float p2 = __shfl_down_sync(FULL, p, 2);
        const float p3 = __shfl_down_sync(FULL, p, 3);
        ch = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(ch, p), p1), p2), p3);  // lanes j == 0 keep theirs
      }
      chain[t] = ch;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // this group's stage is consumed
      if (c == nkc - 1) {
        // ---- epilogue of the group: lane (r, 0) holds row (g0 + gi) * 8 + r ----
        const uint32_t row = (g0 + gi) * 8u + (uint32_t)r;
        if (EPI == EPI_SWIGLU_Q8) {
          const float up = __shfl_down_sync(FULL, ch, 4);  // rows 2i (gate) and 2i + 1 (up)
          if (j == 0 && !(r & 1) && row + 1 < a.rows) a.out[row / 2] = silu_mul(ch, up);
        } else if (j == 0 && row < a.rows) {
          if (EPI == EPI_STORE) a.out[row] = ch;
          else a.out[row] = __fadd_rn(a.out[row], ch);  // EPI_ADD: the residual add
        }
      }
    }
  }

  if (EPI == EPI_SWIGLU_Q8) {
    // h = out[j0, j1) of this CTA: blocks inside it are quantized here, a
    // block shared with a neighbouring CTA by whichever completes it last
    // (per-block arrival counters, zero between launches)
    __threadfence();
    named_bar_sync(1, M2_NCW * 32);
    int* sw_last = reinterpret_cast<int*>(smem + L.red) + 4;
    const uint32_t j0 = g0 * 4u, j1 = min(g1 * 8u, a.rows) / 2u;
    const uint32_t b0 = j0 / 32u, b1 = (j1 + 31u) / 32u;
    if (cw == 0 && lane < 2) {
      const uint32_t b = lane == 0 ? b0 : b1 - 1;
      const uint32_t lo = max(j0, b * 32u), hi = min(j1, b * 32u + 32u);
      const bool partial = j1 > j0 && hi - lo < 32u && (lane == 0 || b1 - 1 != b0);
      int last = 0;
      if (partial) last = atomicAdd(a.hcount + b, hi - lo) + (hi - lo) == 32u;
      sw_last[lane] = partial ? last : 1;
    }
    named_bar_sync(1, M2_NCW * 32);
    if (j1 > j0) {
      for (uint32_t b = b0 + cw; b < b1; b += M2_NCW) {
        const bool first = b == b0, lastb = b == b1 - 1;
        if ((first && !sw_last[0]) || (lastb && !sw_last[1])) continue;  // a neighbour finishes it
        if (first || lastb) __threadfence();  // see the neighbour's h values
        const uint32_t hk = b * 32u + lane;
        float sc;
        const int8_t qv = quant_q8_lane(__ldcg(a.out + hk), &sc);
        a.hq[hk] = qv;
        if (lane == 0) {
          a.hs[b] = sc;
          if (b * 32u < j0 || b * 32u + 32u > j1) a.hcount[b] = 0u;  // for the next launch
        }
      }
    }
  }
  grid_dep_wait();  // every thread of the grid waits before exit
}

// cuTensorMapEncodeTiled through the runtime's entry-point query
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn m2_encode_fn() {
  static EncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeFn>(p);
  }();
  return fn;
}

// The scales [rows][width] bytes (row stride `stride`), tiles box_w bytes x 8 rows
bool m2_encode_scales(CUtensorMap* m, const void* base, uint64_t width, uint64_t rows, uint64_t stride,
                      uint32_t box_w) {
  EncodeFn fn = m2_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {width, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {box_w, 8};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The quants [rows][K] (row stride `stride`) as a 3-D tensor {128 bytes,
// rows, K/128 chunks} (chunk stride 128 bytes): one box of {128, 8, nchunk}
// brings 8 rows x nchunk*128 bytes, each 128-byte row swizzled, chunk c of
// the box at c * 1024 bytes of the destination.
bool m2_encode_quants(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint64_t stride, uint32_t nchunk) {
  EncodeFn fn = m2_encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {128, rows, K / 128};
  const cuuint64_t strides[2] = {stride, 128};
  const cuuint32_t box[3] = {128, 8, nchunk};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool SF16, int EPI, int PRO>
cudaError_t m2_launch(const CUtensorMap& mq, const CUtensorMap& ms, const Mv2Args& a, uint32_t grid, uint32_t smem,
                      const LaunchCfg& lc) {
  cudaError_t e = cudaFuncSetAttribute(mv2_kernel<SF16, EPI, PRO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  return launch_kernel(mv2_kernel<SF16, EPI, PRO>, dim3(grid), dim3(M2_THREADS), smem, lc, mq, ms, a);
}

template <bool SF16, int PRO>
cudaError_t m2_epi(const CUtensorMap& mq, const CUtensorMap& ms, const Mv2Args& a, int epi, uint32_t grid,
                   uint32_t smem, const LaunchCfg& lc) {
  switch (epi) {
    case EPI_STORE: return m2_launch<SF16, EPI_STORE, PRO>(mq, ms, a, grid, smem, lc);
    case EPI_ADD: return m2_launch<SF16, EPI_ADD, PRO>(mq, ms, a, grid, smem, lc);
    case EPI_SWIGLU_Q8: return m2_launch<SF16, EPI_SWIGLU_Q8, PRO>(mq, ms, a, grid, smem, lc);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool matvec2_supported(const MvArgs& a, int fmt, bool sf16, int epi) {
  (void)sf16;
  if (fmt != FMT_Q8 || a.ntok != 1 || a.tp_mode != 0 || a.trace) return false;
  if (a.pro != PRO_LOAD && a.pro != PRO_NORM) return false;
  if (epi != EPI_STORE && epi != EPI_ADD && epi != EPI_SWIGLU_Q8) return false;
  if (a.K % 256 || a.K == 0 || a.rows == 0 || a.row_bytes < a.K || a.row_bytes % 16 || a.scale_row_bytes % 16)
    return false;
  if ((uintptr_t)a.wq % 16 || (uintptr_t)a.ws % 16) return false;
  if (a.pro == PRO_NORM && (!a.xres || !a.norm_w || (uintptr_t)a.xres % 16)) return false;
  if (a.pro == PRO_LOAD && (!a.xq || !a.xs || (uintptr_t)a.xq % 16)) return false;
  if (epi == EPI_SWIGLU_Q8 && (a.rows % 64 || !a.hq || !a.hs || !a.hcount)) return false;
  return m2_encode_fn() != nullptr;
}

cudaError_t matvec2(const MvArgs& a, bool sf16, int epi, uint32_t ctas_per_sm, uint32_t kc_pref,
                    const LaunchCfg& lc) {
  if (!matvec2_supported(a, FMT_Q8, sf16, epi)) return cudaErrorInvalidValue;
  const uint32_t nsm = lc.grid ? lc.grid : 148u;
  const uint32_t NG = (a.rows + 7u) / 8u;
  const uint32_t grid = std::min<uint32_t>(nsm * std::max<uint32_t>(1u, ctas_per_sm), NG);
  const uint32_t ngmax = (NG + grid - 1) / grid;
  if (ngmax > (uint32_t)(M2_NCW * M2_MAXT)) return cudaErrorInvalidValue;
  const uint32_t A = std::min<uint32_t>(ngmax, M2_NCW);
  // K-chunk: the largest of 1024 / 512 / 256 bytes that divides K and leaves
  // every active warp a sub-ring of two stages (or the preferred chunk)
  uint32_t kc = 0, sbytes = 0;
  int stages = 0;
  M2Layout L0{};
  for (uint32_t cand : {1024u, 512u, 256u}) {
    if (a.K % cand || (kc_pref && cand != kc_pref)) continue;
    const uint32_t sb = cand / 32 * (sf16 ? 2u : 4u);
    const M2Layout L = m2_layout(a.K, cand, sb, 0, a.pro == PRO_NORM);
    int st = (int)((lc.smem_budget > L.total ? lc.smem_budget - L.total : 0) / (L.sq_bytes + L.ss_bytes));
    st = std::min(st, M2_MAXS);
    if (st < (int)A) continue;
    kc = cand;
    sbytes = sb;
    stages = st;
    L0 = L;
    if (st >= 2 * (int)A) break;
  }
  if (kc == 0) return cudaErrorInvalidConfiguration;
  stages = (int)((uint32_t)stages / A * A);  // whole sub-rings
  const uint32_t smem = L0.total + (uint32_t)stages * (L0.sq_bytes + L0.ss_bytes);
  if (smem > 227u * 1024u) return cudaErrorInvalidConfiguration;
  CUtensorMap mq, ms;
  if (!m2_encode_quants(&mq, a.wq, a.K, a.rows, a.row_bytes, kc / 128) ||
      !m2_encode_scales(&ms, a.ws, a.scale_row_bytes, a.rows, a.scale_row_bytes, sbytes))
    return cudaErrorInvalidValue;
  Mv2Args b{};
  b.rows = a.rows;
  b.K = a.K;
  b.kc = kc;
  b.stages = stages;
  b.xq = a.xq;
  b.xs = a.xs;
  b.xres = a.xres;
  b.norm_w = a.norm_w;
  b.eps = a.eps;
  b.out = a.out;
  b.hq = a.hq;
  b.hs = a.hs;
  b.hcount = a.hcount;
  b.err = a.err;
  if (a.pro == PRO_NORM)
    return sf16 ? m2_epi<true, PRO_NORM>(mq, ms, b, epi, grid, smem, lc)
                : m2_epi<false, PRO_NORM>(mq, ms, b, epi, grid, smem, lc);
  return sf16 ? m2_epi<true, PRO_LOAD>(mq, ms, b, epi, grid, smem, lc)
              : m2_epi<false, PRO_LOAD>(mq, ms, b, epi, grid, smem, lc);
}

}  // namespace k
}  // namespace yl
