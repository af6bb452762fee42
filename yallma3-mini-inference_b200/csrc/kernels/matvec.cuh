// Weight-streaming matvec for decode and small batches (1..8 tokens per pass):
//   out[t][r] = sum_g ((float)isum(t, r, g) * w_scale[r][g]) * x_scale[t][g]
// with isum the exact int32 dot of one 32-element block (weight_type.rs:176-279,
// `matmul_q8_slices`), or the f32 dot of matmul_f32 (weight_type.rs:281-323) for
// F16 weights and for the f32-activation lm_head (forward.rs:261-279).
//
// Design (B200): the op is HBM-bound (one byte of weight per 2 int ops at
// batch 1), so the kernel is built to keep many bytes in flight and never stall
// on compute:
//  * one CTA per SM; warp 0 is a producer that streams the CTA's contiguous
//    range of weight rows into a shared-memory ring with 1-D bulk async copies
//    (cp.async.bulk, TMA engine) completing on mbarriers; weights are marked
//    evict-first in L2;
//  * 8 consumer warps read the ring with 128-bit conflict-free shared loads and
//    do dp4a block dots (exact int32 per 32-element block) and the f32 scale
//    fold; warp w owns RPW rows of every stage;
//  * the producer starts streaming before griddepcontrol.wait, so under
//    programmatic dependent launch the weight fetch of this kernel overlaps the
//    tail of the previous kernel; consumers wait for the activations only.
//  * epilogues: store, residual add, the reference's `+=` quirk, and SwiGLU on
//    interleaved (gate, up) row pairs.
#pragma once
#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {

constexpr int MV_NCW = 8;                   // consumer warps
constexpr int MV_THREADS = 32 * (1 + MV_NCW);

template <int FMT>
__host__ __device__ constexpr uint32_t mv_qbytes(uint32_t kn) {
  return FMT == FMT_Q4 || FMT == FMT_Q4F ? kn / 2 : (FMT == FMT_F16 ? kn * 2 : kn);
}
template <int FMT>
__host__ __device__ constexpr bool mv_has_scales() { return FMT != FMT_F16; }
template <int FMT>
__host__ __device__ constexpr bool mv_f32_act() {
  return FMT == FMT_F16 || FMT == FMT_Q8F || FMT == FMT_Q4F;
}

// Shared-memory layout, computed identically on host and device.
struct MvLayout {
  uint32_t bar_off, x_off, xs_off, xsum_off, ring_off;
  uint32_t stage_q_row, stage_s_row, stage_bytes, total;
};
template <int FMT, int NT>
__host__ __device__ inline MvLayout mv_layout(uint32_t K, uint32_t kc, int rpw, int stages) {
  MvLayout L;
  L.bar_off = 0;
  uint32_t off = 256;
  L.x_off = off;
  if (mv_f32_act<FMT>()) {
    off += NT * K * 4;
    L.xs_off = L.xsum_off = off;
  } else {
    off += NT * K;  // int8 activations (Q4: split lo/hi halves per block)
    off = (off + 15) & ~15u;
    L.xs_off = off;
    off += NT * (K / 32) * 4;
    L.xsum_off = off;
    if (FMT == FMT_Q4) off += NT * (K / 32) * 4;
  }
  off = (off + 127) & ~127u;
  L.ring_off = off;
  L.stage_q_row = mv_qbytes<FMT>(kc);
  L.stage_s_row = mv_has_scales<FMT>() ? kc / 32 * 4 : 0;  // room for f32 scales
  L.stage_bytes = (uint32_t)(MV_NCW * rpw) * (L.stage_q_row + L.stage_s_row);
  L.total = off + stages * L.stage_bytes;
  return L;
}

template <bool SF16>
__device__ __forceinline__ float ld_scale(const uint8_t* base, int idx) {
  if (SF16) return __half2float(reinterpret_cast<const __half*>(base)[idx]);
  return reinterpret_cast<const float*>(base)[idx];
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  // forward.rs:230-235: g / (1 + exp(-g)) * u
  float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

template <int FMT, int NT, int EPI, bool SF16, int RPW>
__global__ void __launch_bounds__(MV_THREADS, 1) mv_kernel(MvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  using namespace yl::dev;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t K = a.K, kc = a.kc;
  const int S = a.stages;
  const MvLayout L = mv_layout<FMT, NT>(K, kc, RPW, S);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + S;

  // Row range of this CTA (row pairs for SwiGLU so gate/up stay together).
  const uint32_t unit = (EPI == EPI_SWIGLU) ? 2u : 1u;
  const uint64_t units = a.rows / unit;
  const uint32_t r_begin = (uint32_t)(units * blockIdx.x / gridDim.x) * unit;
  const uint32_t r_end = (uint32_t)(units * (blockIdx.x + 1) / gridDim.x) * unit;
  const uint32_t RS = MV_NCW * RPW;
  const uint32_t nch = (K + kc - 1) / kc;
  const uint32_t nrs = (r_end - r_begin + RS - 1) / RS;
  const uint32_t n_it = nrs * nch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MV_NCW);
    }
    mbar_fence_init();
  }
  __syncthreads();
  grid_dep_launch();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t issued = 0;
      for (uint32_t it = 0; it < n_it; ++it) {
        const int slot = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait(&empty[slot], ph ^ 1, a.err)) break;
        const uint32_t rs = it / nch, ch = it % nch;
        const uint32_t row0 = r_begin + rs * RS;
        const uint32_t nrows = min(RS, r_end - row0);
        const uint32_t k0 = ch * kc, kn = min(kc, K - k0);
        const uint32_t qb = mv_qbytes<FMT>(kn);
        const uint32_t ssz = SF16 ? 2u : 4u;
        const uint32_t sb = mv_has_scales<FMT>() ? ((kn / 32 * ssz + 15u) & ~15u) : 0u;
        uint8_t* stage = smem + L.ring_off + slot * L.stage_bytes;
        mbar_arrive_expect_tx(&full[slot], nrows * (qb + sb));
        for (uint32_t r = 0; r < nrows; ++r) {
          const uint64_t row = row0 + r;
          bulk_g2s(stage + r * L.stage_q_row, a.wq + row * a.row_bytes + mv_qbytes<FMT>(k0), qb, &full[slot], pol);
          if (sb)
            bulk_g2s(stage + RS * L.stage_q_row + r * L.stage_s_row,
                     a.ws + row * a.scale_row_bytes + (k0 / 32) * ssz, sb, &full[slot], pol);
        }
        issued = it + 1;
      }
      // Drain: no bulk copy may still target this CTA's shared memory at exit.
      // In a healthy run every issued stage was consumed, so this returns at once.
      for (uint32_t it = issued > (uint32_t)S ? issued - S : 0; it < issued; ++it)
        mbar_wait(&full[it % S], (it / S) & 1, a.err, 100000000ull);
    }
    grid_dep_wait();  // every thread of the grid waits before exit (keeps PDL chains transitive)
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  grid_dep_wait();

  // Stage the activations into shared memory.
  if (mv_f32_act<FMT>()) {
    float* xf = reinterpret_cast<float*>(smem + L.x_off);
    for (int t = 0; t < NT; ++t) {
      const float4* src = reinterpret_cast<const float4*>(a.xf + (uint64_t)t * a.x_tok_stride);
      float4* dst = reinterpret_cast<float4*>(xf + t * K);
      const bool valid = t < (int)a.ntok;
      for (uint32_t i = ctid; i < K / 4; i += MV_NCW * 32) dst[i] = valid ? src[i] : make_float4(0, 0, 0, 0);
    }
  } else {
    int8_t* xq = reinterpret_cast<int8_t*>(smem + L.x_off);
    float* xs = reinterpret_cast<float*>(smem + L.xs_off);
    int* xsum = reinterpret_cast<int*>(smem + L.xsum_off);
    const uint32_t nb = K / 32;
    for (int t = 0; t < NT; ++t) {
      const bool valid = t < (int)a.ntok;
      const int4* src = reinterpret_cast<const int4*>(a.xq + (uint64_t)t * a.x_tok_stride);
      if (FMT == FMT_Q4) {
        // split layout: first 16 bytes of every block, then the second halves,
        // so a lane reading one block's halves hits consecutive 16-byte slots
        for (uint32_t b = ctid; b < nb; b += MV_NCW * 32) {
          int4 lo = valid ? src[2 * b] : make_int4(0, 0, 0, 0);
          int4 hi = valid ? src[2 * b + 1] : make_int4(0, 0, 0, 0);
          reinterpret_cast<int4*>(xq + t * K)[b] = lo;
          reinterpret_cast<int4*>(xq + t * K)[nb + b] = hi;
          int s = dp4a(lo.x, 0x01010101, 0);
          s = dp4a(lo.y, 0x01010101, s);
          s = dp4a(lo.z, 0x01010101, s);
          s = dp4a(lo.w, 0x01010101, s);
          s = dp4a(hi.x, 0x01010101, s);
          s = dp4a(hi.y, 0x01010101, s);
          s = dp4a(hi.z, 0x01010101, s);
          s = dp4a(hi.w, 0x01010101, s);
          xsum[t * nb + b] = s;
        }
      } else {
        for (uint32_t i = ctid; i < K / 16; i += MV_NCW * 32)
          reinterpret_cast<int4*>(xq + t * K)[i] = valid ? src[i] : make_int4(0, 0, 0, 0);
      }
      const float* ssrc = a.xs + (uint64_t)t * a.xs_tok_stride;
      for (uint32_t i = ctid; i < nb; i += MV_NCW * 32) xs[t * nb + i] = valid ? ssrc[i] : 0.0f;
    }
  }
  named_bar_sync(1, MV_NCW * 32);

  float acc[RPW][NT];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[r][t] = 0.0f;

  for (uint32_t it = 0; it < n_it; ++it) {
    const int slot = it % S;
    const uint32_t ph = (it / S) & 1;
    const bool ok = mbar_wait(&full[slot], ph, a.err);
    if (!ok) break;
    const uint32_t rs = it / nch, ch = it % nch;
    const uint32_t row0 = r_begin + rs * RS;
    const uint32_t k0 = ch * kc, kn = min(kc, K - k0);
    const uint8_t* stage = smem + L.ring_off + slot * L.stage_bytes;
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
      const uint32_t rl = cw * RPW + rr;
      if (!ok || row0 + rl >= r_end) continue;
      const uint8_t* wrow = stage + rl * L.stage_q_row;
      const uint8_t* srow = stage + RS * L.stage_q_row + rl * L.stage_s_row;
      if (FMT == FMT_Q8) {
        const int8_t* xq = reinterpret_cast<const int8_t*>(smem + L.x_off);
        const float* xs = reinterpret_cast<const float*>(smem + L.xs_off);
        const uint32_t nck = kn / 16;  // 16-byte chunks, two per block
        for (uint32_t c0 = 0; c0 < nck; c0 += 32) {
          const uint32_t c = c0 + lane;
          const bool v = c < nck;
          const int4 w = v ? *reinterpret_cast<const int4*>(wrow + 16 * c) : make_int4(0, 0, 0, 0);
          const float wsc = v ? ld_scale<SF16>(srow, c >> 1) : 0.0f;
          const uint32_t kb = (k0 >> 5) + (c >> 1);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            int4 x = v ? *reinterpret_cast<const int4*>(xq + t * K + k0 + 16 * c) : make_int4(0, 0, 0, 0);
            int s = dp4a(w.x, x.x, 0);
            s = dp4a(w.y, x.y, s);
            s = dp4a(w.z, x.z, s);
            s = dp4a(w.w, x.w, s);
            s += __shfl_xor_sync(FULL, s, 1);  // exact int32 dot of the whole block
            if (v && !(lane & 1)) {
              float p = __fmul_rn(__fmul_rn((float)s, wsc), xs[t * (K / 32) + kb]);
              acc[rr][t] = __fadd_rn(acc[rr][t], p);
            }
          }
        }
      } else if (FMT == FMT_Q4) {
        const int8_t* xq = reinterpret_cast<const int8_t*>(smem + L.x_off);
        const float* xs = reinterpret_cast<const float*>(smem + L.xs_off);
        const int* xsum = reinterpret_cast<const int*>(smem + L.xsum_off);
        const uint32_t nb = K / 32, nbk = kn / 32;  // one 16-byte chunk per block
        for (uint32_t b0 = 0; b0 < nbk; b0 += 32) {
          const uint32_t b = b0 + lane;
          if (b >= nbk) break;
          const int4 w = *reinterpret_cast<const int4*>(wrow + 16 * b);
          const float wsc = ld_scale<SF16>(srow, b);
          const uint32_t kb = (k0 >> 5) + b;
          const int wl[4] = {w.x & 0x0F0F0F0F, w.y & 0x0F0F0F0F, w.z & 0x0F0F0F0F, w.w & 0x0F0F0F0F};
          const int wh[4] = {(w.x >> 4) & 0x0F0F0F0F, (w.y >> 4) & 0x0F0F0F0F, (w.z >> 4) & 0x0F0F0F0F,
                             (w.w >> 4) & 0x0F0F0F0F};
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const int4 xl = reinterpret_cast<const int4*>(xq + t * K)[kb];
            const int4 xh = reinterpret_cast<const int4*>(xq + t * K)[nb + kb];
            int s = dp4a(wl[0], xl.x, 0);
            s = dp4a(wl[1], xl.y, s);
            s = dp4a(wl[2], xl.z, s);
            s = dp4a(wl[3], xl.w, s);
            s = dp4a(wh[0], xh.x, s);
            s = dp4a(wh[1], xh.y, s);
            s = dp4a(wh[2], xh.z, s);
            s = dp4a(wh[3], xh.w, s);
            s -= 8 * xsum[t * nb + kb];  // sum (q-8)*x exactly
            float p = __fmul_rn(__fmul_rn((float)s, wsc), xs[t * nb + kb]);
            acc[rr][t] = __fadd_rn(acc[rr][t], p);
          }
        }
      } else if (FMT == FMT_F16) {
        const float* xf = reinterpret_cast<const float*>(smem + L.x_off);
        const uint32_t nck = kn / 8;  // 8 halves per 16-byte chunk
        for (uint32_t c = lane; c < nck; c += 32) {
          const int4 w = *reinterpret_cast<const int4*>(wrow + 16 * c);
          const __half2* h2 = reinterpret_cast<const __half2*>(&w);
          float wf[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float2 f = __half22float2(h2[j]);
            wf[2 * j] = f.x;
            wf[2 * j + 1] = f.y;
          }
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float4 x0 = *reinterpret_cast<const float4*>(xf + t * K + k0 + 8 * c);
            const float4 x1 = *reinterpret_cast<const float4*>(xf + t * K + k0 + 8 * c + 4);
            float s = acc[rr][t];
            s = __fadd_rn(s, __fmul_rn(x0.x, wf[0]));
            s = __fadd_rn(s, __fmul_rn(x0.y, wf[1]));
            s = __fadd_rn(s, __fmul_rn(x0.z, wf[2]));
            s = __fadd_rn(s, __fmul_rn(x0.w, wf[3]));
            s = __fadd_rn(s, __fmul_rn(x1.x, wf[4]));
            s = __fadd_rn(s, __fmul_rn(x1.y, wf[5]));
            s = __fadd_rn(s, __fmul_rn(x1.z, wf[6]));
            s = __fadd_rn(s, __fmul_rn(x1.w, wf[7]));
            acc[rr][t] = s;
          }
        }
      } else {  // FMT_Q8F / FMT_Q4F: quantized weights, f32 activations (lm_head)
        const float* xf = reinterpret_cast<const float*>(smem + L.x_off);
        if (FMT == FMT_Q8F) {
          const uint32_t nck = kn / 16;
          for (uint32_t c0 = 0; c0 < nck; c0 += 32) {
            const uint32_t c = c0 + lane;
            const bool v = c < nck;
            const int4 w = v ? *reinterpret_cast<const int4*>(wrow + 16 * c) : make_int4(0, 0, 0, 0);
            const float wsc = v ? ld_scale<SF16>(srow, c >> 1) : 0.0f;
            const int8_t* wb = reinterpret_cast<const int8_t*>(&w);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              float s = 0.0f;
              if (v) {
                const float4* xp = reinterpret_cast<const float4*>(xf + t * K + k0 + 16 * c);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float4 x = xp[j];
                  s = fmaf(x.x, (float)wb[4 * j + 0], s);
                  s = fmaf(x.y, (float)wb[4 * j + 1], s);
                  s = fmaf(x.z, (float)wb[4 * j + 2], s);
                  s = fmaf(x.w, (float)wb[4 * j + 3], s);
                }
              }
              s += __shfl_xor_sync(FULL, s, 1);
              if (v && !(lane & 1)) acc[rr][t] = fmaf(s, wsc, acc[rr][t]);
            }
          }
        } else {
          const uint32_t nbk = kn / 32;
          for (uint32_t b = lane; b < nbk; b += 32) {
            const int4 w = *reinterpret_cast<const int4*>(wrow + 16 * b);
            const float wsc = ld_scale<SF16>(srow, b);
            const uint8_t* wb = reinterpret_cast<const uint8_t*>(&w);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              const float* xp = xf + t * K + k0 + 32 * b;
              float s = 0.0f;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                s = fmaf(xp[j], (float)((int)(wb[j] & 0xF) - 8), s);
                s = fmaf(xp[j + 16], (float)((int)(wb[j] >> 4) - 8), s);
              }
              acc[rr][t] = fmaf(s, wsc, acc[rr][t]);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);

    if (ch == nch - 1) {
      // Epilogue for this warp's rows of the finished row set.
#pragma unroll
      for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int rr = 0; rr < RPW; ++rr) acc[rr][t] = warp_sum(acc[rr][t]);
      }
      if (lane == 0 && ok) {
        if (EPI == EPI_SWIGLU) {
          const uint32_t r = row0 + cw * RPW;  // gate row (even), up row = r + 1
          if (r + 1 < r_end) {
#pragma unroll
            for (int t = 0; t < NT; ++t)
              if (t < (int)a.ntok) a.out[(uint64_t)t * a.out_tok_stride + r / 2] = silu_mul(acc[0][t], acc[1][t]);
          }
        } else {
#pragma unroll
          for (int rr = 0; rr < RPW; ++rr) {
            const uint32_t r = row0 + cw * RPW + rr;
            if (r >= r_end) continue;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              if (t >= (int)a.ntok) continue;
              float* o = a.out + (uint64_t)t * a.out_tok_stride + r;
              if (EPI == EPI_STORE) *o = acc[rr][t];
              else if (EPI == EPI_ADD) *o = __fadd_rn(*o, acc[rr][t]);
              else *o = (r < a.quirk_cols) ? __fadd_rn(*o, acc[rr][t]) : acc[rr][t];
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int rr = 0; rr < RPW; ++rr) acc[rr][t] = 0.0f;
    }
  }
}

// Host-side launcher for one (FMT, SF16) family; NT and EPI dispatched here.
template <int FMT, bool SF16>
cudaError_t mv_launch(const MvArgs& a0, int epi, const LaunchCfg& lc) {
  MvArgs a = a0;
  const int nt = a.ntok <= 1 ? 1 : a.ntok <= 2 ? 2 : a.ntok <= 4 ? 4 : 8;
  const int rpw = epi == EPI_SWIGLU ? 2 : 1;
  // Stage count from the shared-memory budget.
  MvLayout L0;
  switch (nt) {
    case 1: L0 = mv_layout<FMT, 1>(a.K, a.kc, rpw, 0); break;
    case 2: L0 = mv_layout<FMT, 2>(a.K, a.kc, rpw, 0); break;
    case 4: L0 = mv_layout<FMT, 4>(a.K, a.kc, rpw, 0); break;
    default: L0 = mv_layout<FMT, 8>(a.K, a.kc, rpw, 0); break;
  }
  int stages = (int)((lc.smem_budget > L0.total ? lc.smem_budget - L0.total : 0) / L0.stage_bytes);
  if (stages > 8) stages = 8;
  if (stages < 2) stages = 2;
  a.stages = stages;
  const uint32_t smem = L0.total + stages * L0.stage_bytes;
  if (smem > 227u * 1024u) return cudaErrorInvalidConfiguration;
  void (*kern)(MvArgs) = nullptr;
#define YL_MV_CASE(NT_, EPI_, RPW_) \
  if (nt == NT_ && epi == EPI_) kern = mv_kernel<FMT, NT_, EPI_, SF16, RPW_>;
#define YL_MV_NT(NT_)                   \
  YL_MV_CASE(NT_, EPI_STORE, 1)         \
  YL_MV_CASE(NT_, EPI_ADD, 1)           \
  YL_MV_CASE(NT_, EPI_QUIRK, 1)         \
  if (!mv_f32_act<FMT>() || FMT == FMT_F16) { YL_MV_CASE(NT_, EPI_SWIGLU, 2) }
  YL_MV_NT(1)
  YL_MV_NT(2)
  YL_MV_NT(4)
  YL_MV_NT(8)
#undef YL_MV_NT
#undef YL_MV_CASE
  if (!kern) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  uint32_t grid = lc.grid ? lc.grid : 148;
  const uint32_t unit = epi == EPI_SWIGLU ? 2 : 1;
  if (grid > a.rows / unit) grid = (uint32_t)(a.rows / unit);
  if (grid == 0) return cudaSuccess;
  return launch_kernel(kern, dim3(grid), dim3(MV_THREADS), smem, lc, a);
}

}  // namespace k
}  // namespace yl
