// Weight-streaming matvec for decode and small batches (1..8 tokens per pass):
//   out[t][r] = sum_g ((float)isum(t, r, g) * w_scale[r][g]) * x_scale[t][g]
// with isum the exact int32 dot of one 32-element block (weight_type.rs:122-226,
// `matmul_q8_slices`), or the f32 dot of matmul_f32 (weight_type.rs:228-270) for
// F16 weights and for the f32-activation lm_head (forward.rs:261-279).
//
// Design (B200): the op is HBM-bound (one byte of weight per 2 int ops at
// batch 1), so the kernel is built to keep many bytes in flight and never stall
// on compute:
//  * one CTA per SM; warp 0 is a producer that streams the CTA's contiguous
//    range of weight rows into a shared-memory ring with 1-D bulk async copies
//    (cp.async.bulk, TMA engine) completing on mbarriers; weights are marked
//    evict-first in L2;
//  * 8 consumer warps read the ring with 128-bit conflict-free shared loads,
//    four independent chunks in flight per lane, and do dp4a block dots (exact
//    int32 per 32-element block) and the f32 scale fold;
//  * the producer starts streaming before griddepcontrol.wait, so under
//    programmatic dependent launch the weight fetch overlaps the tail of the
//    previous kernel; consumers wait for the activations only;
//  * prologue PRO_NORM fuses the RMSNorm + Q8_0 quantization of the residual
//    stream (each CTA normalizes the row itself, a few KB from L2);
//  * epilogues: store, residual add, the reference's `+=` quirk, SwiGLU on
//    interleaved (gate, up) row pairs (optionally quantizing h per 32-block),
//    and logits + greedy argmax.
#pragma once
#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {

constexpr int MV_NCW = 8;                   // consumer warps
constexpr int MV_THREADS = 32 * (1 + MV_NCW);
constexpr int MV_U = 4;                     // 16-byte chunks in flight per lane

template <int FMT>
__host__ __device__ constexpr uint32_t mv_qbytes(uint32_t kn) {
  return FMT == FMT_Q4 || FMT == FMT_Q4F ? kn / 2 : (FMT == FMT_F16 ? kn * 2 : kn);
}
template <int FMT>
__host__ __device__ constexpr bool mv_has_scales() { return FMT != FMT_F16; }
// Int8-activation formats fold the block terms ((f32)isum * ws) * xs of a row
// in group order into one f32 chain, as matmul_q8_slices does
// (weight_type.rs:190-201), so their outputs equal the reference's bit for bit.
template <int FMT>
__host__ __device__ constexpr bool mv_exact_fold() { return FMT == FMT_Q8 || FMT == FMT_Q4; }
constexpr uint32_t MV_TERMS = 64;  // block terms one warp pass produces per token
// Single-token passes of those formats hand the fold to a tenth warp: the
// consumer warps write each stage's block terms into the stage's fold slot
// and move on; the fold warp walks the rows' addition chains (lane r = row r
// of the stage) and runs the epilogue. Multi-token passes fold in-warp.
template <int FMT, int NT>
__host__ __device__ constexpr bool mv_fold_warp() { return mv_exact_fold<FMT>() && NT == 1; }
template <int FMT, int NT>
__host__ __device__ constexpr int mv_threads() { return 32 * (1 + MV_NCW + (mv_fold_warp<FMT, NT>() ? 1 : 0)); }
constexpr int MV_FOLD_WARP = 1 + MV_NCW;  // warp index of the fold warp
template <int FMT>
__host__ __device__ constexpr bool mv_f32_act() {
  return FMT == FMT_F16 || FMT == FMT_Q8F || FMT == FMT_Q4F;
}
__host__ __device__ constexpr bool mv_swiglu(int epi) { return epi == EPI_SWIGLU || epi == EPI_SWIGLU_Q8; }
// Consumer groups: SwiGLU stages hold row pairs (twice the bytes of a row), so
// its ring is split into two groups of four warps to keep two stages in the
// budget; every other epilogue uses one group of eight warps.
__host__ __device__ constexpr int mv_groups(int epi) { return mv_swiglu(epi) ? 2 : 1; }
// Rows per stage (MV_NCW / groups warps x rows per warp): 8 for every epilogue.
constexpr uint32_t MV_RS = 8;
// Dynamic SwiGLU+quantize: row sets one CTA may take (its h blocks are
// quantized from this list at the end).
constexpr uint32_t MV_LIST = 32;
constexpr uint32_t MV_END = 0xFFFFFFFFu;  // stage info: no more row sets

// Shared-memory layout, computed identically on host and device.
struct MvLayout {
  uint32_t bar_off, info_off, red_off, fbar_off, x_off, xs_off, xsum_off, nstage_off, terms_off, ring_off;
  uint32_t stage_q_row, stage_s_row, stage_bytes, total;
  // fold warp: each stage slot carries, after its weight rows, a header
  // {first row, row count} (16 bytes) and MV_RS rows of fold_row floats
  uint32_t fold_off, fold_row;
};
// ssz: weight scale element size (2 for f16, 4 for f32). A stage's scale row
// is the chunk's scales padded to 16 bytes, which for a full-row chunk equals
// the HBM scale row stride, so full-row stages are single contiguous copies.
// groups: consumer groups; a stage holds the rows of one group (MV_NCW/groups
// warps x rpw rows each).
template <int FMT, int NT>
// norm_stage: the RMSNorm prologue stages one f32 row (K floats, at
// nstage_off) to walk the reference-order sum-of-squares chains from shared
// memory.
__host__ __device__ inline MvLayout mv_layout(uint32_t K, uint32_t kc, int rpw, int stages, uint32_t ssz = 4,
                                             int groups = 1, bool norm_stage = false) {
  MvLayout L;
  L.bar_off = 0;       // 2 x 16 mbarriers
  L.info_off = 256;    // per slot: first row and row count; row-set list (dynamic SwiGLU)
  L.red_off = 768;     // reductions / argmax / h staging ([2][8][32] floats)
  L.fbar_off = 2816;   // fold warp: 2 x 16 mbarriers (fold slot full / free)
  uint32_t off = 2816 + 256 + 128;
  L.x_off = off;
  if (mv_f32_act<FMT>()) {
    off += NT * K * 4;
    L.xs_off = L.xsum_off = off;
  } else {
    // int8 activations (Q4: split lo/hi halves per block; Q8X: three limb
    // arrays of NT*K bytes each)
    off += (FMT == FMT_Q8X ? 3 : 1) * NT * K;
    off = (off + 15) & ~15u;
    L.xs_off = off;
    off += NT * (K / 32) * 4;
    L.xsum_off = off;
    if (FMT == FMT_Q4) off += NT * (K / 32) * 4;
  }
  off = (off + 15) & ~15u;
  // RMSNorm prologue: one f32 row staged for the sum-of-squares chains. A
  // single-token pass overlays it on the activation area (its chains finish
  // before the quantized row is written there); several tokens need their
  // own area (earlier tokens' quantized rows stay in place).
  L.nstage_off = NT == 1 ? L.x_off : off;
  if (norm_stage) {
    if (NT == 1) off = off > L.x_off + K * 4 ? off : L.x_off + K * 4;
    else off += K * 4;
  }
  L.terms_off = off;  // per consumer warp: [NT][MV_TERMS] block terms of one pass (in-warp fold)
  if (mv_exact_fold<FMT>() && !mv_fold_warp<FMT, NT>()) off += MV_NCW * NT * MV_TERMS * 4;
  off = (off + 127) & ~127u;
  L.ring_off = off;
  L.stage_q_row = mv_qbytes<FMT>(kc);
  L.stage_s_row = mv_has_scales<FMT>() ? ((kc / 32 * ssz + 15u) & ~15u) : 0;
  L.stage_bytes = (uint32_t)(MV_NCW / groups * rpw) * (L.stage_q_row + L.stage_s_row);
  L.fold_off = L.fold_row = 0;
  if (mv_fold_warp<FMT, NT>()) {
    // padded rows: lane r of the fold warp reads row r at a 16-byte offset
    // from its neighbours, so the eight lanes' float4 loads are conflict-free
    L.fold_off = (L.stage_bytes + 15u) & ~15u;
    L.fold_row = kc / 32 + 4;
    L.stage_bytes = L.fold_off + 16 + MV_RS * L.fold_row * 4;
    L.stage_bytes = (L.stage_bytes + 127u) & ~127u;
  }
  L.total = off + stages * L.stage_bytes;
  return L;
}

template <bool SF16>
__device__ __forceinline__ float ld_scale(const uint8_t* base, int idx) {
  if (SF16) return __half2float(reinterpret_cast<const __half*>(base)[idx]);
  return reinterpret_cast<const float*>(base)[idx];
}


// int8 -> f32 for 4 packed bytes without the (quarter-rate) I2F unit:
// 0x4B000000 | (b ^ 0x80) is the float 2^23 + b + 128, exact.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  const uint32_t u = w ^ 0x80808080u;
  f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
  f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
  f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
  f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

// Exact int -> f32 for |v| < 2^22 on the integer and FMA pipes (the I2F unit
// runs at a quarter of their rate): 0x4B400000 + v is the float 1.5*2^23 + v.
__device__ __forceinline__ float small_i2f(int v) {
  return __int_as_float(0x4B400000 + v) - 12582912.0f;
}

__device__ __forceinline__ bool am_better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// ---------------------------------------------------------------------------
// RMSNorm + quantize prologue with the row held in registers (K <= 8192):
// thread ctid owns float4 i = 4*ctid + 1024*u, so every x and norm-weight load
// is issued in one round trip, and a 32-element block sits in 8 lanes x 4
// values (its absmax is an 8-lane reduction). Same sum-of-squares order as
// rmsnorm_quant_kernel and the same per-element operations as
// quant_q8_lane, so the bits equal the standalone kernels'.
// NORM = false: the rows are quantized as they are (y = x, PRO_QUANT).
// Consumers wait here for the kernel that produced the activations
// (programmatic dependent launch); everything before it overlaps that kernel.
__device__ __forceinline__ void mv_wait_inputs(const MvArgs& a) {
  yl::dev::grid_dep_wait();
  if (yl::dev::kTrace && a.trace && threadIdx.x == 32) a.trace[(uint64_t)blockIdx.x * 8 + 2] = yl::dev::globaltimer();
}

constexpr int MV_NORM_MU = 8;    // float4 per thread with a norm (K <= 8192)
constexpr int MV_QUANT_MU = 16;  // float4 per thread without (K <= 16384)
template <int FMT, int NT, bool NORM, int MU>
__device__ __forceinline__ void mv_norm_regs(const MvArgs& a, const MvLayout& L, uint8_t* smem, int cw, int lane) {
  using namespace yl::dev;
  const uint32_t K = a.K, nb = K / 32;
  const int ctid = cw * 32 + lane;
  float* red = reinterpret_cast<float*>(smem + L.red_off);
  // the norm weight is a constant of the model: fetched before the wait on
  // the kernel that produces the rows
  float4 wv[NORM ? MU : 1];
  if (NORM) {
#pragma unroll
    for (int u = 0; u < MU; ++u) {
      const uint32_t i = ctid * 4 + u * MV_NCW * 32 * 4;
      wv[u] = i < K ? *reinterpret_cast<const float4*>(a.norm_w + i) : make_float4(0, 0, 0, 0);
    }
  }
  mv_wait_inputs(a);
  const bool tp_in = NT == 1 && a.tp_mode == 2;
  const uint32_t tp_flag = tp_in ? *a.tp_epoch * a.tp_nsites + a.tp_site + 1u : 0u;
  const uint64_t tp_t0 = tp_in ? clock64() : 0;
  // Norm factors of the resident rows in the reference's summation order (one
  // warp, all tokens at once). Tensor-parallel rows exist only in registers
  // (residual + the ranks' partials), so they keep the register-tree sum.
  float* const stg = reinterpret_cast<float*>(smem + L.nstage_off);
  for (int t = 0; t < NT; ++t) {
    const bool valid = t < (int)a.ntok;
    const float* xr = a.xres + (uint64_t)t * a.x_tok_stride;
    float4 xv[MU];
#pragma unroll
    for (int u = 0; u < MU; ++u) {
      const uint32_t i = ctid * 4 + u * MV_NCW * 32 * 4;
      const bool in = valid && i < K;
      xv[u] = in ? *reinterpret_cast<const float4*>(xr + i) : make_float4(0, 0, 0, 0);
      if (tp_in && in) {  // residual + the ranks' partials, summed in rank order
        const uint64_t* ib = reinterpret_cast<const uint64_t*>(a.tp_base[a.tp_rank] + a.tp_inbox_off) + i;
        float4 sum = make_float4(0, 0, 0, 0);
        for (uint32_t q = 0; q < a.tp_world; ++q) {
          uint64_t e0, e1, e2, e3;
          // wait (bounded, ~2 s) until the four entries carry this pass's flag
          for (uint32_t it = 0;; ++it) {
            ld_volatile_2u64(ib + (uint64_t)q * K, e0, e1);
            ld_volatile_2u64(ib + (uint64_t)q * K + 2, e2, e3);
            if ((uint32_t)(e0 >> 32) == tp_flag && (uint32_t)(e1 >> 32) == tp_flag &&
                (uint32_t)(e2 >> 32) == tp_flag && (uint32_t)(e3 >> 32) == tp_flag)
              break;
            if ((it & 63u) == 63u && (uint64_t)(clock64() - tp_t0) > 4000000000ull) {
              if (a.err) atomicExch(a.err, ERR_WAIT_TIMEOUT);
              break;
            }
          }
          const float p0 = __uint_as_float((uint32_t)e0), p1 = __uint_as_float((uint32_t)e1);
          const float p2 = __uint_as_float((uint32_t)e2), p3 = __uint_as_float((uint32_t)e3);
          if (q == 0) {
            sum = make_float4(p0, p1, p2, p3);
          } else {
            sum.x = __fadd_rn(sum.x, p0);
            sum.y = __fadd_rn(sum.y, p1);
            sum.z = __fadd_rn(sum.z, p2);
            sum.w = __fadd_rn(sum.w, p3);
          }
        }
        xv[u].x = __fadd_rn(xv[u].x, sum.x);
        xv[u].y = __fadd_rn(xv[u].y, sum.y);
        xv[u].z = __fadd_rn(xv[u].z, sum.z);
        xv[u].w = __fadd_rn(xv[u].w, sum.w);
        if (blockIdx.x == 0) *reinterpret_cast<float4*>(a.tp_xout + i) = xv[u];
      }
    }
    float r = 1.0f;
    if (NORM && !tp_in) {
      // the reference's 8-lane sum of squares (util.rs:389-426): the row,
      // already in registers, is staged in shared memory and lanes 0..7 of
      // warp 0 walk the eight addition chains from there
      if (valid) {
#pragma unroll
        for (int u = 0; u < MU; ++u) {
          const uint32_t i = ctid * 4 + u * MV_NCW * 32 * 4;
          if (i < K) *reinterpret_cast<float4*>(stg + i) = xv[u];
        }
      }
      named_bar_sync(1, MV_NCW * 32);
      if (kTrace && a.trace && t == 0 && ctid == 0) a.trace[(uint64_t)blockIdx.x * 8 + 4] = globaltimer();
      if (cw == 0 && valid) {
        const float rv = rms_factor_smem8(stg, K, a.eps, lane);
        if (lane == 0) red[32 + t] = rv;
      }
      named_bar_sync(1, MV_NCW * 32);  // the factor is published; stg is reused by the next token
      if (kTrace && a.trace && t == 0 && ctid == 0) a.trace[(uint64_t)blockIdx.x * 8 + 5] = globaltimer();
      r = valid ? red[32 + t] : 1.0f;
    } else if (NORM) {
      float ss = 0.0f;
#pragma unroll
      for (int u = 0; u < MU; ++u) {
        ss = fmaf(xv[u].x, xv[u].x, ss);
        ss = fmaf(xv[u].y, xv[u].y, ss);
        ss = fmaf(xv[u].z, xv[u].z, ss);
        ss = fmaf(xv[u].w, xv[u].w, ss);
      }
      ss = warp_sum(ss);
      if (kTrace && a.trace && t == 0 && ctid == 0) a.trace[(uint64_t)blockIdx.x * 8 + 4] = globaltimer();
      if (lane == 0) red[cw] = ss;
      named_bar_sync(1, MV_NCW * 32);
      float tot = 0.0f;
#pragma unroll
      for (int i = 0; i < MV_NCW; ++i) tot += red[i];
      r = __fdiv_rn(tot, (float)K);
      r = __fadd_rn(r, a.eps);
      r = __fdiv_rn(1.0f, __fsqrt_rn(r));
      named_bar_sync(1, MV_NCW * 32);  // red[] reused by the next token
      if (kTrace && a.trace && t == 0 && ctid == 0) a.trace[(uint64_t)blockIdx.x * 8 + 5] = globaltimer();
    }
    // y = w * (r * x) in place
#pragma unroll
    for (int u = 0; u < MU; ++u) {
      if (NORM) {
        xv[u].x = __fmul_rn(wv[u].x, __fmul_rn(r, xv[u].x));
        xv[u].y = __fmul_rn(wv[u].y, __fmul_rn(r, xv[u].y));
        xv[u].z = __fmul_rn(wv[u].z, __fmul_rn(r, xv[u].z));
        xv[u].w = __fmul_rn(wv[u].w, __fmul_rn(r, xv[u].w));
      }
    }
    if (mv_f32_act<FMT>()) {
#pragma unroll
      for (int u = 0; u < MU; ++u) {
        const uint32_t i = ctid * 4 + u * MV_NCW * 32 * 4;
        if (i < K) *reinterpret_cast<float4*>(reinterpret_cast<float*>(smem + L.x_off) + t * K + i) = xv[u];
      }
      continue;
    }
    // quantization.rs:29-52 over the blocks held by lanes 8g..8g+7, four
    // slots at a time with every step interleaved across the slots (the
    // shuffle, divide and rounding chains overlap instead of running in turn)
#pragma unroll
    for (int u0 = 0; u0 < MU; u0 += 4) {
      if (u0 * MV_NCW * 32 * 4 >= K) break;  // uniform across the CTA
      float m[4], sc[4], isc[4], lim[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 y = xv[u0 + j];
        // fmaxf returns the other operand for a NaN: NaN never becomes the max
        m[j] = fmaxf(fmaxf(fmaxf(0.0f, fabsf(y.x)), fmaxf(fabsf(y.y), fabsf(y.z))), fabsf(y.w));
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < 4; ++j) m[j] = fmaxf(m[j], __shfl_xor_sync(FULL, m[j], o));
      // the four blocks' scale divisions are shared out: lane g*8 + j of a
      // block group divides for slot j (every lane of the group holds all four
      // maxima), then the results are broadcast within the group
      {
        const int j8 = lane & 7, src = lane & ~7;
        const float mj = j8 == 0 ? m[0] : j8 == 1 ? m[1] : j8 == 2 ? m[2] : m[3];
        const float scj = __fdiv_rn(mj, 127.0f);
        const float iscj = __frcp_rn(scj);
        const float lij = FMT == FMT_Q8X ? __fdiv_rn(254.0f, scj) : 0.0f;  // limb factor
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sc[j] = __shfl_sync(FULL, scj, src | j);
          isc[j] = __shfl_sync(FULL, iscj, src | j);
          if (FMT == FMT_Q8X) lim[j] = __shfl_sync(FULL, lij, src | j);
        }
      }
      int qv[4][4];
      bool exact = false;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qv[j][0] = quot_code_fast(xv[u0 + j].x, isc[j], exact);
        qv[j][1] = quot_code_fast(xv[u0 + j].y, isc[j], exact);
        qv[j][2] = quot_code_fast(xv[u0 + j].z, isc[j], exact);
        qv[j][3] = quot_code_fast(xv[u0 + j].w, isc[j], exact);
      }
      if (__any_sync(FULL, exact)) {  // rare: a quotient next to a half-integer
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          qv[j][0] = quot_code_exact(xv[u0 + j].x, sc[j]);
          qv[j][1] = quot_code_exact(xv[u0 + j].y, sc[j]);
          qv[j][2] = quot_code_exact(xv[u0 + j].z, sc[j]);
          qv[j][3] = quot_code_exact(xv[u0 + j].w, sc[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int u = u0 + j;
        const uint32_t i = ctid * 4 + u * MV_NCW * 32 * 4;
        const bool in = i < K;
        const float y[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
        const uint32_t word = pack4(qv[j][0], qv[j][1], qv[j][2], qv[j][3]);
        int qs = qv[j][0] + qv[j][1] + qv[j][2] + qv[j][3];
        const uint32_t b = i / 32, e0 = i % 32;  // block and first element within it
        int8_t* xq = reinterpret_cast<int8_t*>(smem + L.x_off) + t * K;
        if (FMT == FMT_Q4) {
          qs += __shfl_xor_sync(FULL, qs, 4);
          qs += __shfl_xor_sync(FULL, qs, 2);
          qs += __shfl_xor_sync(FULL, qs, 1);
          const uint32_t off = e0 < 16 ? b * 16 + e0 : nb * 16 + b * 16 + (e0 - 16);
          if (in) *reinterpret_cast<uint32_t*>(xq + off) = word;
          if (in && e0 == 0) reinterpret_cast<int*>(smem + L.xsum_off)[t * nb + b] = qs;
        } else if (FMT == FMT_Q8X) {
          // limbs 1 and 2 refine the Q8_0 value a: y - s*a = (s/254)*b + (s/254^2)*c + e
          const float inv = lim[j];  // 254 / sc: +inf for an all-zero block, limbs become 0
          const float s1 = sc[j] * (1.0f / 254.0f);
          uint32_t w1 = 0, w2 = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int8_t q0 = (int8_t)(word >> (8 * e));
            const float r1 = fmaf(-(float)q0, sc[j], y[e]);
            const int8_t q1 = rust_as_i8(roundf(r1 * inv));
            const float r2 = fmaf(-(float)q1, s1, r1);
            const int8_t q2 = rust_as_i8(roundf(r2 * inv * 254.0f));
            w1 |= (uint32_t)(uint8_t)q1 << (8 * e);
            w2 |= (uint32_t)(uint8_t)q2 << (8 * e);
          }
          if (in) {
            *reinterpret_cast<uint32_t*>(xq + i) = word;
            *reinterpret_cast<uint32_t*>(xq + NT * K + i) = w1;
            *reinterpret_cast<uint32_t*>(xq + 2 * NT * K + i) = w2;
          }
        } else {
          if (in) *reinterpret_cast<uint32_t*>(xq + i) = word;
        }
        if (in && e0 == 0) reinterpret_cast<float*>(smem + L.xs_off)[t * nb + b] = sc[j];
      }
    }
    if (kTrace && a.trace && t == 0 && lane == 0) {  // this warp's rows quantized: warp 0, and the last warp
      const unsigned long long now = globaltimer();
      if (cw == 0) a.trace[(uint64_t)blockIdx.x * 8 + 6] = now;
      atomicMax(reinterpret_cast<unsigned long long*>(a.trace + (uint64_t)blockIdx.x * 8 + 7), now);
    }
  }
}

// Prologue: stage the activations of NT tokens into shared memory.
template <int FMT, int NT>
__device__ __forceinline__ void mv_stage_x(const MvArgs& a, const MvLayout& L, uint8_t* smem, int cw, int lane) {
  using namespace yl::dev;
  const uint32_t K = a.K, nb = K / 32;
  const int ctid = cw * 32 + lane;
  float* red = reinterpret_cast<float*>(smem + L.red_off);
  if (a.pro == PRO_NORM && K <= 4 * MV_NCW * 32 * 4) {  // K <= 4096: four float4 per thread
    mv_norm_regs<FMT, NT, true, 4>(a, L, smem, cw, lane);
    return;
  }
  if (a.pro == PRO_NORM && K <= MV_NORM_MU * MV_NCW * 32 * 4) {
    mv_norm_regs<FMT, NT, true, MV_NORM_MU>(a, L, smem, cw, lane);
    return;
  }
  if (a.pro == PRO_QUANT) {  // host guarantees K <= MV_QUANT_MU * 1024
    mv_norm_regs<FMT, NT, false, MV_QUANT_MU>(a, L, smem, cw, lane);
    return;
  }
  mv_wait_inputs(a);
  if (a.pro == PRO_NORM) {
    // norm factors in the reference's summation order, each row staged in
    // shared memory first (the layout reserves K floats at nstage_off)
    float* stg = reinterpret_cast<float*>(smem + L.nstage_off);
    for (int t = 0; t < NT && t < (int)a.ntok; ++t) {
      const float* xr = a.xres + (uint64_t)t * a.x_tok_stride;
      for (uint32_t i = ctid * 4; i < K; i += MV_NCW * 32 * 4)
        *reinterpret_cast<float4*>(stg + i) = *reinterpret_cast<const float4*>(xr + i);
      named_bar_sync(1, MV_NCW * 32);
      if (cw == 0) {
        const float r = rms_factor_smem8(stg, K, a.eps, lane);
        if (lane == 0) red[32 + t] = r;
      }
      named_bar_sync(1, MV_NCW * 32);
    }
    for (int t = 0; t < NT; ++t) {
      const bool valid = t < (int)a.ntok;
      const float* xr = a.xres + (uint64_t)t * a.x_tok_stride;
      const float r = valid ? red[32 + t] : 1.0f;
      if (mv_f32_act<FMT>()) {
        float* xf = reinterpret_cast<float*>(smem + L.x_off) + t * K;
        for (uint32_t k = ctid; k < K; k += MV_NCW * 32)
          xf[k] = valid ? __fmul_rn(a.norm_w[k], __fmul_rn(r, xr[k])) : 0.0f;
      } else {
        int8_t* xq = reinterpret_cast<int8_t*>(smem + L.x_off) + t * K;
        float* xs = reinterpret_cast<float*>(smem + L.xs_off) + t * nb;
        int* xsum = reinterpret_cast<int*>(smem + L.xsum_off) + t * nb;
        // four blocks per warp pass: their loads and quantizer chains overlap
        for (uint32_t b0 = cw; b0 < nb; b0 += 4 * MV_NCW) {
          float y[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint32_t b = b0 + u * MV_NCW;
            const uint32_t k = b * 32 + lane;
            y[u] = (valid && b < nb) ? __fmul_rn(a.norm_w[k], __fmul_rn(r, xr[k])) : 0.0f;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint32_t b = b0 + u * MV_NCW;
            if (b >= nb) break;  // warp-uniform
            const uint32_t k = b * 32 + lane;
            float sc;
            const int8_t q = quant_q8_lane(y[u], &sc);
            if (FMT == FMT_Q4) {
              const uint32_t off = (lane < 16) ? b * 16 + lane : nb * 16 + b * 16 + (lane - 16);
              xq[off] = q;
              int s = (int)q;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
              if (lane == 0) xsum[b] = s;
            } else {
              xq[k] = q;
            }
            if (lane == 0) xs[b] = sc;
          }
        }
      }
    }
    return;
  }
  if (mv_f32_act<FMT>()) {
    float* xf = reinterpret_cast<float*>(smem + L.x_off);
    for (int t = 0; t < NT; ++t) {
      const float4* src = reinterpret_cast<const float4*>(a.xf + (uint64_t)t * a.x_tok_stride);
      float4* dst = reinterpret_cast<float4*>(xf + t * K);
      const bool valid = t < (int)a.ntok;
      for (uint32_t i = ctid; i < K / 4; i += MV_NCW * 32) dst[i] = valid ? src[i] : make_float4(0, 0, 0, 0);
    }
    return;
  }
  int8_t* xq = reinterpret_cast<int8_t*>(smem + L.x_off);
  float* xs = reinterpret_cast<float*>(smem + L.xs_off);
  int* xsum = reinterpret_cast<int*>(smem + L.xsum_off);
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

// ---------------------------------------------------------------------------
// Lane t < NT adds token t's ng block terms of one pass, in group order, to
// its chain (the reference's sequential `+=` over groups).
template <int NT>
__device__ __forceinline__ void mv_chain(const float* terms, uint32_t ng, int lane, float& chain) {
  __syncwarp();
  if (lane < NT) {
    const float* tt = terms + lane * MV_TERMS;
    float c = chain;
    uint32_t i = 0;
    for (; i + 32 <= ng; i += 32) {  // eight loads in flight, then the dependent adds
      float4 q[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) q[u] = *reinterpret_cast<const float4*>(tt + i + 4 * u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        c = __fadd_rn(c, q[u].x);
        c = __fadd_rn(c, q[u].y);
        c = __fadd_rn(c, q[u].z);
        c = __fadd_rn(c, q[u].w);
      }
    }
    for (; i < ng; ++i) c = __fadd_rn(c, tt[i]);
    chain = c;
  }
  __syncwarp();  // the buffer is rewritten by the next pass
}

// One row's chunk [k0, k0+kn) from the stage, accumulated into acc[NT]; for
// the exact-fold formats lane t's acc[0] is token t's chain and `terms` this
// warp's buffer, or with FW (fold warp) the row's fold-slot row, which takes
// the chunk's block terms in group order and no chain is walked here.
template <int FMT, int NT, bool SF16, bool FW = false>
__device__ __forceinline__ void mv_row_chunk(const uint8_t* wrow, const uint8_t* srow, const uint8_t* smem,
                                             const MvLayout& L, uint32_t K, uint32_t k0, uint32_t kn, int lane,
                                             float (&acc)[NT], float* terms) {
  using namespace yl::dev;
  if (FMT == FMT_Q8) {
    const int8_t* xq = reinterpret_cast<const int8_t*>(smem + L.x_off);
    const float* xs = reinterpret_cast<const float*>(smem + L.xs_off);
    const uint32_t nck = kn / 16;  // 16-byte chunks, two per block
    for (uint32_t c0 = 0; c0 < nck; c0 += 32 * MV_U) {
      int4 w[MV_U];
      float wsc[MV_U];
      bool v[MV_U];
#pragma unroll
      for (int u = 0; u < MV_U; ++u) {
        const uint32_t c = c0 + u * 32 + lane;
        v[u] = c < nck;
        w[u] = v[u] ? *reinterpret_cast<const int4*>(wrow + 16 * c) : make_int4(0, 0, 0, 0);
        wsc[u] = v[u] ? ld_scale<SF16>(srow, c >> 1) : 0.0f;
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        int s[MV_U];
#pragma unroll
        for (int u = 0; u < MV_U; ++u) {
          const uint32_t c = c0 + u * 32 + lane;
          const int4 x = v[u] ? *reinterpret_cast<const int4*>(xq + t * K + k0 + 16 * c) : make_int4(0, 0, 0, 0);
          int d = dp4a(w[u].x, x.x, 0);
          d = dp4a(w[u].y, x.y, d);
          d = dp4a(w[u].z, x.z, d);
          s[u] = dp4a(w[u].w, x.w, d);
        }
#pragma unroll
        for (int u = 0; u < MV_U; ++u) s[u] += __shfl_xor_sync(FULL, s[u], 1);  // exact block dot
#pragma unroll
        for (int u = 0; u < MV_U; ++u) {
          const uint32_t c = c0 + u * 32 + lane;
          if (v[u] && !(lane & 1)) {
            // block term ((f32)isum * ws) * xs; group u*16 + lane/2 of this pass
            const float p = __fmul_rn(__fmul_rn((float)s[u], wsc[u]), xs[t * (K / 32) + (k0 >> 5) + (c >> 1)]);
            if (FW) terms[c >> 1] = p;
            else terms[t * MV_TERMS + u * 16 + (lane >> 1)] = p;
          }
        }
      }
      if (!FW) mv_chain<NT>(terms, min(MV_TERMS, (nck - c0) >> 1), lane, acc[0]);
    }
  } else if (FMT == FMT_Q4) {
    const int8_t* xq = reinterpret_cast<const int8_t*>(smem + L.x_off);
    const float* xs = reinterpret_cast<const float*>(smem + L.xs_off);
    const int* xsum = reinterpret_cast<const int*>(smem + L.xsum_off);
    const uint32_t nb = K / 32, nbk = kn / 32;  // one 16-byte chunk per block
    for (uint32_t b0 = 0; b0 < nbk; b0 += 32 * 2) {
      int4 w[2];
      float wsc[2];
      bool v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t b = b0 + u * 32 + lane;
        v[u] = b < nbk;
        w[u] = v[u] ? *reinterpret_cast<const int4*>(wrow + 16 * b) : make_int4(0, 0, 0, 0);
        wsc[u] = v[u] ? ld_scale<SF16>(srow, b) : 0.0f;
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (!v[u]) continue;
          const uint32_t kb = (k0 >> 5) + b0 + u * 32 + lane;
          const int4 xl = reinterpret_cast<const int4*>(xq + t * K)[kb];
          const int4 xh = reinterpret_cast<const int4*>(xq + t * K)[nb + kb];
          int s = dp4a(w[u].x & 0x0F0F0F0F, xl.x, 0);
          s = dp4a(w[u].y & 0x0F0F0F0F, xl.y, s);
          s = dp4a(w[u].z & 0x0F0F0F0F, xl.z, s);
          s = dp4a(w[u].w & 0x0F0F0F0F, xl.w, s);
          s = dp4a((w[u].x >> 4) & 0x0F0F0F0F, xh.x, s);
          s = dp4a((w[u].y >> 4) & 0x0F0F0F0F, xh.y, s);
          s = dp4a((w[u].z >> 4) & 0x0F0F0F0F, xh.z, s);
          s = dp4a((w[u].w >> 4) & 0x0F0F0F0F, xh.w, s);
          s -= 8 * xsum[t * nb + kb];  // sum (q-8)*x exactly
          const float p = __fmul_rn(__fmul_rn((float)s, wsc[u]), xs[t * nb + kb]);
          if (FW) terms[b0 + u * 32 + lane] = p;
          else terms[t * MV_TERMS + u * 32 + lane] = p;  // group u*32 + lane of this pass
        }
      }
      if (!FW) mv_chain<NT>(terms, min(MV_TERMS, nbk - b0), lane, acc[0]);
    }
  } else if (FMT == FMT_F16) {
    const float* xf = reinterpret_cast<const float*>(smem + L.x_off);
    const uint32_t nck = kn / 8;  // 8 halves per 16-byte chunk
    for (uint32_t c0 = 0; c0 < nck; c0 += 32 * 2) {
      int4 w[2];
      bool v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t c = c0 + u * 32 + lane;
        v[u] = c < nck;
        w[u] = v[u] ? *reinterpret_cast<const int4*>(wrow + 16 * c) : make_int4(0, 0, 0, 0);
      }
      // A lane's 8 activations are two float4 at a 32-byte lane stride; lanes
      // with bit 2 set read the halves in swapped order, which spreads every
      // shared load over all banks (4 wavefronts per 512 bytes, the minimum).
      const int rot = (lane >> 2) & 1;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!v[u]) continue;
        const uint32_t c = c0 + u * 32 + lane;
        const __half2* h2 = reinterpret_cast<const __half2*>(&w[u]);
        float wf[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(h2[j]);
          wf[2 * j] = f.x;
          wf[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float s = acc[t];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int p = (j + rot) & 1;
            const float4 x = *reinterpret_cast<const float4*>(xf + t * K + k0 + 8 * c + 4 * p);
            const float w0 = p ? wf[4] : wf[0], w1 = p ? wf[5] : wf[1];
            const float w2 = p ? wf[6] : wf[2], w3 = p ? wf[7] : wf[3];
            s = __fadd_rn(s, __fmul_rn(x.x, w0));
            s = __fadd_rn(s, __fmul_rn(x.y, w1));
            s = __fadd_rn(s, __fmul_rn(x.z, w2));
            s = __fadd_rn(s, __fmul_rn(x.w, w3));
          }
          acc[t] = s;
        }
      }
    }
  } else if (FMT == FMT_Q8X) {  // Q8_0 weights, three-limb int8 activations (lm_head)
    const int8_t* xq = reinterpret_cast<const int8_t*>(smem + L.x_off);
    const float* xs = reinterpret_cast<const float*>(smem + L.xs_off);
    const uint32_t nck = kn / 16;  // 16-byte chunks, two per block
    for (uint32_t c0 = 0; c0 < nck; c0 += 32 * 2) {
      int4 w[2];
      float wsc[2];
      bool v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t c = c0 + u * 32 + lane;
        v[u] = c < nck;
        w[u] = v[u] ? *reinterpret_cast<const int4*>(wrow + 16 * c) : make_int4(0, 0, 0, 0);
        wsc[u] = v[u] ? ld_scale<SF16>(srow, c >> 1) : 0.0f;
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        int s[2][3];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const uint32_t c = c0 + u * 32 + lane;
#pragma unroll
          for (int l = 0; l < 3; ++l) {
            const int4 x = v[u] ? *reinterpret_cast<const int4*>(xq + l * NT * K + t * K + k0 + 16 * c)
                                : make_int4(0, 0, 0, 0);
            int d = dp4a(w[u].x, x.x, 0);
            d = dp4a(w[u].y, x.y, d);
            d = dp4a(w[u].z, x.z, d);
            s[u][l] = dp4a(w[u].w, x.w, d);
          }
        }
        // per lane: this half-block's w.y / s = A + (B + C/254)/254 (|A|,|B|,|C|
        // < 2^22, exact in f32), then one shuffle completes the block
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const uint32_t c = c0 + u * 32 + lane;
          float blk = small_i2f(s[u][0]) +
                      fmaf(small_i2f(s[u][2]), 1.0f / 254.0f, small_i2f(s[u][1])) * (1.0f / 254.0f);
          blk += __shfl_xor_sync(FULL, blk, 1);
          if (v[u] && !(lane & 1)) acc[t] = fmaf(blk * wsc[u], xs[t * (K / 32) + (k0 >> 5) + (c >> 1)], acc[t]);
        }
      }
    }
  } else if (FMT == FMT_Q8F) {  // Q8_0 weights, f32 activations (lm_head)
    const float* xf = reinterpret_cast<const float*>(smem + L.x_off);
    const uint32_t nck = kn / 16;
    for (uint32_t c0 = 0; c0 < nck; c0 += 32 * 2) {
      int4 w[2];
      float wsc[2];
      bool v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t c = c0 + u * 32 + lane;
        v[u] = c < nck;
        w[u] = v[u] ? *reinterpret_cast<const int4*>(wrow + 16 * c) : make_int4(0, 0, 0, 0);
        wsc[u] = v[u] ? ld_scale<SF16>(srow, c >> 1) : 0.0f;
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float s[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const uint32_t c = c0 + u * 32 + lane;
          s[u] = 0.0f;
          if (v[u]) {
            // 16 activations per lane are four float4 at a 64-byte lane
            // stride; rotating the order by lane pair spreads each shared
            // load over all banks (4 wavefronts per 512 bytes, the minimum)
            const float4* xp = reinterpret_cast<const float4*>(xf + t * K + k0 + 16 * c);
            const int rot = (lane >> 1) & 3;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int p = (j + rot) & 3;
              const float4 x = xp[p];
              const uint32_t ww = p == 0 ? (uint32_t)w[u].x
                                         : p == 1 ? (uint32_t)w[u].y : p == 2 ? (uint32_t)w[u].z : (uint32_t)w[u].w;
              float f0, f1, f2, f3;
              i8x4_to_f32(ww, f0, f1, f2, f3);
              s[u] = fmaf(x.x, f0, s[u]);
              s[u] = fmaf(x.y, f1, s[u]);
              s[u] = fmaf(x.z, f2, s[u]);
              s[u] = fmaf(x.w, f3, s[u]);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) s[u] += __shfl_xor_sync(FULL, s[u], 1);
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (v[u] && !(lane & 1)) acc[t] = fmaf(s[u], wsc[u], acc[t]);
      }
    }
  } else {  // FMT_Q4F
    const float* xf = reinterpret_cast<const float*>(smem + L.x_off);
    const uint32_t nbk = kn / 32;
    // A lane's block is 32 activations (eight float4 at a 128-byte lane
    // stride); lane-rotated order keeps every shared load conflict-free.
    const int rot = lane & 7;
    for (uint32_t b = lane; b < nbk; b += 32) {
      const int4 w = *reinterpret_cast<const int4*>(wrow + 16 * b);
      const float wsc = ld_scale<SF16>(srow, b);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float4* xp = reinterpret_cast<const float4*>(xf + t * K + k0 + 32 * b);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int p = (j + rot) & 7;  // elements 4p..4p+3 of the block
          const float4 x = xp[p];
          const int wi = p & 3;
          const uint32_t word = wi == 0 ? (uint32_t)w.x : wi == 1 ? (uint32_t)w.y : wi == 2 ? (uint32_t)w.z : (uint32_t)w.w;
          // elements 0..15: low nibbles of bytes 0..15; 16..31: high nibbles
          const uint32_t nib = (p >> 2) ? (word >> 4) & 0x0F0F0F0Fu : word & 0x0F0F0F0Fu;
          // 2^23 + q as a float, minus 2^23 + 8: the exact value q - 8
          const float f0 = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7650)) - 8388616.0f;
          const float f1 = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7651)) - 8388616.0f;
          const float f2 = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7652)) - 8388616.0f;
          const float f3 = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7653)) - 8388616.0f;
          s = fmaf(x.x, f0, s);
          s = fmaf(x.y, f1, s);
          s = fmaf(x.z, f2, s);
          s = fmaf(x.w, f3, s);
        }
        acc[t] = fmaf(s, wsc, acc[t]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Batch-1/2 passes are capped so that two CTAs share an SM; larger token
// groups keep their accumulators unspilled.
template <int FMT, int NT, int EPI, bool SF16, int RPW>
__global__ void __launch_bounds__(mv_threads<FMT, NT>(), (NT <= 2 ? 2 : 1)) mv_kernel(MvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  using namespace yl::dev;
  constexpr bool FW = mv_fold_warp<FMT, NT>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t K = a.K, kc = a.kc;
  const int S = a.stages;
  constexpr int G = mv_groups(EPI);
  const MvLayout L = mv_layout<FMT, NT>(K, kc, RPW, S, SF16 ? 2u : 4u, G, a.pro == PRO_NORM);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + S;
  uint64_t* tfull = reinterpret_cast<uint64_t*>(smem + L.fbar_off);  // fold slot written (WPG arrivals)
  uint64_t* tempty = tfull + S;                                        // fold slot consumed (fold warp)

  // Row range: static split (row pairs for SwiGLU, gate/up together), or with
  // a.work the whole matrix, its row sets handed out by an atomic counter.
  const bool dyn = a.work != nullptr;
  const uint32_t unit = mv_swiglu(EPI) ? 2u : 1u;
  const uint64_t units = a.rows / unit;
  const uint32_t r_begin = dyn ? 0u : (uint32_t)(units * blockIdx.x / gridDim.x) * unit;
  const uint32_t r_end = dyn ? a.rows : (uint32_t)(units * (blockIdx.x + 1) / gridDim.x) * unit;
  // stage info written by the producer before it arrives on the stage's full
  // barrier: first row and row count (0: no rows, MV_END: no more stages)
  uint32_t* info_row = reinterpret_cast<uint32_t*>(smem + L.info_off);
  uint32_t* info_n = info_row + 16;
  uint32_t* list = info_row + 32;  // [MV_LIST] first rows of this CTA's row sets (dynamic SwiGLU)
  uint32_t* list_n = info_row + 32 + MV_LIST;
  // Stages carry row sets of RS rows (one consumer group's rows) and K-chunks.
  // Stage order: round p, chunk ch, group g (row set p*G + g), so consecutive
  // stages go to different groups and all groups consume concurrently; the
  // producer and every consumer walk the same nest and count stages in q.
  constexpr int WPG = MV_NCW / G;  // warps per group
  static_assert(WPG * RPW == MV_RS, "a stage holds MV_RS rows");
  if (S % G != 0 || S > 16) {  // the launcher never plans this (parity aliasing)
    if (threadIdx.x == 0 && a.err) atomicExch(a.err, ERR_BAD_ARG);
    return;
  }
  const uint32_t RS = WPG * RPW;
  const uint32_t nch = (K + kc - 1) / kc;
  const uint32_t nrs = (r_end - r_begin + RS - 1) / RS;

  uint64_t* const trace = (kTrace && a.trace) ? a.trace + (uint64_t)blockIdx.x * 8 : nullptr;
  if (trace && threadIdx.x == 0) trace[0] = globaltimer();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], WPG);
      if (FW) {
        mbar_init(&tfull[s], WPG);
        mbar_init(&tempty[s], 1);
      }
    }
    *list_n = 0;
    mbar_fence_init();
  }
  __syncthreads();
  grid_dep_launch();

  if (FW && warp == MV_FOLD_WARP) {
    // ---------------- fold warp ----------------
    // Walks the stages in the consumers' order (stage q: group q % G, chunk
    // (q / G) % nch). Lane r < MV_RS holds the chain of row r of each group's
    // current row set: ((0 + t_0) + t_1) + ... over the row's block terms in
    // group order (matmul_q8_slices' sequential `+=`, weight_type.rs:190-201);
    // after a row set's last chunk it runs the epilogue for its rows.
    float chain[G];
#pragma unroll
    for (int g = 0; g < G; ++g) chain[g] = 0.0f;
    int ended = 0;
    for (uint32_t q = 0;; ++q) {
      const int slot = q % S;
      const uint32_t ph = (q / S) & 1;
      if (!mbar_wait(&tfull[slot], ph, a.err)) break;
      const uint8_t* st = smem + L.ring_off + slot * L.stage_bytes + L.fold_off;
      const uint32_t row0 = reinterpret_cast<const uint32_t*>(st)[0];
      const uint32_t n = reinterpret_cast<const uint32_t*>(st)[1];
      const int g = q % G;
      const uint32_t ch = (q / G) % nch;
      float v = 0.0f;
      if (n != MV_END && n != 0 && (uint32_t)lane < n) {
        const uint32_t kn = min(kc, K - ch * kc), ng = kn / 32;
        const float* tt = reinterpret_cast<const float*>(st + 16) + lane * L.fold_row;
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
          if (gg != g) continue;
          float c = chain[gg];
          uint32_t i = 0;
          for (; i + 32 <= ng; i += 32) {  // eight loads in flight, then the dependent adds
            float4 w4[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) w4[u] = *reinterpret_cast<const float4*>(tt + i + 4 * u);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              c = __fadd_rn(c, w4[u].x);
              c = __fadd_rn(c, w4[u].y);
              c = __fadd_rn(c, w4[u].z);
              c = __fadd_rn(c, w4[u].w);
            }
          }
          for (; i < ng; ++i) c = __fadd_rn(c, tt[i]);
          chain[gg] = c;
          v = c;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[slot]);  // the slot's terms are read
      if (n == MV_END) {
        if (++ended == G) break;
        continue;
      }
      if (n == 0 || ch != nch - 1) continue;
      // ---- epilogue of the row set: lane r -> row row0 + r ----
#pragma unroll
      for (int gg = 0; gg < G; ++gg)
        if (gg == g) chain[gg] = 0.0f;
      const uint32_t r = row0 + lane;
      if (mv_swiglu(EPI)) {
        const float up = __shfl_down_sync(FULL, v, 1);  // rows 2j (gate), 2j+1 (up)
        if (!(lane & 1) && (uint32_t)lane + 1 < n) a.out[r / 2] = silu_mul(v, up);
      } else if ((uint32_t)lane < n) {
        float* o = a.out + r;
        if (EPI == EPI_STORE && a.tp_mode == 1) {
          // tensor parallel: this rank's partial row, flagged, into every
          // rank's inbox (own one included)
          const uint32_t flag = *a.tp_epoch * a.tp_nsites + a.tp_site + 1u;
          const uint64_t e = ((uint64_t)flag << 32) | __float_as_uint(v);
          for (uint32_t qq = 0; qq < a.tp_world; ++qq)
            st_volatile_u64(reinterpret_cast<uint64_t*>(a.tp_base[qq] + a.tp_inbox_off) +
                                (uint64_t)a.tp_rank * a.rows + r, e);
        } else if (EPI == EPI_STORE) *o = v;
        else if (EPI == EPI_ADD) *o = __fadd_rn(*o, v);
        else if (EPI == EPI_QUIRK) *o = (r < a.quirk_cols) ? __fadd_rn(*o, v) : v;
      }
    }
    if (EPI == EPI_SWIGLU_Q8) {  // h complete in global memory before the consumers quantize it
      __threadfence();
      named_bar_sync(2, (MV_NCW + 1) * 32);
    }
    grid_dep_wait();  // every thread of the grid waits before exit (keeps PDL chains transitive)
    return;
  }

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      // One chunk per row whose shared-memory strides equal the HBM strides:
      // a stage's rows are then one contiguous range in both places.
      const bool contig = nch == 1 && L.stage_q_row == a.row_bytes &&
                          (!mv_has_scales<FMT>() || L.stage_s_row == a.scale_row_bytes);
      // q counts stages issued; bit s of datamask: slot s's latest stage
      // carries copies (a stage with no rows or the closing stage has none)
      uint32_t q = 0, nlist = 0, datamask = 0;
      bool ok = true;
      const bool listed = dyn && EPI == EPI_SWIGLU_Q8;
      // rounds of G row sets (one per group); dynamic rounds are claimed one
      // round ahead so the atomic's latency hides behind the copies
      uint32_t base = dyn ? atomicAdd(a.work, (unsigned)G) : 0u;
      for (uint32_t p = 0; ok; ++p) {
        if (!dyn) base = p * G;
        if (base >= nrs) {  // no more row sets: one closing stage per group
          for (int g = 0; g < G; ++g) {
            const int slot = q % S;
            const uint32_t ph = (q / S) & 1;
            if (!mbar_wait(&empty[slot], ph ^ 1, a.err)) { ok = false; break; }
            ++q;
            datamask &= ~(1u << slot);
            info_n[slot] = MV_END;
            mbar_arrive(&full[slot]);
          }
          break;
        }
        uint32_t next = nrs;
        if (dyn && (!listed || nlist + 2u * G <= MV_LIST)) next = atomicAdd(a.work, (unsigned)G);
        for (uint32_t ch = 0; ok && ch < nch; ++ch)
        for (int g = 0; g < G; ++g) {
          const uint32_t rs = base + g;
          const int slot = q % S;
          const uint32_t ph = (q / S) & 1;
          if (!mbar_wait(&empty[slot], ph ^ 1, a.err)) { ok = false; break; }
          ++q;
          if (rs >= nrs) {  // this group has no row set in the last round
            datamask &= ~(1u << slot);
            info_n[slot] = 0;
            mbar_arrive(&full[slot]);
            continue;
          }
          datamask |= 1u << slot;
          const uint32_t row0 = r_begin + rs * RS;
          const uint32_t nrows = min(RS, r_end - row0);
          info_row[slot] = row0;
          info_n[slot] = nrows;
          if (listed && ch == 0) list[nlist++] = row0;
          const uint32_t k0 = ch * kc, kn = min(kc, K - k0);
          const uint32_t qb = mv_qbytes<FMT>(kn);
          const uint32_t ssz = SF16 ? 2u : 4u;
          const uint32_t sb = mv_has_scales<FMT>() ? ((kn / 32 * ssz + 15u) & ~15u) : 0u;
          uint8_t* stage = smem + L.ring_off + slot * L.stage_bytes;
          mbar_arrive_expect_tx(&full[slot], nrows * (qb + sb));
          if (contig) {  // full rows: one copy for the quants, one for the scales
            bulk_g2s(stage, a.wq + (uint64_t)row0 * a.row_bytes, nrows * qb, &full[slot], pol);
            if (sb) bulk_g2s(stage + RS * L.stage_q_row, a.ws + (uint64_t)row0 * a.scale_row_bytes, nrows * sb,
                             &full[slot], pol);
            continue;
          }
          for (uint32_t r = 0; r < nrows; ++r) {
            const uint64_t row = row0 + r;
            bulk_g2s(stage + r * L.stage_q_row, a.wq + row * a.row_bytes + mv_qbytes<FMT>(k0), qb, &full[slot], pol);
            if (sb)
              bulk_g2s(stage + RS * L.stage_q_row + r * L.stage_s_row,
                       a.ws + row * a.scale_row_bytes + (k0 / 32) * ssz, sb, &full[slot], pol);
          }
        }
        if (listed) *list_n = nlist;
        base = next;
      }
      if (dyn) {  // the last CTA to finish claiming resets the counters for the next launch
        __threadfence();
        if (atomicAdd(a.work + 1, 1u) == gridDim.x - 1) {
          atomicExch(a.work, 0u);
          atomicExch(a.work + 1, 0u);
        }
      }
      // every copy of this CTA is issued: the rest of its time HBM would idle
      // on its account, so start fetching the next kernel's first rows
      l2_prefetch_next(a.pf, blockIdx.x, gridDim.x);
      // Drain: no bulk copy may still target this CTA's shared memory at exit
      // (consumers that timed out may have left). A slot whose latest stage
      // carries copies is waited on with that stage's parity (its latest
      // phase, so the parity is unambiguous); a slot whose latest stage has
      // none was released by its consumers before reuse, so its copies landed.
      // In a healthy run every stage was consumed and this returns at once.
      for (int s2 = 0; s2 < S; ++s2) {
        if (!((datamask >> s2) & 1u)) continue;
        const uint32_t ql = q - 1 - ((q - 1 - (uint32_t)s2) % (uint32_t)S);  // latest stage on slot s2
        mbar_wait(&full[s2], (ql / S) & 1, a.err, 100000000ull);
      }
    }
    grid_dep_wait();  // every thread of the grid waits before exit (keeps PDL chains transitive)
    return;
  }

  // ---------------- consumers ----------------
  const int cw = warp - 1;
  mv_stage_x<FMT, NT>(a, L, smem, cw, lane);  // waits for the producing kernel inside
  named_bar_sync(1, MV_NCW * 32);
  if (trace && threadIdx.x == 32) trace[1] = globaltimer();

  float acc[RPW][NT];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[r][t] = 0.0f;
  // EPI_ADD, one token, static split: the residual values this warp will add
  // to (rows r_begin + rs*RS + cw, one row set per lane) are fetched now, so
  // the epilogues do not wait on a global read-modify-write
  const bool pre_add = EPI == EPI_ADD && NT == 1 && G == 1 && !dyn && nrs <= 32;
  float xpre = 0.0f;
  if (pre_add && lane < (int)nrs) {
    const uint32_t r = r_begin + lane * RS + cw;
    if (r < r_end) xpre = a.out[r];
  }
  float am_v = -INFINITY;  // EPI_ARGMAX: this warp's best (lane 0)
  uint32_t am_i = 0xFFFFFFFFu;

  // After a wait timeout the warp stops waiting and computing ("dead") but
  // keeps walking the loop so every named barrier below is still reached.
  // A warp that times out on a wait stops (the error flag is set) and goes on
  // to the named barriers below, which every consumer warp reaches.
  const int grp = cw / WPG, wi = cw % WPG;
  uint32_t q = 0;
  for (bool fin = false; !fin;)
  for (uint32_t ch = 0; !fin && ch < nch; ++ch)
  for (int g = 0; g < G; ++g) {
    const int slot = q % S;
    const uint32_t ph = (q / S) & 1;
    ++q;
    if (g != grp) continue;
    if (!mbar_wait(&full[slot], ph, a.err)) { fin = true; break; }
    const uint32_t n = info_n[slot];
    const uint32_t row0 = info_row[slot];
    uint8_t* const stage = smem + L.ring_off + slot * L.stage_bytes;
    if (FW) {  // the slot's fold area is free once the fold warp read its previous use
      if (!mbar_wait(&tempty[slot], ph ^ 1, a.err)) { fin = true; break; }
      if (wi == 0 && lane == 0) {
        reinterpret_cast<uint32_t*>(stage + L.fold_off)[0] = row0;
        reinterpret_cast<uint32_t*>(stage + L.fold_off)[1] = n;
      }
    }
    if (n == MV_END) {
      if (FW) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfull[slot]);
      }
      fin = true;
      break;
    }
    const uint32_t rend = row0 + n;  // rows of this stage: [row0, rend)
    const uint32_t k0 = ch * kc, kn = min(kc, K - k0);
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
      const uint32_t rl = wi * RPW + rr;
      if (rl >= n) continue;
      float* terms = FW ? reinterpret_cast<float*>(stage + L.fold_off + 16) + rl * L.fold_row
                        : reinterpret_cast<float*>(smem + L.terms_off) + cw * NT * MV_TERMS;
      mv_row_chunk<FMT, NT, SF16, FW>(stage + rl * L.stage_q_row, stage + RS * L.stage_q_row + rl * L.stage_s_row,
                                      smem, L, K, k0, kn, lane, acc[rr], terms);
    }
    __syncwarp();
    if (lane == 0) {
      if (FW) mbar_arrive(&tfull[slot]);  // releases the terms (and the header) to the fold warp
      mbar_arrive(&empty[slot]);
    }
    if (FW) continue;  // the fold warp walks the chains and runs the epilogue
    if (n == 0 || ch != nch - 1) continue;

    // ---- epilogue for this warp's rows of the finished row set ----
    if (mv_exact_fold<FMT>()) {  // lane t holds token t's chain: broadcast
#pragma unroll
      for (int rr = 0; rr < RPW; ++rr) {
        const float c = acc[rr][0];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[rr][t] = __shfl_sync(FULL, c, t);
      }
    } else {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int rr = 0; rr < RPW; ++rr) acc[rr][t] = warp_sum(acc[rr][t]);
    }
    if (mv_swiglu(EPI)) {
      const uint32_t r = row0 + wi * RPW;  // gate row (even), up row = r + 1
      const bool have = r + 1 < rend;
      float hv[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) hv[t] = have ? silu_mul(acc[0][t], acc[1][t]) : 0.0f;
      if (lane == 0 && have) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < (int)a.ntok) a.out[(uint64_t)t * a.out_tok_stride + r / 2] = hv[t];
      }
    } else {
#pragma unroll
      for (int rr = 0; rr < RPW; ++rr) {
        const uint32_t r = row0 + wi * RPW + rr;
        if (r >= rend) continue;
        if (EPI == EPI_ARGMAX) {
          const float v = acc[rr][0];
          if (v == v && am_better(v, r, am_v, am_i)) {
            am_v = v;
            am_i = r;
          }
        }
        const float prev = pre_add ? __shfl_sync(FULL, xpre, (row0 - r_begin) / RS) : 0.0f;
        if (lane == 0) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t >= (int)a.ntok) continue;
            float* o = a.out + (uint64_t)t * a.out_tok_stride + r;
            if (EPI == EPI_STORE && NT == 1 && a.tp_mode == 1) {
              // tensor parallel: this rank's partial row, flagged, into every
              // rank's inbox (own one included)
              const uint32_t flag = *a.tp_epoch * a.tp_nsites + a.tp_site + 1u;
              const uint64_t e = ((uint64_t)flag << 32) | __float_as_uint(acc[rr][0]);
              for (uint32_t q = 0; q < a.tp_world; ++q)
                st_volatile_u64(reinterpret_cast<uint64_t*>(a.tp_base[q] + a.tp_inbox_off) +
                                    (uint64_t)a.tp_rank * a.rows + r, e);
            } else if (EPI == EPI_STORE || EPI == EPI_ARGMAX) *o = acc[rr][t];
            else if (EPI == EPI_ADD) *o = __fadd_rn(pre_add ? prev : *o, acc[rr][t]);
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

  if (EPI == EPI_SWIGLU_Q8) {
    // Quantize h (quantization.rs:29-52, forward.rs:240) once, here, from the
    // h values in global memory: a block of 32 is quantized by the CTA whose
    // arrival completes it (per-block arrival counters, reset by that CTA).
    const uint32_t hn = a.rows / 2;
    __threadfence();
    if (FW) named_bar_sync(2, (MV_NCW + 1) * 32);  // with the fold warp, which wrote h
    else named_bar_sync(1, MV_NCW * 32);
    if (dyn) {
      // every listed row set holds RS/2 consecutive h values of one block
      uint32_t* done_b = reinterpret_cast<uint32_t*>(smem + L.red_off);  // [MV_LIST]
      const uint32_t nl = *list_n;
      const int ctid = cw * 32 + lane;
      for (int t = 0; t < (int)a.ntok && t < NT; ++t) {
        if (ctid < (int)nl) {
          const uint32_t b = list[ctid] / 64;
          const unsigned prev = atomicAdd(a.hcount + (uint64_t)t * (hn / 32) + b, RS / 2);
          done_b[ctid] = prev + RS / 2 == 32 ? b : MV_END;
        }
        named_bar_sync(1, MV_NCW * 32);
        for (uint32_t i = cw; i < nl; i += MV_NCW) {
          const uint32_t b = done_b[i];
          if (b == MV_END) continue;
          __threadfence();  // see the other CTAs' h values
          const uint64_t hk = (uint64_t)t * hn + b * 32 + lane;
          float sc;
          const int8_t qv = quant_q8_lane(__ldcg(a.out + (uint64_t)t * a.out_tok_stride + b * 32 + lane), &sc);
          a.hq[hk] = qv;
          if (lane == 0) {
            a.hs[hk / 32] = sc;
            a.hcount[(uint64_t)t * (hn / 32) + b] = 0u;  // for the next launch
          }
        }
        named_bar_sync(1, MV_NCW * 32);
      }
    } else {
      // this CTA's h range is [j0, j1): blocks inside it are quantized now, a
      // block shared with a neighbouring CTA by whichever completes it
      __shared__ int sw_last[2];
      const uint32_t j0 = r_begin / 2, j1 = r_end / 2;
      const uint32_t b0 = j0 / 32, b1 = (j1 + 31) / 32;  // blocks touched
      for (int t = 0; t < (int)a.ntok && t < NT; ++t) {
        if (cw == 0 && lane < 2) {
          // boundary blocks: first (lane 0) and last (lane 1), when partial
          const uint32_t b = lane == 0 ? b0 : b1 - 1;
          const uint32_t lo = max(j0, b * 32), hi = min(j1, b * 32 + 32);
          const bool partial = hi - lo < 32 && (lane == 0 || b1 - 1 != b0);
          int last = 0;
          if (partial) last = atomicAdd(a.hcount + (uint64_t)t * (hn / 32) + b, hi - lo) + (hi - lo) == 32;
          sw_last[lane] = partial ? last : 1;
        }
        named_bar_sync(1, MV_NCW * 32);
        for (uint32_t b = b0 + cw; b < b1; b += MV_NCW) {
          const bool first = b == b0, lastb = b == b1 - 1;
          if ((first && !sw_last[0]) || (lastb && !sw_last[1])) continue;  // a neighbour finishes it
          if (first || lastb) __threadfence();  // see the neighbour's h values
          const uint64_t hk = (uint64_t)t * hn + b * 32 + lane;
          float sc;
          const int8_t qv = quant_q8_lane(__ldcg(a.out + (uint64_t)t * a.out_tok_stride + b * 32 + lane), &sc);
          a.hq[hk] = qv;
          if (lane == 0) {
            a.hs[hk / 32] = sc;
            if (b * 32 < j0 || b * 32 + 32 > j1) a.hcount[(uint64_t)t * (hn / 32) + b] = 0u;  // for the next launch
          }
        }
        named_bar_sync(1, MV_NCW * 32);
      }
    }
  }

  if (EPI == EPI_ARGMAX) {
    // CTA winner -> global slot; the last CTA to arrive reduces all slots
    // (sampler.rs:67-79: lowest index among equal maxima; NaN never wins).
    float* rv = reinterpret_cast<float*>(smem + L.red_off);
    uint32_t* ri = reinterpret_cast<uint32_t*>(smem + L.red_off + 64);
    __shared__ int is_last;
    if (lane == 0) {
      rv[cw] = am_v;
      ri[cw] = am_i;
    }
    named_bar_sync(1, MV_NCW * 32);
    if (cw == 0) {
      float bv = lane < MV_NCW ? rv[lane] : -INFINITY;
      uint32_t bi = lane < MV_NCW ? ri[lane] : 0xFFFFFFFFu;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, bv, o);
        const uint32_t oi = __shfl_xor_sync(FULL, bi, o);
        if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        a.am_val[blockIdx.x] = bv;
        a.am_idx[blockIdx.x] = bi;
        __threadfence();
        const unsigned prev = atomicAdd(a.am_count, 1u);
        is_last = prev == gridDim.x - 1;
      }
      __syncwarp();
      if (__shfl_sync(FULL, lane == 0 ? is_last : 0, 0)) {
        __threadfence();
        bv = -INFINITY;
        bi = 0xFFFFFFFFu;
        for (uint32_t i = lane; i < gridDim.x; i += 32) {
          const float v = __ldcg(a.am_val + i);
          const uint32_t ix = __ldcg(a.am_idx + i);
          if (am_better(v, ix, bv, bi)) { bv = v; bi = ix; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(FULL, bv, o);
          const uint32_t oi = __shfl_xor_sync(FULL, bi, o);
          if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
          uint32_t res = bi == 0xFFFFFFFFu ? 0u : bi;
          const float l0 = __ldcg(a.out);
          if (a.am_shard) {  // vocabulary shard: publish (value, global index, first-logit NaN)
            a.am_shard[0] = bv;
            reinterpret_cast<uint32_t*>(a.am_shard)[1] = bi == 0xFFFFFFFFu ? 0xFFFFFFFFu : bi + a.am_base;
            reinterpret_cast<uint32_t*>(a.am_shard)[2] = l0 != l0 ? 1u : 0u;
            *a.am_count = 0u;
            return;
          }
          if (l0 != l0) res = 0;  // reference: a NaN first logit is never beaten
          StepState* st = a.state;
          if (a.am_out) a.am_out[st ? st->steps : 0] = res;
          if (st) {
            st->next = (int32_t)res;
            st->token = (int32_t)res;
            st->pos += 1;
            st->steps += 1;
          }
          *a.am_count = 0u;  // ready for the next launch
        }
      }
    }
  }
  if (trace && threadIdx.x == 32) trace[3] = globaltimer();
}

// CTAs of a matvec launch: lc.grid (0: 148), at most one per row (row pair).
inline uint32_t matvec_grid(uint32_t rows, int epi, uint32_t lc_grid) {
  uint32_t grid;
  bool dyn;
  matvec_schedule(rows, epi, lc_grid, 1, false, &grid, &dyn);
  return grid;
}

// Host-side launcher for one (FMT, SF16) family; NT and EPI dispatched here.
template <int FMT, bool SF16>
cudaError_t mv_launch(const MvArgs& a0, int epi, const LaunchCfg& lc) {
  MvArgs a = a0;
  const int nt = a.ntok <= 1 ? 1 : a.ntok <= 2 ? 2 : a.ntok <= 4 ? 4 : 8;
  const int rpw = mv_swiglu(epi) ? 2 : 1;
  MvLayout L0;
  int stages = 0;
  auto layout = [&](int g) {
    switch (nt) {
      case 1: return mv_layout<FMT, 1>(a.K, a.kc, rpw, 0, SF16 ? 2u : 4u, g, a.pro == PRO_NORM);
      case 2: return mv_layout<FMT, 2>(a.K, a.kc, rpw, 0, SF16 ? 2u : 4u, g, a.pro == PRO_NORM);
      case 4: return mv_layout<FMT, 4>(a.K, a.kc, rpw, 0, SF16 ? 2u : 4u, g, a.pro == PRO_NORM);
      default: return mv_layout<FMT, 8>(a.K, a.kc, rpw, 0, SF16 ? 2u : 4u, g, a.pro == PRO_NORM);
    }
  };
  // Ring plan. The stage count S must be a multiple of the group count G:
  // then slot s always serves group s % G, every wait on a slot is exactly one
  // phase after that group's previous use of it, and the mbarrier parity is
  // unambiguous (with S % G != 0 a group could pass a wait on the completion
  // of a phase two uses back, i.e. on another group's stage).
  const int G = mv_groups(epi);
  for (;;) {
    L0 = layout(G);
    stages = (int)((lc.smem_budget > L0.total ? lc.smem_budget - L0.total : 0) / L0.stage_bytes);
    stages = (stages > 16 ? 16 : stages) / G * G;
    // a ring of fewer than two stages inside the budget cannot overlap copy
    // and compute (or costs the SM its second CTA): halve the chunk instead
    if (stages >= 2 || a.kc <= 256) break;
    a.kc = (a.kc / 2 + 255u) / 256u * 256u;
  }
  if (stages < 2) stages = 2;  // activations fill the budget (large token groups)
  if (stages % G || stages > 16) return cudaErrorInvalidConfiguration;
  a.stages = stages;
  const uint32_t smem = L0.total + stages * L0.stage_bytes;
  if (smem > 227u * 1024u) return cudaErrorInvalidConfiguration;
  if (epi == EPI_ARGMAX && nt != 1) return cudaErrorInvalidValue;
  {
    // dynamic row sets pay off with several row sets per CTA; the SwiGLU+
    // quantize tail needs every row set whole and at most MV_LIST per CTA
    static_assert(MV_RS == MV_ROWSET && MV_LIST == MV_SWIGLU_LIST, "one schedule rule for launcher and prefetch");
    uint32_t g;
    bool ok;
    matvec_schedule(a.rows, epi, lc.grid, a.ntok, a.work != nullptr, &g, &ok);
    if (!ok) a.work = nullptr;
  }
  if (epi == EPI_SWIGLU_Q8 && (a.rows % 64 || mv_f32_act<FMT>())) return cudaErrorInvalidValue;
  // tensor-parallel push / all-reduce: single token, store epilogue / register RMSNorm prologue
  if (a.tp_mode && (!a.tp_epoch || a.tp_site >= a.tp_nsites || a.tp_world < 2 || a.tp_world > 8 ||
                    a.tp_rank >= a.tp_world || a.tp_inbox_off % 32))
    return cudaErrorInvalidValue;
  if (a.tp_mode == 1 && (nt != 1 || epi != EPI_STORE)) return cudaErrorInvalidValue;
  if (a.tp_mode == 2 && (nt != 1 || a.pro != PRO_NORM || a.K > (uint32_t)(MV_NORM_MU * MV_NCW * 32 * 4) ||
                         a.K % 32 || !a.tp_xout))
    return cudaErrorInvalidValue;
  if (a.pro == PRO_QUANT && (a.K > MV_QUANT_MU * MV_NCW * 32 * 4 || mv_f32_act<FMT>())) return cudaErrorInvalidValue;
  // three-limb activations are produced only by the register RMSNorm prologue
  if (FMT == FMT_Q8X && (a.pro != PRO_NORM || a.K > MV_NORM_MU * MV_NCW * 32 * 4)) return cudaErrorInvalidValue;
  void (*kern)(MvArgs) = nullptr;
#define YL_MV_CASE(NT_, EPI_, RPW_) \
  if (nt == NT_ && epi == EPI_) kern = mv_kernel<FMT, NT_, EPI_, SF16, RPW_>;
#define YL_MV_NT(NT_)                                           \
  YL_MV_CASE(NT_, EPI_STORE, 1)                                 \
  YL_MV_CASE(NT_, EPI_ADD, 1)                                   \
  YL_MV_CASE(NT_, EPI_QUIRK, 1)                                 \
  if (!mv_f32_act<FMT>() || FMT == FMT_F16) { YL_MV_CASE(NT_, EPI_SWIGLU, 2) } \
  if (!mv_f32_act<FMT>()) { YL_MV_CASE(NT_, EPI_SWIGLU_Q8, 2) }
  if constexpr (FMT == FMT_Q8X) {  // the lm_head: one token, logits and argmax
    YL_MV_CASE(1, EPI_STORE, 1)
    YL_MV_CASE(1, EPI_ARGMAX, 1)
  } else {
    YL_MV_NT(1)
    YL_MV_NT(2)
    YL_MV_NT(4)
    YL_MV_NT(8)
    if (mv_f32_act<FMT>()) { YL_MV_CASE(1, EPI_ARGMAX, 1) }
  }
#undef YL_MV_NT
#undef YL_MV_CASE
  if (!kern) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const uint32_t grid = matvec_grid(a.rows, epi, lc.grid);
  if (grid == 0) return cudaSuccess;
  const int threads = nt == 1 ? mv_threads<FMT, 1>() : MV_THREADS;
  return launch_kernel(kern, dim3(grid), dim3(threads), smem, lc, a);
}

}  // namespace k
}  // namespace yl
