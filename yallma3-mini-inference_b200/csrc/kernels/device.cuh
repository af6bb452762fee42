// Device helpers shared by the sm_100a kernels: PTX wrappers (mbarrier, 1-D
// bulk async copies, programmatic dependent launch), bounded waits, and the
// bit-exact Q8_0 block quantizer.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "expf_exact.h"
#include "kernels.h"

namespace yl {
namespace dev {

constexpr unsigned FULL = 0xFFFFFFFFu;

// Error word codes written by kernels into their `err` argument.
enum : int { ERR_NONE = 0, ERR_WAIT_TIMEOUT = 1, ERR_BAD_ARG = 2 };

// ---- programmatic dependent launch -------------------------------------
// Wait until the preceding kernel in the stream has completed and its writes
// are visible. A no-op when the kernel was launched without the PDL attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to be scheduled (it still waits in
// grid_dep_wait() for this grid to finish before reading our outputs).
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// 8-byte {value, flag} exchange entries: one aligned 64-bit access each is
// single-copy atomic, so a reader that sees the flag sees the value with it.
__device__ __forceinline__ void st_volatile_u64(void* p, uint64_t v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void ld_volatile_2u64(const void* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// Timeline stamps of the decode step (yl_trace_decode_step) exist only in a
// diagnostics build (YL_WITH_TRACE=1); the product build compiles every stamp
// branch out.
#ifndef YL_WITH_TRACE
#define YL_WITH_TRACE 0
#endif
constexpr bool kTrace = YL_WITH_TRACE != 0;
// Global nanosecond timer (timeline tracing of the decode step).
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// SwiGLU of one gate/up pair: forward.rs:230-235, g / (1 + exp(-g)) * u, with
// exp the correctly rounded e^x (yl_expf), each operation rounded as in f32.
__device__ __forceinline__ float silu_mul(float g, float u) {
  float s = __fdiv_rn(g, __fadd_rn(1.0f, yl::yl_expf(-g)));
  return __fmul_rn(s, u);
}

// ---- time ----------------------------------------------------------------
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier --------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit_cycles` SM clock cycles (4e9 is about
// 2 s at the 1.965 GHz boost clock, longer at lower clocks) and records
// ERR_WAIT_TIMEOUT. The SM cycle counter is used because it advances with the
// SM itself, whatever else observes the GPU. Returns false on timeout so the
// caller can stop issuing work.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          uint64_t limit_cycles = 4000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = clock64();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u && (uint64_t)(clock64() - t0) > limit_cycles) {
      if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

// ---- 1-D bulk async copy global -> shared (TMA, non-tensor) --------------
// Both addresses 16-byte aligned, size a multiple of 16. Completion is
// signalled on `bar` as transaction bytes. Weights are streamed once per
// step, so they are marked evict-first in L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Bulk prefetch of [src, src+bytes) into L2 (no completion to wait on).
// src 16-byte aligned, bytes a multiple of 16; issued in 64 KB pieces.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint64_t bytes) {
  const uint8_t* p = static_cast<const uint8_t*>(src);
  while (bytes) {
    const uint32_t n = bytes > 65536u ? 65536u : (uint32_t)bytes;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(n) : "memory");
    p += n;
    bytes -= n;
  }
}

// RMSNorm factors 1/sqrt(sum(x^2)/n + eps) of up to 16 rows of n floats
// (n % 8 == 0, rows 16-byte aligned), bit-identical to util.rs:389-426: the
// sum of squares runs in eight lane accumulators, lane l adding x[8j+l]^2 for
// j = 0, 1, 2, ... (each square rounded, then added), folded as
// ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)); then /n, +eps, 1/sqrt, all rounded
// as IEEE f32 operations. Called by all 32 lanes of one warp: lanes 2t and
// 2t+1 walk row t (lanes 0..3 and 4..7 of its accumulators, one float4 per
// step), so the cost is the n/8-long addition chain, not n.
__device__ __forceinline__ void rms_factors_exact(const float* x0, uint64_t stride, uint32_t nrows, uint32_t n,
                                                  float eps, float* out, int lane) {
  const uint32_t t = (uint32_t)lane >> 1, half = (uint32_t)lane & 1u;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (t < nrows) {
    const float* x = x0 + (uint64_t)t * stride + 4 * half;
    const uint32_t nj = n / 8;
    uint32_t j = 0;
    for (; j + 8 <= nj; j += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = *reinterpret_cast<const float4*>(x + 8 * (j + u));
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc.x = __fadd_rn(acc.x, __fmul_rn(v[u].x, v[u].x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(v[u].y, v[u].y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(v[u].z, v[u].z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(v[u].w, v[u].w));
      }
    }
    for (; j < nj; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(x + 8 * j);
      acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, v.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, v.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, v.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, v.w));
    }
  }
  const float h0 = __shfl_down_sync(FULL, acc.x, 1), h1 = __shfl_down_sync(FULL, acc.y, 1);
  const float h2 = __shfl_down_sync(FULL, acc.z, 1), h3 = __shfl_down_sync(FULL, acc.w, 1);
  if (half == 0 && t < nrows) {
    const float a0 = __fadd_rn(acc.x, h0), a1 = __fadd_rn(acc.y, h1);
    const float a2 = __fadd_rn(acc.z, h2), a3 = __fadd_rn(acc.w, h3);
    const float ss = __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
    float r = __fdiv_rn(ss, (float)n);
    r = __fadd_rn(r, eps);
    out[t] = __fdiv_rn(1.0f, __fsqrt_rn(r));
  }
}

// The same factor from a row staged in shared memory (n floats, n % 8 == 0),
// computed by lanes 8g..8g+7 of a warp: lane 8g+l walks accumulator l, the
// lanes fold with shuffles, and lane 8g returns the factor (other lanes return
// garbage). Shared-memory latency instead of L2 latency on every step of the
// n/8-long chains.
__device__ __forceinline__ float rms_factor_smem8(const float* x, uint32_t n, float eps, int lane) {
  const int l = lane & 7;
  float acc = 0.0f;
  const uint32_t nj = n / 8;
  uint32_t j = 0;
  if (nj >= 16) {  // software-pipelined: the next 16 squares load while these 16 add
    float v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) v[u] = x[8 * u + l];
    for (j = 16; j + 16 <= nj; j += 16) {
      float nv[16], sq[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) nv[u] = x[8 * (j + u) + l];
      // the squares first, so the adds issue back to back on the chain
#pragma unroll
      for (int u = 0; u < 16; ++u) sq[u] = __fmul_rn(v[u], v[u]);
#pragma unroll
      for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, sq[u]);
#pragma unroll
      for (int u = 0; u < 16; ++u) v[u] = nv[u];
    }
    float sq[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) sq[u] = __fmul_rn(v[u], v[u]);
#pragma unroll
    for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, sq[u]);
  }
  for (; j < nj; ++j) {
    const float v = x[8 * j + l];
    acc = __fadd_rn(acc, __fmul_rn(v, v));
  }
  // ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)) within each group of eight lanes
  const float a = __fadd_rn(acc, __shfl_down_sync(FULL, acc, 4));   // lane l<4: l_l + l_{l+4}
  const float b = __fadd_rn(a, __shfl_down_sync(FULL, a, 2));       // lane 0: a0+a2, lane 1: a1+a3
  const float ss = __fadd_rn(b, __shfl_down_sync(FULL, b, 1));      // lane 0: (a0+a2)+(a1+a3)
  float r = __fdiv_rn(ss, (float)n);
  r = __fadd_rn(r, eps);
  return __fdiv_rn(1.0f, __fsqrt_rn(r));
}

// Prefetches this CTA's share (slots cta, cta + ncta, ...) of the next
// kernel's first rows (see L2Prefetch).
__device__ __forceinline__ void l2_prefetch_next(const k::L2Prefetch& pf, uint32_t cta, uint32_t ncta) {
  if (!pf.q || !pf.slots || !pf.rows_each) return;
  const uint64_t units = pf.rows / pf.unit;
  for (uint32_t c = cta; c < pf.slots; c += ncta) {
    uint64_t r0, r1;
    if (pf.dyn) {
      r0 = (uint64_t)c * pf.rows_each;
      r1 = r0 + pf.rows_each;
    } else {
      r0 = units * c / pf.slots * pf.unit;
      r1 = units * (c + 1) / pf.slots * pf.unit;
      if (r1 > r0 + pf.rows_each) r1 = r0 + pf.rows_each;
    }
    if (r1 > pf.rows) r1 = pf.rows;
    if (r0 >= r1) continue;
    bulk_prefetch_l2(pf.q + r0 * pf.row_bytes, (r1 - r0) * pf.row_bytes);
    if (pf.s) bulk_prefetch_l2(pf.s + r0 * pf.srow_bytes, (r1 - r0) * pf.srow_bytes);
  }
}

// ---- named barrier over a subset of warps ---------------------------------
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- integer dot ----------------------------------------------------------
__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

// ---- Q8_0 quantization of one 32-element block by one warp ----------------
// quantization.rs:29-52: wmax = max |x| (NaN never wins the `>` scan, the
// scan starts from 0), scale = wmax / 127 (IEEE f32 division),
// q = round-half-away-from-zero(x / scale) converted like Rust `as i8`
// (saturating, NaN -> 0). Lane i holds element i; returns lane i's int8, the
// scale is returned in every lane.
__device__ __forceinline__ int8_t rust_as_i8(float v) {
  // the device float -> int conversion truncates, saturates and maps NaN to
  // 0, which with a clamp to [-128, 127] is exactly Rust's `as i8`
  const int i = __float2int_rz(v);
  return (int8_t)max(-128, min(127, i));
}
// q = rust_as_i8(roundf(x / d)) with the quotient correctly rounded to f32
// (the quantizer's `(x / scale).round() as i8`), from v = x * inv, inv = 1/d
// correctly rounded. |v - x/d| <= 2^-23 |x/d| and the f32 quotient is within
// 2^-24 |x/d| of x/d, so for |x/d| <= 128 the two differ by under 2.3e-5:
// when v is farther than 3.1e-5 from a half-integer both round to the same
// integer, which the 1.5*2^23 shift gives in two full-rate instructions.
// Otherwise (a few in 1e5 of the inputs), and for NaN/inf, `exact` is set and
// the caller takes quot_code_exact for the warp.
__device__ __forceinline__ int quot_code_fast(float x, float inv, bool& exact) {
  const float v = __fmul_rn(x, inv);
  const float t = __fadd_rn(v, 12582912.0f);  // v rounded to an integer in the low mantissa bits
  const float d = __fsub_rn(v, __fsub_rn(t, 12582912.0f));  // v minus that integer, exact
  // |d| just below 1/2 means v is next to a half-integer; NaN/inf fail the test
  exact |= !(fabsf(v) <= 128.0f && fabsf(d) < 0.5f - 3.1e-5f);
  const int q = __float_as_int(t) - 0x4B400000;
  return min(q, 127);
}
__device__ __forceinline__ int quot_code_exact(float x, float d) { return rust_as_i8(roundf(__fdiv_rn(x, d))); }
// Packs four int8 codes (low bytes of q0..q3) into one word, q0 lowest.
__device__ __forceinline__ uint32_t pack4(int q0, int q1, int q2, int q3) {
  return __byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410);
}
__device__ __forceinline__ int8_t quant_q8_lane(float x, float* scale_out) {
  const float a = fmaxf(fabsf(x), 0.0f);  // NaN -> 0 so it never becomes the max
  const float wmax = warp_max(a);
  const float scale = __fdiv_rn(wmax, 127.0f);
  *scale_out = scale;
  bool exact = false;
  int q = quot_code_fast(x, __frcp_rn(scale), exact);
  if (__any_sync(FULL, exact)) q = quot_code_exact(x, scale);
  return (int8_t)q;
}

}  // namespace dev
}  // namespace yl
