// Device helpers shared by the sm_100a kernels: PTX wrappers (mbarrier, 1-D
// bulk async copies, programmatic dependent launch), bounded waits, and the
// bit-exact Q8_0 block quantizer.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

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

// SwiGLU of one gate/up pair.
__device__ __forceinline__ float silu_mul(float g, float u) {
  // forward.rs:230-235: g / (1 + exp(-g)) * u
  float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
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
