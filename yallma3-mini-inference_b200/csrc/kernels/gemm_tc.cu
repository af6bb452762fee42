// Multi-token projections over Q8_0 weights on the 5th-generation tensor
// cores: tcgen05.mma kind::i8 with TMA-fed shared-memory operands and the
// accumulators in tensor memory, folded into f32 in the reference's order
// (weight_type.rs:122-226):
//   out[t][r] = sum over 32-blocks g, in order, of ((f32)isum(r,t,g) * ws[r][g]) * xs[t][g]
//
// One MMA (M = 128 weight rows, N = 128 tokens, K = 32) covers exactly one
// block, so each block's exact int32 dot lands in its own tensor-memory
// buffer. Four buffers of 128 columns rotate: the MMAs of blocks g+1..g+3 run
// while the epilogue warps read block g, and a buffer is handed back to the
// MMA as soon as its words are in registers. A word plus the integer
// 0x4B400000 (the bits of 1.5 * 2^23), read as f32, is exactly
// 12582912 + isum (|isum| < 2^22): the int-to-float conversion is one integer
// add. With an f16 weight scale w (11 significant bits) 12582912 * w is exact
// and
//   fma(v, w, -12582912 * w) = round(isum * w),
// the reference's (isum as f32) * w; with f32 scales the fold subtracts
// 12582912 first (exact) and multiplies. The fold runs on packed f32x2
// operations. ptxas contracts a packed multiply followed by a packed add into
// a fused multiply-add even when both carry .rn (measured on sm_100a), which
// would round the product by the activation scale and the accumulation once
// instead of twice; so that product is a packed fma with a -0.0 addend that
// arrives as a kernel argument: fma(p, x, -0) = round(p * x) exactly (signed
// zeros included), and a fused multiply-add cannot absorb the following add.
//
// Warps: 0 producer (TMA of 4 blocks of weights and activations per stage
// into 128-byte-swizzled tiles, plus the stage's scales, activation scales
// transposed to [block][token]); 1 tensor-memory allocator and MMA issuer
// (one thread); 2..9 epilogue (warp w reads tensor-memory lanes
// 32*(w%4)..+31, i.e. weight rows, and token columns 64*((w-2)/4)..+63).
// Every wait is bounded; on a timeout the kernel records ERR_WAIT_TIMEOUT,
// stops issuing, drains its own MMAs and frees tensor memory.
#include <cuda.h>

#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {
using namespace yl::dev;

namespace {

constexpr uint32_t TC_M = 128;     // weight rows per CTA (the MMA's M)
constexpr uint32_t TC_N = 128;     // tokens per CTA (the MMA's N)
constexpr uint32_t TC_GPS = 4;     // 32-blocks per stage: 128 bytes of K, one swizzle atom
constexpr uint32_t TC_STAGES = 4;  // shared-memory ring
constexpr uint32_t TC_NBUF = 4;    // tensor-memory accumulator buffers of TC_N columns
constexpr uint32_t TC_EPI_WARPS = 8;
constexpr uint32_t TC_EC = TC_N * 4 / TC_EPI_WARPS;  // token columns per epilogue warp
static_assert(TC_EC == 64, "the fold reads two 32-column loads per block");
constexpr uint32_t TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr uint32_t TC_TMEM_COLS = TC_NBUF * TC_N;  // 512: the whole tensor memory (one CTA per SM)
constexpr uint32_t TC_A_BYTES = TC_M * 128;
constexpr uint32_t TC_B_BYTES = TC_N * 128;
constexpr uint32_t TC_XS_FLOATS = TC_GPS * TC_N;  // [block][token]
constexpr uint32_t TC_WS_FLOATS = TC_M * TC_GPS;  // [row][block]
constexpr uint32_t TC_STAGE = TC_A_BYTES + TC_B_BYTES + 4 * (TC_XS_FLOATS + TC_WS_FLOATS);
constexpr uint32_t TC_BAR_BYTES = 256;
constexpr uint32_t TC_SMEM = 1024 + TC_STAGES * TC_STAGE + TC_BAR_BYTES;  // + alignment slack
constexpr float TC_BIAS_F = 12582912.0f;  // 1.5 * 2^23
constexpr uint32_t TC_BIAS_BITS = 0x4B400000u;
static_assert(TC_STAGE % 1024 == 0, "swizzled tiles need 1024-byte alignment");
static_assert(TC_SMEM <= 227 * 1024, "shared memory");
static_assert(TC_SMEM > 114 * 1024, "one CTA per SM: the CTA holds all 512 tensor-memory columns");
static_assert(TC_N * 64 * 4 <= TC_STAGES * TC_STAGE, "SwiGLU staging fits the ring");

// ---- tcgen05 / TMA wrappers -------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] = A[smem] * B[smem]^T + D (s32), one elected thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The mbarrier gets one arrival when every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define YL_R32(p) p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7], p[8], p[9], p[10], p[11], p[12], p[13], p[14], \
                  p[15], p[16], p[17], p[18], p[19], p[20], p[21], p[22], p[23], p[24], p[25], p[26], p[27],     \
                  p[28], p[29], p[30], p[31]
#define YL_V32 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, " \
               "%21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}"

// 32 consecutive columns of this warp's 32 lanes: register i = column i of the thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 " YL_V32 ", [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                 "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                 "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                 "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// 2-D tiled TMA load of this GPU's memory (no multicast); x in bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint32_t x, uint32_t y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major tile of 128-byte rows, 128-byte
// swizzle, 8-row groups 1024 bytes apart (descriptor version 1 of sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: s32 accumulators, signed int8 A and B, both K-major, M = 128, N = TC_N.
constexpr uint32_t TC_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((TC_N >> 3) << 17) | ((TC_M >> 4) << 24);

// Packed f32x2 arithmetic, each lane rounded once (the explicit .rn keeps
// the multiply and the add from being contracted into a fused multiply-add).
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Asynchronous global -> shared copy of N bytes (4, 8 or 16; both addresses
// N-aligned), zero-filling what lies past src_bytes (0: nothing is read).
template <uint32_t N>
__device__ __forceinline__ void cp_async_zfill(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(smem_u32(dst)), "l"(src), "n"(N), "r"(src_bytes)
               : "memory");
}
// One arrival on the mbarrier (counted in its expected arrivals) once every
// cp.async this thread issued before has landed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that parks the thread in the barrier between polls (suspend
// hint of 0.2 ms per try) instead of spinning on issue slots the fold needs.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* err,
                                        uint64_t limit_cycles = 4000000000ull) {
  const uint64_t t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(200000u)
        : "memory");
    if (ok) return true;
    if ((uint64_t)(clock64() - t0) > limit_cycles) {
      if (err) atomicExch(err, ERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

// Warp-uniform bounded wait: lane 0 waits, the outcome is broadcast, and on
// success every lane takes its own acquire of the completed phase.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, uint32_t lane) {
  bool ok = true;
  if (lane == 0) ok = tc_wait(bar, parity, err);
  ok = __shfl_sync(FULL, ok ? 1 : 0, 0) != 0;
  if (ok) (void)mbar_try_wait(bar, parity);
  return ok;
}

__device__ __forceinline__ void named_bar(uint32_t id, uint32_t n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <bool SF16, int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x, GemmArgs a) {
  extern __shared__ uint8_t tc_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * TC_STAGE);  // stage landed (TMA + scales)
  uint64_t* empty = full + TC_STAGES;                                          // stage consumed (MMAs + scales read)
  uint64_t* tfull = empty + TC_STAGES;                                         // accumulator buffer holds a block
  uint64_t* tempty = tfull + TC_NBUF;                                          // buffer read and re-biased
  uint64_t* drain = tempty + TC_NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n0 = blockIdx.x * TC_N, m0 = blockIdx.y * TC_M;
  const uint32_t G = a.K / 32, nstage = (G + TC_GPS - 1) / TC_GPS;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < TC_STAGES; ++s) {
      mbar_init(&full[s], 32);
      mbar_init(&empty[s], 1 + TC_EPI_WARPS);
    }
    for (uint32_t b = 0; b < TC_NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], TC_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TC_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_wait();  // activations (and, for the residual add, out) come from the preceding kernels

  if (warp == 0) {
    // ---- producer: weights and activations by TMA, scales by cp.async ----
    // Lane l copies the scales of tokens l + 32k and rows l + 32k (k < 4):
    // activation scales one float at a time into [block][token] order, weight
    // scales as one 8- (f16) or 16-byte (f32) piece per row. Out-of-range
    // tokens, rows and blocks are zero-filled (source size 0). The full
    // barrier counts one asynchronous arrival per lane, made when the lane's
    // copies have landed, plus the TMA bytes.
    uint32_t issued = 0;
    for (uint32_t i = 0; i < nstage; ++i) {
      const uint32_t s = i % TC_STAGES, u = i / TC_STAGES;
      if (i >= TC_STAGES && !warp_wait(&empty[s], (u - 1) & 1, a.err, lane)) {
        *abort_flag = 1;
        break;
      }
      if (__shfl_sync(FULL, *abort_flag, 0)) break;
      uint8_t* st = smem + s * TC_STAGE;
      if (lane == 0) {
        mbar_expect_tx(&full[s], TC_A_BYTES + TC_B_BYTES);
        tma_load_2d(st, &tma_w, i * 128, m0, &full[s]);
        tma_load_2d(st + TC_A_BYTES, &tma_x, i * 128, n0, &full[s]);
      }
      float* xsT = reinterpret_cast<float*>(st + TC_A_BYTES + TC_B_BYTES);
      uint8_t* wsS = reinterpret_cast<uint8_t*>(xsT + TC_XS_FLOATS);
      const uint32_t g0 = i * TC_GPS;
#pragma unroll
      for (uint32_t kk = 0; kk < 4; ++kk) {
        const uint32_t t = lane + 32 * kk, gt = n0 + t;
#pragma unroll
        for (uint32_t gg = 0; gg < TC_GPS; ++gg) {
          const bool in = gt < a.ntok && g0 + gg < G;
          cp_async_zfill<4>(xsT + gg * TC_N + t, in ? a.xs + (uint64_t)gt * a.xs_stride + g0 + gg : a.xs, in ? 4u : 0u);
        }
        const uint32_t r = lane + 32 * kk, gr = m0 + r;
        constexpr uint32_t WB = SF16 ? 8 : 16;  // this stage's 4 scales of one row
        const bool in = gr < a.rows;
        cp_async_zfill<WB>(wsS + r * WB, in ? a.ws + (uint64_t)gr * a.scale_row_bytes + (uint64_t)g0 * (WB / 4) : a.ws,
                           in ? WB : 0u);
      }
      cp_async_arrive_noinc(&full[s]);
      issued = i + 1;
    }
    // on an abort, the copies this warp issued land before the CTA exits
    if (*abort_flag && lane == 0)
      for (uint32_t i = issued > TC_STAGES ? issued - TC_STAGES : 0; i < issued; ++i)
        tc_wait(&full[i % TC_STAGES], (i / TC_STAGES) & 1, nullptr, 200000000ull);
  } else if (warp == 1) {
    // ---- MMA issuer: one K = 32 MMA per block into the next accumulator buffer ----
    if (lane == 0) {
      for (uint32_t i = 0; i < nstage; ++i) {
        const uint32_t s = i % TC_STAGES, u = i / TC_STAGES;
        if (*abort_flag || !tc_wait(&full[s], u & 1, a.err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * TC_STAGE);
        const uint64_t adesc = smem_desc_sw128(sa), bdesc = smem_desc_sw128(sa + TC_A_BYTES);
        const uint32_t nb = min(TC_GPS, G - i * TC_GPS);
        bool ok = true;
        for (uint32_t gg = 0; gg < nb; ++gg) {
          const uint32_t kb = i * TC_GPS + gg, b = kb % TC_NBUF, ku = kb / TC_NBUF;
          if (!tc_wait(&tempty[b], ku & 1, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // the block's 32 bytes inside the 128-byte swizzle atom: start address + 32 * gg
          mma_i8(tmem + b * TC_N, adesc + 2 * gg, bdesc + 2 * gg, TC_IDESC, 0u);  // D = A * B
          tc_commit(&tfull[b]);
        }
        tc_commit(&empty[s]);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
      tc_commit(drain);  // every MMA this thread issued has completed when drain flips
      tc_wait(drain, 0, a.err);
    }
    __syncwarp();
  } else {
    // ---- epilogue: fold each block into f32 accumulators, then the output ----
    const uint32_t q = warp & 3, cq = (warp - 2) >> 2;
    const uint32_t row = 32 * q + lane, col0 = TC_EC * cq;
    const uint32_t tbase = tmem + ((32 * q) << 16) + col0;  // lane quarter q, this warp's TC_EC columns
    if (lane == 0)
      for (uint32_t b = 0; b < TC_NBUF; ++b) mbar_arrive(&tempty[b]);  // every buffer starts free
    float2 acc[TC_EC / 2];
#pragma unroll
    for (int j = 0; j < (int)TC_EC / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
    const float2 nz = make_float2(a.neg_zero, a.neg_zero);
    // ((f32)isum * w) * x accumulated over 32 columns. isum + 0x4B400000
    // (an integer add, off the floating-point pipe) read as f32 is exactly
    // 12582912 + isum.
    auto fold32 = [&](const uint32_t (&v)[32], const float* xh, float2* ah, float w) {
      const float2 w2 = make_float2(w, w);
      if (SF16) {  // f16 weight scales, none infinite (the caller checks: the upload records it)
        const float c = -TC_BIAS_F * w;  // exact: w has 11 significant bits
        const float2 c2 = make_float2(c, c);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 x = *reinterpret_cast<const float4*>(xh + j);
          const float2 p0 = fma2_rn(make_float2(__uint_as_float(v[j] + TC_BIAS_BITS), __uint_as_float(v[j + 1] + TC_BIAS_BITS)), w2, c2);
          const float2 p1 = fma2_rn(make_float2(__uint_as_float(v[j + 2] + TC_BIAS_BITS), __uint_as_float(v[j + 3] + TC_BIAS_BITS)), w2, c2);
          ah[j / 2] = add2_rn(ah[j / 2], fma2_rn(p0, make_float2(x.x, x.y), nz));
          ah[j / 2 + 1] = add2_rn(ah[j / 2 + 1], fma2_rn(p1, make_float2(x.z, x.w), nz));
        }
      } else {
        const float2 nbias = make_float2(-TC_BIAS_F, -TC_BIAS_F);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 x = *reinterpret_cast<const float4*>(xh + j);
          const float2 d0 = add2_rn(make_float2(__uint_as_float(v[j] + TC_BIAS_BITS), __uint_as_float(v[j + 1] + TC_BIAS_BITS)), nbias);
          const float2 d1 = add2_rn(make_float2(__uint_as_float(v[j + 2] + TC_BIAS_BITS), __uint_as_float(v[j + 3] + TC_BIAS_BITS)), nbias);
          ah[j / 2] = add2_rn(ah[j / 2], fma2_rn(mul2_rn(d0, w2), make_float2(x.x, x.y), nz));
          ah[j / 2 + 1] = add2_rn(ah[j / 2 + 1], fma2_rn(mul2_rn(d1, w2), make_float2(x.z, x.w), nz));
        }
      }
    };
    bool ok = true;
    float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);  // this row's scales of the current stage's 4 blocks
    const float* xsT = nullptr;
    for (uint32_t kb = 0; kb < G && ok; ++kb) {
      const uint32_t i = kb / TC_GPS, gg = kb % TC_GPS, s = i % TC_STAGES, u = i / TC_STAGES;
      const uint32_t b = kb % TC_NBUF, ku = kb / TC_NBUF;
      if (gg == 0) {
        if (!(ok = warp_wait(&full[s], u & 1, a.err, lane))) break;  // this stage's scales are in place
        xsT = reinterpret_cast<const float*>(smem + s * TC_STAGE + TC_A_BYTES + TC_B_BYTES);
        if (SF16) {
          const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(xsT + TC_XS_FLOATS) + row * 8);
          const __half2 h0 = *reinterpret_cast<const __half2*>(&h.x), h1 = *reinterpret_cast<const __half2*>(&h.y);
          w4 = make_float4(__low2float(h0), __high2float(h0), __low2float(h1), __high2float(h1));
        } else {
          w4 = *reinterpret_cast<const float4*>(xsT + TC_XS_FLOATS + row * TC_GPS);
        }
      }
      if (!(ok = warp_wait(&tfull[b], ku & 1, a.err, lane))) break;
      tc_fence_after();
      uint32_t va[32], vb[32];
      tmem_ld32(tbase + b * TC_N, va);
      tmem_ld32(tbase + b * TC_N + 32, vb);
      tmem_wait_ld();
      tc_fence_before();  // the buffer is in registers: the MMA may overwrite it
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      const float w = gg == 0 ? w4.x : gg == 1 ? w4.y : gg == 2 ? w4.z : w4.w;
      const float* xr = xsT + gg * TC_N + col0;
      fold32(va, xr, acc, w);
      fold32(vb, xr + 32, acc + 16, w);
      if (gg + 1 == TC_GPS || kb + 1 == G) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // done with this stage's scales
      }
    }
    if (!ok) *abort_flag = 1;
    // every epilogue warp is past its last read of the ring, and all take the same branch below
    named_bar(1, 32 * TC_EPI_WARPS);
    ok = *abort_flag == 0;

    if (ok && EPI == EPI_SWIGLU_Q8) {
      // gate row 2j on even lanes, up row 2j+1 on the odd neighbour: h into
      // shared memory [token][64 pairs], then Q8_0 blocks of 32 per token
      float* hb = reinterpret_cast<float*>(smem);
#pragma unroll
      for (int j = 0; j < (int)TC_EC / 2; ++j) {
        const float ux = __shfl_xor_sync(FULL, acc[j].x, 1), uy = __shfl_xor_sync(FULL, acc[j].y, 1);
        if (!(lane & 1)) {
          hb[(col0 + 2 * j) * 64 + row / 2] = silu_mul(acc[j].x, ux);
          hb[(col0 + 2 * j + 1) * 64 + row / 2] = silu_mul(acc[j].y, uy);
        }
      }
      named_bar(1, 32 * TC_EPI_WARPS);
      const uint32_t f = a.rows / 2;
      for (uint32_t p = warp - 2; p < TC_N * 2; p += TC_EPI_WARPS) {
        const uint32_t tl = p >> 1, blk = p & 1, t = n0 + tl;
        if (t >= a.ntok) continue;  // warp-uniform
        const float hv = hb[tl * 64 + blk * 32 + lane];
        float sc;
        const int8_t qv = quant_q8_lane(hv, &sc);
        const uint32_t j = m0 / 2 + blk * 32 + lane;
        a.hq[(uint64_t)t * f + j] = qv;
        if (lane == 0) a.hs[(uint64_t)t * (f / 32) + j / 32] = sc;
        if (a.out) a.out[(uint64_t)t * a.out_stride + j] = hv;
      }
    } else if (ok) {
      const uint32_t r = m0 + row;
      if (r < a.rows) {
#pragma unroll
        for (int j = 0; j < (int)TC_EC; ++j) {
          const uint32_t t = n0 + col0 + j;
          if (t >= a.ntok) break;
          const float v = (j & 1) ? acc[j / 2].y : acc[j / 2].x;
          float* o = a.out + (uint64_t)t * a.out_stride + r;
          if (EPI == EPI_STORE) *o = v;
          else if (EPI == EPI_ADD) *o = __fadd_rn(*o, v);
          else *o = r < a.quirk_cols ? __fadd_rn(*o, v) : v;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TC_TMEM_COLS);
}

// cuTensorMapEncodeTiled from the driver, through the runtime's entry-point query.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// [rows][K] int8 with `stride` bytes per row, tiles of 128 bytes x `box_rows`, 128-byte swizzle.
bool encode_i8_rows(CUtensorMap* m, const void* base, uint64_t K, uint64_t rows, uint64_t stride, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {K, rows};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool SF16, int EPI>
cudaError_t tc_launch(const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& a, const LaunchCfg& lc) {
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<SF16, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)TC_SMEM);
  if (e != cudaSuccess) return e;
  const dim3 grid((a.ntok + TC_N - 1) / TC_N, (a.rows + TC_M - 1) / TC_M);
  return launch_kernel(gemm_tc_kernel<SF16, EPI>, grid, dim3(TC_THREADS), TC_SMEM, lc, mw, mx, a);
}

template <bool SF16>
cudaError_t tc_epi(const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& a, int epi, const LaunchCfg& lc) {
  switch (epi) {
    case EPI_STORE: return tc_launch<SF16, EPI_STORE>(mw, mx, a, lc);
    case EPI_ADD: return tc_launch<SF16, EPI_ADD>(mw, mx, a, lc);
    case EPI_QUIRK: return tc_launch<SF16, EPI_QUIRK>(mw, mx, a, lc);
    case EPI_SWIGLU_Q8: return tc_launch<SF16, EPI_SWIGLU_Q8>(mw, mx, a, lc);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool gemm_tc_supported(const GemmArgs& a, int fmt, bool sf16, int epi) {
  if (fmt != FMT_Q8 || !gemm_supported(a, fmt, sf16, epi) || !encode_fn()) return false;
  if ((uintptr_t)a.wq % 16 || a.row_bytes % 16 || (uintptr_t)a.xq % 16 || a.x_stride % 16) return false;
  if ((a.rows + TC_M - 1) / TC_M > 65535u || a.ntok > 0x7FFFFFFFu) return false;
  if (epi == EPI_SWIGLU_Q8 && a.rows % TC_M) return false;
  // a stage copies 4 scales per row: rows padded to whole stages, pieces aligned
  const uint32_t G4 = (a.K / 32 + TC_GPS - 1) / TC_GPS * TC_GPS;
  if (sf16 ? (a.scale_row_bytes % 8 || a.scale_row_bytes < 2 * G4 || (uintptr_t)a.ws % 8)
           : (a.scale_row_bytes % 16 || a.scale_row_bytes < 4 * G4 || (uintptr_t)a.ws % 16))
    return false;
  return true;
}

cudaError_t gemm_tc(const GemmArgs& a, bool sf16, int epi, const LaunchCfg& lc) {
  if (!gemm_tc_supported(a, FMT_Q8, sf16, epi)) return cudaErrorInvalidValue;
  CUtensorMap mw, mx;
  if (!encode_i8_rows(&mw, a.wq, a.K, a.rows, a.row_bytes, TC_M) ||
      !encode_i8_rows(&mx, a.xq, a.K, a.ntok, a.x_stride, TC_N))
    return cudaErrorInvalidValue;
  GemmArgs b = a;
  b.neg_zero = -0.0f;
  return sf16 ? tc_epi<true>(mw, mx, b, epi, lc) : tc_epi<false>(mw, mx, b, epi, lc);
}

}  // namespace k
}  // namespace yl
