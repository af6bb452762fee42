// Multi-token projections (prefill, batched matmul): an int8 tensor-core GEMM
// over Q8_0 / Q4_0 weights with the reference's per-32-block fold
// (weight_type.rs:122-226):
//   out[t][r] = sum over groups g, in order, of ((f32)isum(r,t,g) * ws[r][g]) * xs[t][g]
// One mma.sync m16n8k32 (s8 x s8 -> s32) covers exactly one 32-element block,
// so every block's exact int32 dot is folded into the f32 accumulators right
// after its instruction, in the reference's order. Q4_0 nibbles are widened to
// int8 (q - 8) in registers.
//
// Tiles: 128 weight rows x 64 tokens per CTA, 8 warps as 4 (rows) x 2 (tokens),
// 32 x 32 outputs per warp (passes of up to 32 tokens: 128 x 32, 16 x 32 per
// warp); K is staged 4 blocks at a time through a 3-stage
// cp.async ring (rows padded by 16 bytes: the ldmatrix fragment loads are
// bank-conflict free). The grid walks token tiles fastest, so the CTAs sharing a weight tile
// run together and the tile comes from HBM once.
//
// Epilogues: store, residual add, the reference's `+=` quirk on quad columns,
// and SwiGLU + Q8_0 quantization of h (forward.rs:206-240) for interleaved
// gate/up rows (gate j at 2j, up j at 2j+1): the loader puts gate rows in the
// upper and up rows in the lower half of every 16-row MMA tile, so one thread
// holds both values of a pair; a CTA's 64 h values per token are two whole
// quantization blocks, quantized by the bit-exact warp quantizer.
#include "device.cuh"
#include "gemm_util.cuh"
#include "kernels.h"

namespace yl {
namespace k {
using namespace yl::dev;

namespace {
using namespace gu;
constexpr int GB_M = 128, GB_N = 64, GB_KB = 4, GB_S = 3;

template <int FMT, int BN, int BM = 128>
struct GTile {
  static constexpr int QB = FMT == FMT_Q4 ? 16 : 32;  // weight bytes per 32-block
  static constexpr int WROW = GB_KB * QB + 16;         // padded shared-memory rows
  static constexpr int XROW = GB_KB * 32 + 16;
  static constexpr int W_BYTES = BM * WROW;
  static constexpr int X_BYTES = BN * XROW;
  static constexpr int WS_BYTES = BM * GB_KB * 4;
  static constexpr int XS_BYTES = BN * GB_KB * 4;
  static constexpr int STAGE = W_BYTES + X_BYTES + WS_BYTES + XS_BYTES;
  static constexpr int SMEM = GB_S * STAGE;
};
static_assert(GTile<FMT_Q8, 64>::STAGE % 16 == 0 && GTile<FMT_Q4, 64>::STAGE % 16 == 0, "stage alignment");
static_assert(GTile<FMT_Q8, 32>::STAGE % 16 == 0 && GTile<FMT_Q4, 32>::STAGE % 16 == 0, "stage alignment");
static_assert(32 * GB_M / 2 * 4 <= GTile<FMT_Q4, 32>::SMEM && GB_N * GB_M / 2 * 4 <= GTile<FMT_Q4, 64>::SMEM,
              "SwiGLU staging fits the ring");

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(0));
}

template <int FMT, bool SF16, bool PERM, int BN, int BM, int NTH>
__device__ __forceinline__ void gemm_load(const GemmArgs& a, uint8_t* st, uint32_t m0, uint32_t n0, uint32_t g0,
                                          uint32_t nb) {
  using T = GTile<FMT, BN, BM>;
  uint8_t* wt = st;
  uint8_t* xt = wt + T::W_BYTES;
  uint8_t* wsc = xt + T::X_BYTES;
  uint8_t* xsc = wsc + T::WS_BYTES;
  const uint32_t tid = threadIdx.x;
  // rows / tokens past the end re-read the last one (in bounds); their
  // results are never stored
  const uint32_t wp = nb * T::QB / 16;  // 16-byte pieces per weight row
  for (uint32_t i = tid; i < BM * wp; i += NTH) {
    const uint32_t r = i / wp, p = i - r * wp;
    const uint32_t gr = min(m0 + r, a.rows - 1);
    cp_async16(wt + tile_row<PERM>(r) * T::WROW + p * 16,
               a.wq + (uint64_t)gr * a.row_bytes + (uint64_t)g0 * T::QB + p * 16);
  }
  const uint32_t xp = nb * 2;
  for (uint32_t i = tid; i < BN * xp; i += NTH) {
    const uint32_t t = i / xp, p = i - t * xp;
    const uint32_t gt = min(n0 + t, a.ntok - 1);
    cp_async16(xt + t * T::XROW + p * 16, a.xq + (uint64_t)gt * a.x_stride + (uint64_t)g0 * 32 + p * 16);
  }
  if (SF16) {  // f16 scales in pairs (the launcher checks the row padding holds an odd tail's pair)
    const uint32_t sp = (nb + 1) / 2;
    for (uint32_t i = tid; i < BM * sp; i += NTH) {
      const uint32_t r = i / sp, p = i - r * sp;
      const uint32_t gr = min(m0 + r, a.rows - 1);
      cp_async4(wsc + (tile_row<PERM>(r) * GB_KB + 2 * p) * 2,
                a.ws + (uint64_t)gr * a.scale_row_bytes + (uint64_t)(g0 + 2 * p) * 2);
    }
  } else {
    for (uint32_t i = tid; i < BM * nb; i += NTH) {
      const uint32_t r = i / nb, b = i - r * nb;
      const uint32_t gr = min(m0 + r, a.rows - 1);
      cp_async4(wsc + (tile_row<PERM>(r) * GB_KB + b) * 4, a.ws + (uint64_t)gr * a.scale_row_bytes + (uint64_t)(g0 + b) * 4);
    }
  }
  for (uint32_t i = tid; i < BN * nb; i += NTH) {  // stored [block][token]
    const uint32_t t = i / nb, b = i - t * nb;
    const uint32_t gt = min(n0 + t, a.ntok - 1);
    cp_async4(xsc + (b * BN + t) * 4, a.xs + (uint64_t)gt * a.xs_stride + g0 + b);
  }
}

// Threads of a CTA: 8 warps for 64-token tiles, else one warp per 16 rows.
template <int BN, int BM>
__host__ __device__ constexpr int gemm_threads() { return (BN >= 64 ? 8 : BM / 16) * 32; }

template <int FMT, bool SF16, int EPI, int BN, int BM>
__global__ void __launch_bounds__(gemm_threads<BN, BM>(), 512 / gemm_threads<BN, BM>()) gemm_q_kernel(GemmArgs a) {
  using T = GTile<FMT, BN, BM>;
  constexpr int NTH = gemm_threads<BN, BM>(), NW = NTH / 32;
  constexpr bool PERM = EPI == EPI_SWIGLU_Q8;
  // BN = 64: warps 4 (rows) x 2 (tokens), 32 x 32 each; BN = 32: 8 x 1,
  // 16 x 32; BN = 16 / 8: 8 x 1, 16 x 16 / 16 x 8 (fewer padded tokens folded
  // for small batches). NTW: 8-token n-tiles per warp.
  constexpr int WN = BN >= 64 ? 2 : 1, MT = BN >= 64 ? 2 : 1, RW = 16 * MT;
  constexpr int NTW = BN >= 32 ? 4 : BN / 8;
  static_assert(BN == 8 || BN == 16 || BN == 32 || BN == 64, "token tile");
  static_assert((BN == 64 && BM == 128) || (BN < 64 && BM % 16 == 0 && BM <= 128), "row tile");
  static_assert(EPI != EPI_SWIGLU_Q8 || BM % 64 == 0, "a SwiGLU tile holds whole 32-value h blocks");
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int wm = warp % (NW / WN), wn = warp / (NW / WN);
  const uint32_t G = a.K / 32, nch = (G + GB_KB - 1) / GB_KB;

  grid_dep_wait();  // activations come from the preceding kernel
#pragma unroll
  for (int s = 0; s < GB_S - 1; ++s) {
    if ((uint32_t)s < nch)
      gemm_load<FMT, SF16, PERM, BN, BM, NTH>(a, smem + s * T::STAGE, m0, n0, s * GB_KB, min((uint32_t)GB_KB, G - s * GB_KB));
    cp_async_commit();
  }

  float acc[MT][NTW][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NTW; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;

  for (uint32_t c = 0; c < nch; ++c) {
    cp_async_wait<GB_S - 2>();
    __syncthreads();  // stage c landed for every thread; stage c-1 is free
    const uint32_t cn = c + GB_S - 1;
    if (cn < nch)
      gemm_load<FMT, SF16, PERM, BN, BM, NTH>(a, smem + (cn % GB_S) * T::STAGE, m0, n0, cn * GB_KB,
                                 min((uint32_t)GB_KB, G - cn * GB_KB));
    cp_async_commit();

    const uint8_t* wt = smem + (c % GB_S) * T::STAGE;
    const uint8_t* xt = wt + T::W_BYTES;
    const uint8_t* wsc = xt + T::X_BYTES;
    const float* xsc = reinterpret_cast<const float*>(wsc + T::WS_BYTES);
    const uint32_t nb = min((uint32_t)GB_KB, G - c * GB_KB);
#pragma unroll
    for (uint32_t b = 0; b < (uint32_t)GB_KB; ++b) {
      if (b >= nb) break;
      uint32_t af[MT][4], bf[NTW][2];
      float w0[MT], w1[MT];
      float2 xv[NTW];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int rr = wm * RW + mt * 16 + gid;
        const int lr = wm * RW + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;  // this lane's ldmatrix row
        if (FMT == FMT_Q8) {
          ldsm_x4(af[mt], wt + lr * T::WROW + b * T::QB + (lane >> 4) * 16);
        } else {  // element j: low nibble of byte j, element j + 16: high nibble; value q - 8
          uint32_t v0, v1;
          ldsm_x2(v0, v1, wt + lr * T::WROW + b * T::QB);
          af[mt][0] = __vsub4(v0 & 0x0F0F0F0Fu, 0x08080808u);
          af[mt][1] = __vsub4(v1 & 0x0F0F0F0Fu, 0x08080808u);
          af[mt][2] = __vsub4((v0 >> 4) & 0x0F0F0F0Fu, 0x08080808u);
          af[mt][3] = __vsub4((v1 >> 4) & 0x0F0F0F0Fu, 0x08080808u);
        }
        if (SF16) {
          w0[mt] = __half2float(reinterpret_cast<const __half*>(wsc)[rr * GB_KB + b]);
          w1[mt] = __half2float(reinterpret_cast<const __half*>(wsc)[(rr + 8) * GB_KB + b]);
        } else {
          w0[mt] = reinterpret_cast<const float*>(wsc)[rr * GB_KB + b];
          w1[mt] = reinterpret_cast<const float*>(wsc)[(rr + 8) * GB_KB + b];
        }
      }
      if (NTW == 1) {  // one n-tile: lanes 0..15 address its two 8x8 matrices
        const int lt = lane & 7;
        ldsm_x2(bf[0][0], bf[0][1], xt + lt * T::XROW + b * 32 + ((lane >> 3) & 1) * 16);
      } else {
#pragma unroll
        for (int np = 0; np < NTW / 2; ++np) {  // n-tiles 2np and 2np + 1
          const int lt = wn * 32 + np * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
          uint32_t r[4];
          ldsm_x4(r, xt + lt * T::XROW + b * 32 + ((lane >> 3) & 1) * 16);
          bf[2 * np][0] = r[0];
          bf[2 * np][1] = r[1];
          bf[(2 * np + 1) % NTW][0] = r[2];
          bf[(2 * np + 1) % NTW][1] = r[3];
        }
      }
#pragma unroll
      for (int nt = 0; nt < NTW; ++nt)
        xv[nt] = *reinterpret_cast<const float2*>(xsc + b * BN + wn * 32 + nt * 8 + tig * 2);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NTW; ++nt) {
          int d[4];
          mma_s8(d, af[mt], bf[nt]);
          // ((f32)isum * w_scale) * x_scale, added in group order
          acc[mt][nt][0] = __fadd_rn(acc[mt][nt][0], __fmul_rn(__fmul_rn(__int2float_rn(d[0]), w0[mt]), xv[nt].x));
          acc[mt][nt][1] = __fadd_rn(acc[mt][nt][1], __fmul_rn(__fmul_rn(__int2float_rn(d[1]), w0[mt]), xv[nt].y));
          acc[mt][nt][2] = __fadd_rn(acc[mt][nt][2], __fmul_rn(__fmul_rn(__int2float_rn(d[2]), w1[mt]), xv[nt].x));
          acc[mt][nt][3] = __fadd_rn(acc[mt][nt][3], __fmul_rn(__fmul_rn(__int2float_rn(d[3]), w1[mt]), xv[nt].y));
        }
    }
  }

  if (EPI == EPI_SWIGLU_Q8) {
    cp_async_wait<0>();
    __syncthreads();  // the ring is free: it now stages h [64 tokens][64 pairs]
    float* hb = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NTW; ++nt) {
        const int jl = (wm * RW + mt * 16) / 2 + gid;  // pair of this thread's rows gid (gate) and gid + 8 (up)
        const int tl = wn * 32 + nt * 8 + tig * 2;
        hb[tl * (BM / 2) + jl] = silu_mul(acc[mt][nt][0], acc[mt][nt][2]);
        hb[(tl + 1) * (BM / 2) + jl] = silu_mul(acc[mt][nt][1], acc[mt][nt][3]);
      }
    __syncthreads();
    const uint32_t f = a.rows / 2;
    constexpr int HB = BM >= 64 ? BM / 64 : 1;  // h blocks of 32 per token in this tile
    static_assert(BN * (BM / 2) * 4 <= T::SMEM, "the h staging fits the ring");
    for (int pi = warp; pi < BN * HB; pi += NW) {
      const int tl = pi / HB, blk = pi % HB;
      const uint32_t t = n0 + tl;
      if (t >= a.ntok) continue;  // warp-uniform
      const float v = hb[tl * (BM / 2) + blk * 32 + lane];
      float sc;
      const int8_t q = quant_q8_lane(v, &sc);
      const uint32_t j = m0 / 2 + blk * 32 + lane;
      a.hq[(uint64_t)t * f + j] = q;
      if (lane == 0) a.hs[(uint64_t)t * (f / 32) + j / 32] = sc;
      if (a.out) a.out[(uint64_t)t * a.out_stride + j] = v;
    }
    return;
  }

#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NTW; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t r = m0 + wm * RW + mt * 16 + gid + (e >> 1) * 8;
        const uint32_t t = n0 + wn * 32 + nt * 8 + tig * 2 + (e & 1);
        if (r >= a.rows || t >= a.ntok) continue;
        float* o = a.out + (uint64_t)t * a.out_stride + r;
        const float v = acc[mt][nt][e];
        if (EPI == EPI_STORE) *o = v;
        else if (EPI == EPI_ADD) *o = __fadd_rn(*o, v);
        else *o = r < a.quirk_cols ? __fadd_rn(*o, v) : v;
      }
}

template <int FMT, bool SF16, int EPI, int BN, int BM>
cudaError_t gemm_launch_bn(const GemmArgs& a, const LaunchCfg& lc) {
  using T = GTile<FMT, BN, BM>;
  cudaError_t e = cudaFuncSetAttribute(gemm_q_kernel<FMT, SF16, EPI, BN, BM>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, T::SMEM);
  if (e != cudaSuccess) return e;
  const dim3 grid((a.ntok + BN - 1) / BN, (a.rows + BM - 1) / BM);
  return launch_kernel(gemm_q_kernel<FMT, SF16, EPI, BN, BM>, grid, dim3(gemm_threads<BN, BM>()), (uint32_t)T::SMEM,
                       lc, a);
}

// Token tiles of 8, 16, 32 or 64: a small batch folds no more padded tokens
// than it must (the fold, not the tensor core, bounds this kernel). Up to 16
// tokens the row tiles shrink to 32 rows (64 with the SwiGLU epilogue, whose
// tile holds whole 32-value h blocks), so a 4096-row projection still spreads
// over 128 CTAs.
template <int FMT, bool SF16, int EPI>
cudaError_t gemm_launch(const GemmArgs& a, const LaunchCfg& lc) {
  constexpr int SBM = EPI == EPI_SWIGLU_Q8 ? 64 : 32;
  if (a.ntok <= 8) return gemm_launch_bn<FMT, SF16, EPI, 8, SBM>(a, lc);
  if (a.ntok <= 16) return gemm_launch_bn<FMT, SF16, EPI, 16, SBM>(a, lc);
  return a.ntok <= 32 ? gemm_launch_bn<FMT, SF16, EPI, 32, 128>(a, lc) : gemm_launch_bn<FMT, SF16, EPI, 64, 128>(a, lc);
}

template <int FMT, bool SF16>
cudaError_t gemm_epi(const GemmArgs& a, int epi, const LaunchCfg& lc) {
  switch (epi) {
    case EPI_STORE: return gemm_launch<FMT, SF16, EPI_STORE>(a, lc);
    case EPI_ADD: return gemm_launch<FMT, SF16, EPI_ADD>(a, lc);
    case EPI_QUIRK: return gemm_launch<FMT, SF16, EPI_QUIRK>(a, lc);
    case EPI_SWIGLU_Q8: return gemm_launch<FMT, SF16, EPI_SWIGLU_Q8>(a, lc);
    default: return cudaErrorInvalidValue;
  }
}
}  // namespace

bool gemm_supported(const GemmArgs& a, int fmt, bool sf16, int epi) {
  if (fmt != FMT_Q8 && fmt != FMT_Q4) return false;
  if (epi != EPI_STORE && epi != EPI_ADD && epi != EPI_QUIRK && epi != EPI_SWIGLU_Q8) return false;
  if (!a.wq || !a.ws || !a.xq || !a.xs || a.rows == 0 || a.ntok == 0 || a.K == 0 || a.K % 32) return false;
  if ((a.rows + 31) / 32 > 65535u) return false;
  const uint32_t G = a.K / 32;
  const uint32_t qb = fmt == FMT_Q4 ? 16 : 32;
  if ((uintptr_t)a.wq % 16 || a.row_bytes % 16 || a.row_bytes < G * qb) return false;
  if ((uintptr_t)a.xq % 16 || a.x_stride % 16 || a.x_stride < a.K) return false;
  if ((uintptr_t)a.xs % 4 || a.xs_stride < G) return false;
  if ((uintptr_t)a.ws % 4 || a.scale_row_bytes % 4) return false;
  if (sf16 ? a.scale_row_bytes < 2 * (G + (G & 1)) : a.scale_row_bytes < 4 * G) return false;
  if (epi == EPI_SWIGLU_Q8) return a.rows % (a.ntok <= 16 ? 64u : (uint32_t)GB_M) == 0 && a.hq && a.hs;
  return a.out != nullptr;
}

cudaError_t gemm_q(const GemmArgs& a, int fmt, bool sf16, int epi, const LaunchCfg& lc) {
  if (!gemm_supported(a, fmt, sf16, epi)) return cudaErrorInvalidValue;
  if (fmt == FMT_Q8) return sf16 ? gemm_epi<FMT_Q8, true>(a, epi, lc) : gemm_epi<FMT_Q8, false>(a, epi, lc);
  return sf16 ? gemm_epi<FMT_Q4, true>(a, epi, lc) : gemm_epi<FMT_Q4, false>(a, epi, lc);
}

}  // namespace k
}  // namespace yl
