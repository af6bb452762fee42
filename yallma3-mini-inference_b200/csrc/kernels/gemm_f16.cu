// Multi-token F16 projections on the tensor cores (prefill and batched passes
// of F16 models, yl_matmul on F16 tensors): matmul_f32 (weight_type.rs:228-270)
//   out[t][r] = sum_k (f32)w[r][k] * x[t][k]
// with f32 activations and f16 weights. f16_split writes each token's row as
// x * 2^e = hi + lo (two f16 values per element, e the power of two that puts
// the row's max |x| in [2^14, 2^15), so lo stays a normal f16 for every
// element that matters to the sum); the GEMM runs mma.sync m16n8k16
// (f16 x f16 -> f32) on w*hi and w*lo into the same f32 accumulators and
// multiplies by 2^-e in the epilogue. Every f16 x f16 product is exact in f32
// and hi + lo holds x to about 2^-22 relative; the sum runs in the tensor
// core's order, not the reference's sequential one (the F16 matvec does not
// keep that order either).
//
// Tiles as in gemm_q8.cu: 128 weight rows x 64 tokens per CTA with 8 warps
// (4 x 2, 32 x 32 outputs each), 128 x 32 and 32 x 16 for smaller passes; K
// is staged 64 elements at a time (four 16-wide MMA steps) through a 3-stage
// cp.async ring, rows padded by 16 bytes so the ldmatrix loads are free of
// bank conflicts. A 16-wide f16 step is 32 bytes of a row, as one int8 block
// is in gemm_q8.cu, so the fragment addressing is the same.
#include <cuda_fp16.h>

#include "device.cuh"
#include "gemm_util.cuh"
#include "kernels.h"

namespace yl {
namespace k {
using namespace yl::dev;

namespace {
using namespace gu;
constexpr int FB_KS = 4, FB_S = 3;  // 16-wide k steps per stage, stages
constexpr int FS_THREADS = 256;     // f16_split

template <int BN, int BM>
struct FTile {
  static constexpr int ROW = FB_KS * 32 + 16;  // padded bytes per row of a stage
  static constexpr int W_BYTES = BM * ROW;
  static constexpr int X_BYTES = BN * ROW;     // hi rows; as many lo rows follow
  static constexpr int STAGE = W_BYTES + 2 * X_BYTES;
  static constexpr int SMEM = FB_S * STAGE;
};
static_assert(FTile<64, 128>::STAGE % 16 == 0 && FTile<16, 32>::STAGE % 16 == 0, "stage alignment");

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// One CTA per token: stage the row, apply the RMSNorm when asked (the
// matvec prologue's arithmetic: the factor in the reference's summation
// order, then w * (r * x)), find the row's max |x| and write hi, lo and e.
__global__ void __launch_bounds__(FS_THREADS) f16_split_kernel(GemmF16Args a) {
  extern __shared__ __align__(16) float fs_row[];  // [K]
  __shared__ float red[FS_THREADS / 32];
  __shared__ float rf;
  __shared__ int ex_s;
  grid_dep_launch();
  grid_dep_wait();
  const uint32_t t = blockIdx.x, K = a.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xr = a.x + (uint64_t)t * a.x_stride;
  for (uint32_t i = threadIdx.x * 4; i < K; i += FS_THREADS * 4)
    *reinterpret_cast<float4*>(fs_row + i) = *reinterpret_cast<const float4*>(xr + i);
  __syncthreads();
  if (a.norm_w) {
    if (warp == 0) {
      const float r = rms_factor_smem8(fs_row, K, a.eps, lane);
      if (lane == 0) rf = r;
    }
    __syncthreads();
  }
  float m = 0.0f;
  for (uint32_t k = threadIdx.x; k < K; k += FS_THREADS) {
    float y = fs_row[k];
    if (a.norm_w) {
      y = __fmul_rn(a.norm_w[k], __fmul_rn(rf, y));
      fs_row[k] = y;
    }
    m = fmaxf(m, fabsf(y));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = red[0];
    for (int w = 1; w < FS_THREADS / 32; ++w) mm = fmaxf(mm, red[w]);
    int e2 = 0;
    frexpf(mm, &e2);  // mm = f * 2^e2 with f in [0.5, 1)
    const int e = (mm == 0.0f || !isfinite(mm)) ? 0 : 15 - e2;
    ex_s = e;
    a.exps[t] = e;
  }
  __syncthreads();
  const int e = ex_s;
  __half* hi = reinterpret_cast<__half*>(a.hi) + (uint64_t)t * K;
  __half* lo = reinterpret_cast<__half*>(a.lo) + (uint64_t)t * K;
  for (uint32_t k = threadIdx.x; k < K; k += FS_THREADS) {
    const float s = ldexpf(fs_row[k], e);
    const __half h = __float2half_rn(s);
    hi[k] = h;
    lo[k] = __float2half_rn(isfinite(s) ? __fsub_rn(s, __half2float(h)) : 0.0f);
  }
}

template <int BN, int BM>
__host__ __device__ constexpr int f16_threads() { return (BN >= 64 ? 8 : BM / 16) * 32; }

// Stage ns 16-wide steps from step s0: weight rows m0.., hi and lo rows n0..
// (rows and tokens past the end re-read the last one, in bounds; their
// results are never stored).
template <bool PERM, int BN, int BM, int NTH>
__device__ __forceinline__ void f16_load(const GemmF16Args& a, uint8_t* st, uint32_t m0, uint32_t n0, uint32_t s0,
                                         uint32_t ns) {
  using T = FTile<BN, BM>;
  uint8_t* wt = st;
  uint8_t* xh = st + T::W_BYTES;
  uint8_t* xl = xh + T::X_BYTES;
  const uint32_t tid = threadIdx.x;
  const uint32_t pr = ns * 2;  // 16-byte pieces per row
  for (uint32_t i = tid; i < BM * pr; i += NTH) {
    const uint32_t r = i / pr, p = i - r * pr;
    const uint32_t gr = min(m0 + r, a.rows - 1);
    cp_async16(wt + tile_row<PERM>(r) * T::ROW + p * 16,
               a.w + (uint64_t)gr * a.row_bytes + (uint64_t)s0 * 32 + p * 16);
  }
  const uint8_t* hb = reinterpret_cast<const uint8_t*>(a.hi);
  const uint8_t* lb = reinterpret_cast<const uint8_t*>(a.lo);
  for (uint32_t i = tid; i < BN * pr; i += NTH) {
    const uint32_t t = i / pr, p = i - t * pr;
    const uint32_t gt = min(n0 + t, a.ntok - 1);
    const uint64_t off = (uint64_t)gt * a.K * 2 + (uint64_t)s0 * 32 + p * 16;
    cp_async16(xh + t * T::ROW + p * 16, hb + off);
    cp_async16(xl + t * T::ROW + p * 16, lb + off);
  }
}

template <int EPI, int BN, int BM>
__global__ void __launch_bounds__(f16_threads<BN, BM>(), 512 / f16_threads<BN, BM>()) gemm_f16_kernel(GemmF16Args a) {
  using T = FTile<BN, BM>;
  constexpr int NTH = f16_threads<BN, BM>(), NW = NTH / 32;
  constexpr bool PERM = EPI == EPI_SWIGLU;
  // BN = 64: warps 4 (rows) x 2 (tokens), 32 x 32 each; BN = 32: 8 x 1,
  // 16 x 32; BN = 16: 2 x 1, 16 x 16. NTW: 8-token n-tiles per warp.
  constexpr int WN = BN >= 64 ? 2 : 1, MT = BN >= 64 ? 2 : 1, RW = 16 * MT;
  constexpr int NTW = BN >= 32 ? 4 : BN / 8;
  static_assert(BN == 16 || BN == 32 || BN == 64, "token tile");
  static_assert((BN == 64 && BM == 128) || (BN < 64 && BM % 16 == 0 && BM <= 128), "row tile");
  static_assert(NW / WN * RW == BM && WN * NTW * 8 == BN, "the warps cover the tile");
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int wm = warp % (NW / WN), wn = warp / (NW / WN);
  const uint32_t S = a.K / 16, nch = (S + FB_KS - 1) / FB_KS;

  grid_dep_wait();  // hi / lo come from f16_split
#pragma unroll
  for (int s = 0; s < FB_S - 1; ++s) {
    if ((uint32_t)s < nch)
      f16_load<PERM, BN, BM, NTH>(a, smem + s * T::STAGE, m0, n0, s * FB_KS, min((uint32_t)FB_KS, S - s * FB_KS));
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
    cp_async_wait<FB_S - 2>();
    __syncthreads();  // stage c landed for every thread; stage c-1 is free
    const uint32_t cn = c + FB_S - 1;
    if (cn < nch)
      f16_load<PERM, BN, BM, NTH>(a, smem + (cn % FB_S) * T::STAGE, m0, n0, cn * FB_KS,
                                  min((uint32_t)FB_KS, S - cn * FB_KS));
    cp_async_commit();

    const uint8_t* wt = smem + (c % FB_S) * T::STAGE;
    const uint8_t* xh = wt + T::W_BYTES;
    const uint8_t* xl = xh + T::X_BYTES;
    const uint32_t ns = min((uint32_t)FB_KS, S - c * FB_KS);
#pragma unroll
    for (uint32_t b = 0; b < (uint32_t)FB_KS; ++b) {
      if (b >= ns) break;
      uint32_t af[MT][4], bh[NTW][2], bl[NTW][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int lr = wm * RW + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;  // this lane's ldmatrix row
        ldsm_x4(af[mt], wt + lr * T::ROW + b * 32 + (lane >> 4) * 16);
      }
#pragma unroll
      for (int np = 0; np < NTW / 2; ++np) {  // n-tiles 2np and 2np + 1
        const int lt = wn * 32 + np * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
        const int col = b * 32 + ((lane >> 3) & 1) * 16;
        uint32_t r[4];
        ldsm_x4(r, xh + lt * T::ROW + col);
        bh[2 * np][0] = r[0];
        bh[2 * np][1] = r[1];
        bh[2 * np + 1][0] = r[2];
        bh[2 * np + 1][1] = r[3];
        ldsm_x4(r, xl + lt * T::ROW + col);
        bl[2 * np][0] = r[0];
        bl[2 * np][1] = r[1];
        bl[2 * np + 1][0] = r[2];
        bl[2 * np + 1][1] = r[3];
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NTW; ++nt) {
          mma_f16(acc[mt][nt], af[mt], bh[nt]);
          mma_f16(acc[mt][nt], af[mt], bl[nt]);
        }
    }
  }

  if constexpr (EPI == EPI_SWIGLU) {
    // slots gid / gid + 8 of each 16-row tile hold gate / up of pair (tile row base)/2 + gid
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NTW; ++nt) {
        const uint32_t pair = (m0 + wm * RW + mt * 16) / 2 + gid;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t t = n0 + wn * 32 + nt * 8 + tig * 2 + h;
          if (t >= a.ntok || pair >= a.rows / 2) continue;
          const int e = a.exps[t];
          a.out[(uint64_t)t * a.out_stride + pair] =
              silu_mul(ldexpf(acc[mt][nt][h], -e), ldexpf(acc[mt][nt][2 + h], -e));
        }
      }
  } else {
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
          const float v = ldexpf(acc[mt][nt][e], -a.exps[t]);
          if (EPI == EPI_STORE) *o = v;
          else if (EPI == EPI_ADD) *o = __fadd_rn(*o, v);
          else *o = r < a.quirk_cols ? __fadd_rn(*o, v) : v;
        }
  }
}

template <int EPI, int BN, int BM>
cudaError_t f16_gemm_launch_bn(const GemmF16Args& a, const LaunchCfg& lc) {
  using T = FTile<BN, BM>;
  cudaError_t e = cudaFuncSetAttribute(gemm_f16_kernel<EPI, BN, BM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       T::SMEM);
  if (e != cudaSuccess) return e;
  const dim3 grid((a.ntok + BN - 1) / BN, (a.rows + BM - 1) / BM);
  return launch_kernel(gemm_f16_kernel<EPI, BN, BM>, grid, dim3(f16_threads<BN, BM>()), (uint32_t)T::SMEM, lc, a);
}

// 16-token passes on 32-row tiles (a 4096-row projection still spreads over
// 128 CTAs), up to 32 tokens on 128 x 32 tiles, more on 128 x 64.
template <int EPI>
cudaError_t f16_gemm_launch(const GemmF16Args& a, const LaunchCfg& lc) {
  if (a.ntok <= 16) return f16_gemm_launch_bn<EPI, 16, 32>(a, lc);
  return a.ntok <= 32 ? f16_gemm_launch_bn<EPI, 32, 128>(a, lc) : f16_gemm_launch_bn<EPI, 64, 128>(a, lc);
}
}  // namespace

bool gemm_f16_supported(const GemmF16Args& a, int epi) {
  if (epi != EPI_STORE && epi != EPI_ADD && epi != EPI_QUIRK && epi != EPI_SWIGLU) return false;
  if (!a.w || !a.x || !a.hi || !a.lo || !a.exps || !a.out) return false;
  if (a.rows == 0 || a.ntok == 0 || a.K == 0 || a.K % 32) return false;
  if ((a.rows + 31) / 32 > 65535u) return false;
  if ((uintptr_t)a.w % 16 || a.row_bytes % 16 || a.row_bytes < 2ull * a.K) return false;
  if ((uintptr_t)a.x % 16 || a.x_stride % 4 || a.x_stride < a.K) return false;  // float4 row loads
  if ((uintptr_t)a.hi % 16 || (uintptr_t)a.lo % 16 || (uintptr_t)a.exps % 4) return false;
  if (a.norm_w && (uintptr_t)a.norm_w % 4) return false;
  if ((uint64_t)a.K * 4 > 227u * 1024u) return false;  // f16_split stages a row in shared memory
  if (epi == EPI_SWIGLU && a.rows % 16) return false;  // gate/up pairs inside 16-row tiles
  return true;
}

cudaError_t gemm_f16(const GemmF16Args& a, int epi, const LaunchCfg& lc) {
  if (!gemm_f16_supported(a, epi)) return cudaErrorInvalidValue;
  const uint32_t smem = a.K * 4;
  cudaError_t e = cudaFuncSetAttribute(f16_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  e = launch_kernel(f16_split_kernel, dim3(a.ntok), dim3(FS_THREADS), smem, lc, a);
  if (e != cudaSuccess) return e;
  switch (epi) {
    case EPI_STORE: return f16_gemm_launch<EPI_STORE>(a, lc);
    case EPI_ADD: return f16_gemm_launch<EPI_ADD>(a, lc);
    case EPI_QUIRK: return f16_gemm_launch<EPI_QUIRK>(a, lc);
    default: return f16_gemm_launch<EPI_SWIGLU>(a, lc);
  }
}

}  // namespace k
}  // namespace yl
