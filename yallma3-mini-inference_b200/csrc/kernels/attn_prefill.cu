// Causal GQA attention for multi-token passes (prefill), forward.rs:299-400:
// s = (q.k) * scale, keys after the query's position masked, softmax over the
// visible keys, out = sum p * V, then the Q8_0 quantization of the output
// (forward.rs:191). f32 on the CUDA cores, flash-style:
//  * one CTA per (KV head, block of query tokens): the block's query rows are
//    (token, query head of this KV head) pairs, 64 rows, so every key/value
//    row brought into shared memory serves 64 queries (the per-token kernel
//    re-reads the whole cache for each token);
//  * keys in tiles of 32 (cp.async), online softmax per row in registers
//    (max, sum and the 4 x HD/16 output accumulators of a thread's rows),
//    probabilities exchanged through shared memory for the P.V product;
//  * the longest (latest) query blocks are scheduled first.
#include "device.cuh"
#include "kernels.h"

namespace yl {
namespace k {
using namespace yl::dev;

namespace {
constexpr int AP_THREADS = 256, AP_R = 64, AP_BK = 32;

template <int HD>
struct ApSmem {
  static constexpr int QS = HD + 4;  // padded rows
  static constexpr int KS = HD + 4;
  static constexpr int PS = AP_BK + 1;
  static constexpr int Q_FLOATS = AP_R * QS;
  static constexpr int K_FLOATS = AP_BK * KS;
  static constexpr int V_FLOATS = AP_BK * HD;
  static constexpr int P_FLOATS = AP_R * PS;
  static constexpr int BYTES = (Q_FLOATS + K_FLOATS + V_FLOATS + P_FLOATS) * 4;
};

__device__ __forceinline__ void ap_cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

template <int HD>
__global__ void __launch_bounds__(AP_THREADS, 2) attn_prefill_kernel(AttnArgs a, uint32_t bq) {
  grid_dep_launch();
  grid_dep_wait();
  using L = ApSmem<HD>;
  constexpr int EV = HD / 16;  // output columns per thread
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;
  float* ks = qs + L::Q_FLOATS;
  float* vs = ks + L::K_FLOATS;
  float* ps = vs + L::V_FLOATS;
  const uint32_t kvh = blockIdx.x;
  const uint32_t qb = gridDim.y - 1 - blockIdx.y;  // latest (longest) blocks first
  const uint32_t kv_mul = a.n_heads / a.n_kv_heads;
  const uint32_t t0 = qb * bq, nt = min(bq, a.ntok - t0);
  const uint32_t nrows = nt * kv_mul;  // row = token_in_block * kv_mul + head_in_group
  const uint32_t pos0 = a.state ? (uint32_t)a.state->pos : a.pos0;
  const uint32_t att = a.n_heads * HD;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;

  for (uint32_t i = tid; i < (uint32_t)AP_R * (HD / 4); i += AP_THREADS) {
    const uint32_t r = i / (HD / 4), d4 = i % (HD / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nrows) {
      const uint32_t tl = r / kv_mul, hh = r % kv_mul;
      v = *reinterpret_cast<const float4*>(a.q + (uint64_t)(t0 + tl) * att + (kvh * kv_mul + hh) * HD + d4 * 4);
    }
    *reinterpret_cast<float4*>(qs + r * L::QS + d4 * 4) = v;
  }
  // this thread's rows ty*4..+3: absolute query positions (rows past the
  // block's tokens act as its first token; they are never stored)
  uint32_t qp[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t r = ty * 4 + i;
    qp[i] = pos0 + t0 + (r < nrows ? r / kv_mul : 0);
  }
  float o[4][EV], m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int e = 0; e < EV; ++e) o[i][e] = 0.0f;
  }
  const uint32_t kend = pos0 + t0 + nt;  // keys [0, kend) are visible to the block's last token
  for (uint32_t p0 = 0; p0 < kend; p0 += AP_BK) {
    __syncthreads();  // the previous tile's K, V and P are consumed (and q is stored)
    for (uint32_t i = tid; i < (uint32_t)AP_BK * (HD / 4); i += AP_THREADS) {
      const uint32_t kk = i / (HD / 4), d4 = i % (HD / 4);
      const uint32_t p = min(p0 + kk, kend - 1);  // past-the-end keys re-read the last one (masked)
      ap_cp16(ks + kk * L::KS + d4 * 4, a.kcache + (uint64_t)p * a.kv_dim + kvh * HD + d4 * 4);
      ap_cp16(vs + kk * HD + d4 * 4, a.vcache + (uint64_t)p * a.kv_dim + kvh * HD + d4 * 4);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();

    float s[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = 0.0f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
      float4 qv[4], kv[2];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(qs + (ty * 4 + i) * L::QS + d);
#pragma unroll
      for (int j = 0; j < 2; ++j) kv[j] = *reinterpret_cast<const float4*>(ks + (tx * 2 + j) * L::KS + d);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
          s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
          s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
          s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t p = p0 + tx * 2 + j;
        s[i][j] = p <= qp[i] ? __fmul_rn(s[i][j], a.scale) : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      // key 0 is in the first tile and visible to every row, so m[i] is
      // finite from then on and fully masked later tiles give exp(-inf) = 0
      const float m_new = fmaxf(m[i], mx);
      const float corr = expf(m[i] - m_new);
      const float e0 = expf(s[i][0] - m_new), e1 = expf(s[i][1] - m_new);
      float rs = e0 + e1;
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * corr + rs;
      m[i] = m_new;
#pragma unroll
      for (int e = 0; e < EV; ++e) o[i][e] *= corr;
      ps[(ty * 4 + i) * L::PS + tx * 2] = e0;
      ps[(ty * 4 + i) * L::PS + tx * 2 + 1] = e1;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < AP_BK; ++kk) {
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = ps[(ty * 4 + i) * L::PS + kk];
      float vv[EV];
#pragma unroll
      for (int e4 = 0; e4 < EV; e4 += 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(vs + kk * HD + tx * EV + e4);
        vv[e4] = v4.x;
        vv[e4 + 1] = v4.y;
        vv[e4 + 2] = v4.z;
        vv[e4 + 3] = v4.w;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < EV; ++e) o[i][e] = fmaf(pv[i], vv[e], o[i][e]);
    }
  }
  __syncthreads();  // q rows are no longer read: they take the normalized output
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float inv = l[i] > 0.0f ? 1.0f / l[i] : 0.0f;
#pragma unroll
    for (int e = 0; e < EV; ++e) qs[(ty * 4 + i) * L::QS + tx * EV + e] = o[i][e] * inv;
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  for (uint32_t pi = warp; pi < nrows * (HD / 32); pi += AP_THREADS / 32) {  // warp-uniform
    const uint32_t r = pi / (HD / 32), b = pi % (HD / 32);
    const uint32_t tl = r / kv_mul, hh = r % kv_mul;
    const float v = qs[r * L::QS + b * 32 + lane];
    const uint64_t k = (uint64_t)(t0 + tl) * att + (kvh * kv_mul + hh) * HD + b * 32 + lane;
    if (a.out) a.out[k] = v;
    if (a.q8) {
      float sc;
      const int8_t qv = quant_q8_lane(v, &sc);
      a.q8[k] = qv;
      if (lane == 0) a.s8[k / 32] = sc;
    }
  }
}

template <int HD>
cudaError_t ap_launch(const AttnArgs& a, const LaunchCfg& lc) {
  const uint32_t kv_mul = a.n_heads / a.n_kv_heads;
  const uint32_t bq = AP_R / kv_mul;
  cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       ApSmem<HD>::BYTES);
  if (e != cudaSuccess) return e;
  const dim3 grid(a.n_kv_heads, (a.ntok + bq - 1) / bq);
  return launch_kernel(attn_prefill_kernel<HD>, grid, dim3(AP_THREADS), (uint32_t)ApSmem<HD>::BYTES, lc, a, bq);
}
}  // namespace

bool attention_prefill_ok(const AttnArgs& a) {
  if (a.ntok == 0 || a.n_kv_heads == 0 || a.n_heads % a.n_kv_heads) return false;
  const uint32_t kv_mul = a.n_heads / a.n_kv_heads;
  if (kv_mul == 0 || kv_mul > 8 || (a.head_size != 64 && a.head_size != 128)) return false;
  if ((a.ntok + AP_R / kv_mul - 1) / (AP_R / kv_mul) > 65535u) return false;
  if (((uintptr_t)a.q | (uintptr_t)a.kcache | (uintptr_t)a.vcache) % 16 || a.kv_dim % 4) return false;
  if (a.kv_dim < a.n_kv_heads * a.head_size) return false;
  return a.out || (a.q8 && a.s8);
}

cudaError_t attention_prefill(const AttnArgs& a, const LaunchCfg& lc) {
  if (!attention_prefill_ok(a)) return cudaErrorInvalidValue;
  return a.head_size == 64 ? ap_launch<64>(a, lc) : ap_launch<128>(a, lc);
}

}  // namespace k
}  // namespace yl
