// Staging and fragment helpers shared by the mma.sync GEMMs (gemm_q8.cu,
// gemm_f16.cu): cp.async copies into shared memory, ldmatrix fragment loads,
// and the gate/up row permutation of the SwiGLU tiles.
#pragma once
#include "device.cuh"

namespace yl {
namespace k {
namespace gu {
using yl::dev::smem_u32;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ldmatrix: four (two) 8x8 tiles of 16-bit elements, tile j's row addresses
// from lanes 8j..8j+7; lane l receives the 4 bytes at (l%4)*4 of row l/4 of
// each tile. For f16 data that is the m16n8k16 fragment layout, for int8 data
// the m16n8k32 one (4 consecutive bytes).
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}

// Shared-memory row of weight row i of the tile: with PERM, in each aligned
// group of 16 rows the even rows (gate) go to the first 8 slots and the odd
// rows (up) to the last 8, in order.
template <bool PERM>
__device__ __forceinline__ uint32_t tile_row(uint32_t i) {
  if (!PERM) return i;
  const uint32_t w = i & 15u;
  return (i & ~15u) + (w >> 1) + ((w & 1u) << 3);
}

}  // namespace gu
}  // namespace k
}  // namespace yl
