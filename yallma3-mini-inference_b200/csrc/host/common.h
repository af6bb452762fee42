// Shared host-side helpers: error reporting, f16 conversion, CUDA checks.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <new>
#include <string>

#include "../../../include/yallma3.h"

namespace yl {

// Thread-local message behind yl_last_error().
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

// Runs f (which returns a yl status) so that no C++ exception crosses the
// C-ABI into the host: a failed host allocation becomes YL_ERR_OOM, any other
// exception YL_ERR_FORMAT.
template <class F>
int guarded(F&& f) {
  try {
    return f();
  } catch (const std::bad_alloc&) {
    return fail(YL_ERR_OOM, "host memory allocation failed");
  } catch (const std::exception& e) {
    return fail(YL_ERR_FORMAT, std::string("unexpected error: ") + e.what());
  } catch (...) {
    return fail(YL_ERR_FORMAT, "unexpected error");
  }
}

// IEEE binary16 <-> binary32 (round to nearest even on narrowing).
inline float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
      bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0));
  if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to inf
  if (absx < 0x38800000u) {                                    // subnormal or zero in f16
    if (absx < 0x33000000u) return (uint16_t)sign;
    uint32_t e = absx >> 23;
    uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126 - e;  // 14 - (e - 127) + 13 - 1
    uint32_t r = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (r & 1))) ++r;
    return (uint16_t)(sign | r);
  }
  uint32_t r = ((absx >> 13) - (112u << 10));
  uint32_t rem = absx & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) ++r;
  return (uint16_t)(sign | r);
}

inline uint64_t round_up(uint64_t a, uint64_t b) { return (a + b - 1) / b * b; }

// Argument checks shared by yl_fused_attention and yl_fused_attention_static
// (one definition, so the two entry points accept the same requests).
int check_attention_args(const float* output, const float* sq, const float* kc, const float* vc, uint64_t seq_len,
                         uint64_t batch, uint64_t n_heads, uint64_t n_kv_heads, uint64_t head_size,
                         uint32_t start_pos, uint64_t kv_dim);

}  // namespace yl

#define YL_CUDA_TRY(expr)                                                              \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return yl::fail(e_ == cudaErrorMemoryAllocation ? YL_ERR_OOM : YL_ERR_CUDA,      \
                      std::string(#expr) + ": " + cudaGetErrorString(e_));             \
  } while (0)
