// yl_expf: e^x of a float, evaluated in double precision and rounded once to
// float. Written from the mathematics, for host and device alike:
//   x = n*ln2 + r, n = rint(x/ln2), |r| <= ln2/2  (ln2 split in a high part
//   with 44 significant bits, so n*LN2_HI is exact, and a low part);
//   e^r by its Taylor series to r^13/13! (truncation below 4e-18 relative),
//   Horner steps as fused multiply-adds;
//   e^x = e^r * 2^n (exact scaling), then one round-to-nearest to float.
// The double result is within about 2^-51 of e^x, so the float rounding is
// the correctly rounded one except where e^x lies that close to a rounding
// midpoint. Every operation is an IEEE double add, multiply or fused
// multiply-add (no contraction choices left to the compiler), so the host and
// the device produce the same bits; tests/test_expf_exact.py checks the host
// instantiation against the C library's expf (the function the reference's
// f32::exp calls) for every float input.
//
// The device forward uses it wherever the reference calls exp: the softmax of
// fused_attention (forward.rs:299-400) and the SiLU of forward.rs:221-237.
#pragma once
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define YL_EXP_HD __host__ __device__ __forceinline__
#else
#define YL_EXP_HD inline
#endif

namespace yl {

YL_EXP_HD double yl_pow2i(int n) {  // 2^n for n in [-1022, 1023]
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)(n + 1023) << 52);
#else
  const uint64_t b = (uint64_t)(n + 1023) << 52;
  double d;
  memcpy(&d, &b, 8);
  return d;
#endif
}

YL_EXP_HD float yl_f64_to_f32(double d) {
#if defined(__CUDA_ARCH__)
  return __double2float_rn(d);
#else
  return (float)d;
#endif
}

YL_EXP_HD double yl_rint(double d) {
#if defined(__CUDA_ARCH__)
  return rint(d);
#else
  return __builtin_rint(d);
#endif
}

YL_EXP_HD double yl_fma(double a, double b, double c) {
#if defined(__CUDA_ARCH__)
  return fma(a, b, c);
#else
  return __builtin_fma(a, b, c);
#endif
}

YL_EXP_HD float yl_expf(float x) {
  if (!(x == x)) return x;                          // NaN
  if (x > 100.0f) return __builtin_huge_valf();     // above ln(FLT_MAX): +inf
  if (x < -110.0f) return 0.0f;                     // below ln(smallest subnormal / 2): +0
  const double d = (double)x;
  const double kInvLn2 = 0x1.71547652b82fep+0;
  const double kLn2Hi = 0x1.62e42fefa3a00p-1;       // 44 significant bits
  const double kLn2Lo = -0x1.0ca86c3898d00p-49;     // ln2 - kLn2Hi
  const double n = yl_rint(d * kInvLn2);
  double r = yl_fma(-n, kLn2Hi, d);                 // exact
  r = yl_fma(-n, kLn2Lo, r);
  // 1/k!, k = 13 .. 0
  double p = 0x1.6124613a86d09p-33;
  p = yl_fma(p, r, 0x1.1eed8eff8d898p-29);
  p = yl_fma(p, r, 0x1.ae64567f544e4p-26);
  p = yl_fma(p, r, 0x1.27e4fb7789f5cp-22);
  p = yl_fma(p, r, 0x1.71de3a556c734p-19);
  p = yl_fma(p, r, 0x1.a01a01a01a01ap-16);
  p = yl_fma(p, r, 0x1.a01a01a01a01ap-13);
  p = yl_fma(p, r, 0x1.6c16c16c16c17p-10);
  p = yl_fma(p, r, 0x1.1111111111111p-7);
  p = yl_fma(p, r, 0x1.5555555555555p-5);
  p = yl_fma(p, r, 0x1.5555555555555p-3);
  p = yl_fma(p, r, 0x1.0000000000000p-1);
  p = yl_fma(p, r, 1.0);
  p = yl_fma(p, r, 1.0);
  return yl_f64_to_f32(p * yl_pow2i((int)n));
}

}  // namespace yl
