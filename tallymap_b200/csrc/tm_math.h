// f32 transcendentals of the tallymap B200 backend, identical on the host and the device.
//
// The reference lowers float transcendentals to libdevice on the GPU and to libm on the CPU target
// (backends/kernel/kernel.py:29-57, backends/kernel/host.py:9-11), so its two targets agree only to rounding and a
// chaotic item (photon transport, an adaptive ODE) can take a different number of steps on each.  Here one
// implementation serves both: each function evaluates a textbook method in double precision using only IEEE
// + - * / (every operation correctly rounded; FMA contraction is off on both sides: --fmad=false on the device,
// -ffp-contract=off on the host) and rounds once to f32, so host and device results are bitwise equal and within
// about half an ulp of the exact value.  Methods:
//   log   x = 2^e m, m in [sqrt(1/2), sqrt(2)); log m = 2 atanh(t), t = (m - 1) / (m + 1), |t| <= 0.1716, by its
//         odd power series to t^21 (truncation below 1e-17 relative); log x = e ln 2 + log m
//   exp   x = n ln 2 + r, n = nearest integer to x / ln 2, r by a two-part (Cody-Waite) ln 2, |r| <= 0.35; e^r by
//         its Taylor series to r^16; scaled by 2^n built from the exponent bits
//   sin, cos   x = n pi/2 + r by a three-part pi/2 (exact products for |x| < 2^20), |r| <= pi/4; Taylor series of sin and cos
//         to r^19 / r^20, then the quadrant's sign and swap
//   pow   x^y = exp(y log x) for x > 0 (the exponent's argument formed in double), IEEE special cases otherwise
#pragma once
#ifdef __CUDACC_RTC__
#include <cuda/std/cstdint>
typedef cuda::std::uint32_t uint32_t;
typedef cuda::std::uint64_t uint64_t;
typedef cuda::std::int32_t int32_t;
typedef cuda::std::int64_t int64_t;
#else
#include <cstdint>
#include <cstring>
#endif

#if defined(__CUDACC__)
#define TM_HD __host__ __device__ __forceinline__
#else
#define TM_HD inline
#endif

namespace tmm {

TM_HD uint32_t f2u(float x) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(x);
#else
  uint32_t u;
  std::memcpy(&u, &x, 4);
  return u;
#endif
}
TM_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float x;
  std::memcpy(&x, &u, 4);
  return x;
#endif
}
TM_HD double u64_2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)u);
#else
  double x;
  std::memcpy(&x, &u, 8);
  return x;
#endif
}
// 2^n as a double for -1022 <= n <= 1023 (exact)
TM_HD double pow2(int n) { return u64_2d((uint64_t)(n + 1023) << 52); }
TM_HD float f32_inf() { return u2f(0x7f800000u); }
TM_HD float f32_nan() { return u2f(0x7fc00000u); }
TM_HD bool isnan_(float x) { return x != x; }

// double -> float, round to nearest even (the host's and the device's conversion)
TM_HD float to_f32(double x) {
#if defined(__CUDA_ARCH__)
  return __double2float_rn(x);
#else
  return (float)x;
#endif
}

constexpr double kLn2Hi = 6.93147180369123816490e-01;   // ln 2, high part (32 significant bits)
constexpr double kLn2Lo = 1.90821492927058770002e-10;   // ln 2 - kLn2Hi (sum within 2e-26)
constexpr double kLn2 = 6.93147180559945286227e-01;
constexpr double kInvLn2 = 1.44269504088896338700e+00;
constexpr double kSqrtHalf = 7.07106781186547572737e-01;
constexpr double kPio2_1 = 1.5707963267341256;          // pi/2 in three parts: 32 + 32 + 53 significant bits, so
constexpr double kPio2_2 = 6.077100506303966e-11;        // n * part is exact for |n| < 2^21 (sum within 1e-37)
constexpr double kPio2_3 = 2.0222662487959506e-21;
constexpr double kTwoOverPi = 6.36619772367581382433e-01;

// log m for m in [sqrt(1/2), sqrt(2)): 2 (t + t^3/3 + ... + t^21/21)
TM_HD double log_core(double m) {
  const double t = (m - 1.0) / (m + 1.0);
  const double t2 = t * t;
  double p = 1.0 / 21.0;
  p = p * t2 + 1.0 / 19.0;
  p = p * t2 + 1.0 / 17.0;
  p = p * t2 + 1.0 / 15.0;
  p = p * t2 + 1.0 / 13.0;
  p = p * t2 + 1.0 / 11.0;
  p = p * t2 + 1.0 / 9.0;
  p = p * t2 + 1.0 / 7.0;
  p = p * t2 + 1.0 / 5.0;
  p = p * t2 + 1.0 / 3.0;
  p = p * t2 + 1.0;
  return 2.0 * t * p;
}

// natural log of a positive finite double argument formed from an f32 (or an f32 product): e ln 2 + log m
TM_HD double log_pos(double x) {
  // split x = 2^e m with m in [1, 2) using the double's exponent bits
#if defined(__CUDA_ARCH__)
  uint64_t b = (uint64_t)__double_as_longlong(x);
#else
  uint64_t b;
  std::memcpy(&b, &x, 8);
#endif
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  double m = u64_2d((b & 0x000fffffffffffffull) | 0x3ff0000000000000ull);
  if (m > 1.0 / kSqrtHalf) {   // m in (sqrt 2, 2): use m / 2 in (sqrt(1/2), 1)
    m = m * 0.5;
    e += 1;
  }
  return (double)e * kLn2Hi + (log_core(m) + (double)e * kLn2Lo);
}

TM_HD float logf(float x) {
  if (isnan_(x) || x < 0.0f) return f32_nan();
  if (x == 0.0f) return -f32_inf();
  if (x == f32_inf()) return x;
  return to_f32(log_pos((double)x));    // (an f32 subnormal is a normal double)
}

// e^r for |r| <= 0.35: Taylor to r^16
TM_HD double exp_core(double r) {
  double p = 1.0 / 20922789888000.0;   // 1/16!
  p = p * r + 1.0 / 1307674368000.0;
  p = p * r + 1.0 / 87178291200.0;
  p = p * r + 1.0 / 6227020800.0;
  p = p * r + 1.0 / 479001600.0;
  p = p * r + 1.0 / 39916800.0;
  p = p * r + 1.0 / 3628800.0;
  p = p * r + 1.0 / 362880.0;
  p = p * r + 1.0 / 40320.0;
  p = p * r + 1.0 / 5040.0;
  p = p * r + 1.0 / 720.0;
  p = p * r + 1.0 / 120.0;
  p = p * r + 1.0 / 24.0;
  p = p * r + 1.0 / 6.0;
  p = p * r + 0.5;
  p = p * r + 1.0;
  return p * r + 1.0;
}

// e^x in double for |x| <= 200 (enough for any f32 result: e^89 overflows f32, e^-104 underflows it)
TM_HD double exp_d(double x) {
  const double k = x * kInvLn2;
  const double n = (double)(long long)(k < 0.0 ? k - 0.5 : k + 0.5);
  const double r = (x - n * kLn2Hi) - n * kLn2Lo;
  return exp_core(r) * pow2((int)n);
}

TM_HD float expf(float x) {
  if (isnan_(x)) return x;
  if (x > 89.0f) return f32_inf();
  if (x < -104.0f) return 0.0f;
  return to_f32(exp_d((double)x));
}

TM_HD double sin_core(double r) {   // |r| <= pi/4
  const double r2 = r * r;
  double p = -1.0 / 121645100408832000.0;   // -1/19!
  p = p * r2 + 1.0 / 355687428096000.0;
  p = p * r2 - 1.0 / 1307674368000.0;
  p = p * r2 + 1.0 / 6227020800.0;
  p = p * r2 - 1.0 / 39916800.0;
  p = p * r2 + 1.0 / 362880.0;
  p = p * r2 - 1.0 / 5040.0;
  p = p * r2 + 1.0 / 120.0;
  p = p * r2 - 1.0 / 6.0;
  return r + r * (r2 * p);
}

TM_HD double cos_core(double r) {   // |r| <= pi/4
  const double r2 = r * r;
  double p = 1.0 / 2432902008176640000.0;   // 1/20!
  p = p * r2 - 1.0 / 6402373705728000.0;
  p = p * r2 + 1.0 / 20922789888000.0;
  p = p * r2 - 1.0 / 87178291200.0;
  p = p * r2 + 1.0 / 479001600.0;
  p = p * r2 - 1.0 / 3628800.0;
  p = p * r2 + 1.0 / 40320.0;
  p = p * r2 - 1.0 / 720.0;
  p = p * r2 + 1.0 / 24.0;
  p = p * r2 - 0.5;
  return 1.0 + r2 * p;
}

// sin and cos of an f32 argument with |x| < 2^20 (larger: NaN; the items here stay within [-8, 8])
TM_HD void sincosf(float xf, float* s, float* c) {
  const double x = (double)xf;
  if (isnan_(xf) || !(x < 1048576.0 && x > -1048576.0)) {
    *s = f32_nan();
    *c = f32_nan();
    return;
  }
  const double k = x * kTwoOverPi;
  const long long n = (long long)(k < 0.0 ? k - 0.5 : k + 0.5);
  const double dn = (double)n;
  const double r = ((x - dn * kPio2_1) - dn * kPio2_2) - dn * kPio2_3;
  const double sr = sin_core(r), cr = cos_core(r);
  switch ((int)(n & 3)) {
    case 0: *s = to_f32(sr); *c = to_f32(cr); break;
    case 1: *s = to_f32(cr); *c = to_f32(-sr); break;
    case 2: *s = to_f32(-sr); *c = to_f32(-cr); break;
    default: *s = to_f32(-cr); *c = to_f32(sr); break;
  }
}

TM_HD float sinf(float x) { float s, c; sincosf(x, &s, &c); return s; }
TM_HD float cosf(float x) { float s, c; sincosf(x, &s, &c); return c; }

// x^y for x > 0 finite, y finite: e^(y log x) formed in double; x = 0, negative, non-finite: the IEEE special cases
// the items need (x = 0: 0 for y > 0, +inf for y < 0; 1 for y = 0; NaN for x < 0 with non-integer y)
TM_HD float powf(float x, float y) {
  if (y == 0.0f) return 1.0f;
  if (isnan_(x) || isnan_(y)) return f32_nan();
  if (x == 0.0f) return y > 0.0f ? 0.0f : f32_inf();
  if (x < 0.0f) return f32_nan();
  if (x == f32_inf()) return y > 0.0f ? f32_inf() : 0.0f;
  const double a = (double)y * log_pos((double)x);
  if (a > 89.0) return f32_inf();
  if (a < -104.0) return 0.0f;
  return to_f32(exp_d(a));
}

}  // namespace tmm
