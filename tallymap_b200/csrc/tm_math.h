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
//   atan  |x| > 1: pi/2 - atan(1/x); t > tan(pi/12): pi/6 + atan((t sqrt3 - 1) / (t + sqrt3)); then the odd Taylor
//         series to t^31 for t <= 0.268 (truncation below 2e-20 relative); atan2 the quadrant of atan(|y| / |x|) and
//         C's special cases; asin x = atan(x / sqrt((1 - x)(1 + x))), acos x = 2 atan(sqrt((1 - x) / (1 + x)))
//   tan   the sin / cos reduction above, sin r / cos r or -cos r / sin r by the quadrant's parity
//   sinh, cosh, asinh, acosh, atanh   their exponential and logarithmic forms, by the Taylor series to x^7 for
//         |x| < 2^-10 where the forms cancel
//   exp2, log2   e^(x ln 2) and log x / ln 2; cbrt e^(log|x| / 3) and one Newton step, with the sign of x
//   erf   |x| < 2: its Maclaurin series (46 terms); erfc, x >= 2: Laplace's continued fraction
//         erfc x = e^(-x^2) / sqrt(pi) / (x + (1/2) / (x + 1 / (x + (3/2) / (x + ...)))) to depth 60; else 1 - the other
//   erfinv  five Newton steps on erf (on erfc above 1/2, from 1 - y exact in double), from the series
//         (sqrt(pi) / 2)(y + pi y^3 / 12 + 7 pi^2 y^5 / 480 + 127 pi^3 y^7 / 40320) for y <= 0.9 and from the
//         asymptotic x^2 = -log(sqrt(pi) x (1 - y)), iterated three times, above
#pragma once
#ifdef __CUDACC_RTC__
#include <cuda/std/cstdint>
typedef cuda::std::uint32_t uint32_t;
typedef cuda::std::uint64_t uint64_t;
typedef cuda::std::int32_t int32_t;
typedef cuda::std::int64_t int64_t;
#else
#include <cmath>
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
  if (xf == 0.0f) {   // sin(-0) = -0
    *s = xf;
    *c = 1.0f;
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

constexpr double kPi = 3.14159265358979311600e+00;
constexpr double kPio2 = 1.57079632679489655800e+00;
constexpr double kPio4 = 7.85398163397448278999e-01;
constexpr double kPio6 = 5.23598775598298815658e-01;
constexpr double kSqrt3 = 1.73205080756887719318e+00;
constexpr double kTanPio12 = 2.67949192431122695603e-01;   // 2 - sqrt 3
constexpr double kSqrtPi = 1.77245385090551588192e+00;
constexpr double kTwoOverSqrtPi = 1.12837916709551255856e+00;
constexpr double kTiny = 9.765625e-04;                      // 2^-10: below it the odd Taylor forms

TM_HD double sqrt_d(double x) {     // IEEE square root, correctly rounded on both sides
#if defined(__CUDA_ARCH__)
  return __dsqrt_rn(x);
#else
  return std::sqrt(x);
#endif
}
TM_HD bool sign_(float x) { return (f2u(x) >> 31) != 0u; }
TM_HD bool isinf_(float x) { return x == f32_inf() || x == -f32_inf(); }
TM_HD float with_sign(double r, bool neg) { return to_f32(neg ? -r : r); }

// atan t for 0 <= t <= tan(pi/12): sum_k (-1)^k t^(2k+1) / (2k+1), k <= 15
TM_HD double atan_core(double t) {
  const double t2 = t * t;
  double p = -1.0 / 31.0;
  p = p * t2 + 1.0 / 29.0;
  p = p * t2 - 1.0 / 27.0;
  p = p * t2 + 1.0 / 25.0;
  p = p * t2 - 1.0 / 23.0;
  p = p * t2 + 1.0 / 21.0;
  p = p * t2 - 1.0 / 19.0;
  p = p * t2 + 1.0 / 17.0;
  p = p * t2 - 1.0 / 15.0;
  p = p * t2 + 1.0 / 13.0;
  p = p * t2 - 1.0 / 11.0;
  p = p * t2 + 1.0 / 9.0;
  p = p * t2 - 1.0 / 7.0;
  p = p * t2 + 1.0 / 5.0;
  p = p * t2 - 1.0 / 3.0;
  p = p * t2 + 1.0;
  return t * p;
}
TM_HD double atan_unit(double t) {   // 0 <= t <= 1
  if (t > kTanPio12) return kPio6 + atan_core((t * kSqrt3 - 1.0) / (t + kSqrt3));
  return atan_core(t);
}
TM_HD double atan_d(double x) {      // x >= 0, +inf allowed
  if (x > 1.0) return kPio2 - atan_unit(1.0 / x);
  return atan_unit(x);
}

TM_HD float atanf(float x) {
  if (isnan_(x) || x == 0.0f) return x;
  return with_sign(atan_d(sign_(x) ? -(double)x : (double)x), sign_(x));
}

// C's atan2: the angle of (x, y), with its signed-zero and infinite special cases
TM_HD float atan2f(float y, float x) {
  if (isnan_(x) || isnan_(y)) return f32_nan();
  const bool yn = sign_(y), xn = sign_(x);
  double r;
  if (y == 0.0f) {
    r = xn ? kPi : 0.0;
  } else if (x == 0.0f) {
    r = kPio2;
  } else if (isinf_(y)) {
    r = isinf_(x) ? (xn ? 3.0 * kPio4 : kPio4) : kPio2;
  } else if (isinf_(x)) {
    r = xn ? kPi : 0.0;
  } else {
    const double ay = yn ? -(double)y : (double)y, ax = xn ? -(double)x : (double)x;
    const double a = atan_d(ay / ax);
    r = xn ? kPi - a : a;
  }
  return with_sign(r, yn);
}

TM_HD float asinf(float x) {
  if (isnan_(x) || x == 0.0f) return x;
  const double a = sign_(x) ? -(double)x : (double)x;
  if (a > 1.0) return f32_nan();
  if (a == 1.0) return with_sign(kPio2, sign_(x));
  return with_sign(atan_d(a / sqrt_d((1.0 - a) * (1.0 + a))), sign_(x));
}

TM_HD float acosf(float x) {
  if (isnan_(x) || x > 1.0f || x < -1.0f) return f32_nan();
  if (x == 1.0f) return 0.0f;
  if (x == -1.0f) return to_f32(kPi);
  const double d = (double)x;
  return to_f32(2.0 * atan_d(sqrt_d((1.0 - d) / (1.0 + d))));
}

// tan of an f32 argument with |x| < 2^20 (larger: NaN), by the sin / cos reduction
TM_HD float tanf(float xf) {
  const double x = (double)xf;
  if (isnan_(xf) || !(x < 1048576.0 && x > -1048576.0)) return f32_nan();
  if (xf == 0.0f) return xf;
  const double k = x * kTwoOverPi;
  const long long n = (long long)(k < 0.0 ? k - 0.5 : k + 0.5);
  const double dn = (double)n;
  const double r = ((x - dn * kPio2_1) - dn * kPio2_2) - dn * kPio2_3;
  const double sr = sin_core(r), cr = cos_core(r);
  return to_f32((n & 1) ? -cr / sr : sr / cr);
}

TM_HD float sinhf(float x) {
  if (isnan_(x) || x == 0.0f) return x;
  const double a = sign_(x) ? -(double)x : (double)x;
  if (a > 200.0) return sign_(x) ? -f32_inf() : f32_inf();
  double r;
  if (a < kTiny) {
    const double a2 = a * a;
    r = a + a * (a2 * (1.0 / 6.0 + a2 * (1.0 / 120.0 + a2 * (1.0 / 5040.0))));
  } else {
    const double e = exp_d(a);
    r = 0.5 * (e - 1.0 / e);
  }
  return with_sign(r, sign_(x));
}

TM_HD float coshf(float x) {
  if (isnan_(x)) return x;
  const double a = sign_(x) ? -(double)x : (double)x;
  if (a > 200.0) return f32_inf();
  const double e = exp_d(a);
  return to_f32(0.5 * (e + 1.0 / e));
}

TM_HD float asinhf(float x) {
  if (isnan_(x) || isinf_(x) || x == 0.0f) return x;
  const double a = sign_(x) ? -(double)x : (double)x;
  double r;
  if (a < kTiny) {
    const double a2 = a * a;
    r = a + a * (a2 * (-1.0 / 6.0 + a2 * (3.0 / 40.0 + a2 * (-5.0 / 112.0))));
  } else {
    r = log_pos(a + sqrt_d(a * a + 1.0));
  }
  return with_sign(r, sign_(x));
}

TM_HD float acoshf(float x) {
  if (isnan_(x) || x < 1.0f) return f32_nan();
  if (x == f32_inf()) return x;
  if (x == 1.0f) return 0.0f;
  const double d = (double)x;
  return to_f32(log_pos(d + sqrt_d((d - 1.0) * (d + 1.0))));
}

TM_HD float atanhf(float x) {
  if (isnan_(x) || x > 1.0f || x < -1.0f) return f32_nan();
  if (x == 1.0f || x == -1.0f) return x == 1.0f ? f32_inf() : -f32_inf();
  if (x == 0.0f) return x;
  const double a = sign_(x) ? -(double)x : (double)x;
  double r;
  if (a < kTiny) {
    const double a2 = a * a;
    r = a + a * (a2 * (1.0 / 3.0 + a2 * (1.0 / 5.0 + a2 * (1.0 / 7.0))));
  } else {
    r = 0.5 * log_pos((1.0 + a) / (1.0 - a));
  }
  return with_sign(r, sign_(x));
}

TM_HD float exp2f(float x) {
  if (isnan_(x)) return x;
  if (x >= 128.0f) return f32_inf();
  if (x < -150.0f) return 0.0f;
  return to_f32(exp_d((double)x * kLn2));
}

TM_HD float log2f(float x) {
  if (isnan_(x) || x < 0.0f) return f32_nan();
  if (x == 0.0f) return -f32_inf();
  if (x == f32_inf()) return x;
  return to_f32(log_pos((double)x) / kLn2);
}

TM_HD float cbrtf(float x) {
  if (isnan_(x) || isinf_(x) || x == 0.0f) return x;
  const double a = sign_(x) ? -(double)x : (double)x;
  double r = exp_d(log_pos(a) / 3.0);
  r = r - (r * r * r - a) / (3.0 * r * r);
  return with_sign(r, sign_(x));
}

// erf x for 0 <= x < 2: (2 / sqrt pi) sum_n (-1)^n x^(2n+1) / (n! (2n+1)), n <= 45
TM_HD double erf_series(double x) {
  const double x2 = x * x;
  double term = x, sum = x;
  for (int n = 1; n <= 45; ++n) {
    term = term * (-x2) / (double)n;
    sum = sum + term / (double)(2 * n + 1);
  }
  return kTwoOverSqrtPi * sum;
}
// erfc x for 2 <= x <= 14: Laplace's continued fraction, evaluated from depth 60 up
TM_HD double erfc_cf(double x) {
  double f = 0.0;
  for (int k = 60; k >= 1; --k) f = ((double)k * 0.5) / (x + f);
  return exp_d(-x * x) / kSqrtPi / (x + f);
}
TM_HD double erfc_pos(double x) {   // x >= 0
  if (x < 2.0) return 1.0 - erf_series(x);
  if (x > 14.0) return 0.0;
  return erfc_cf(x);
}

TM_HD float erff(float x) {
  if (isnan_(x) || x == 0.0f) return x;
  const double a = sign_(x) ? -(double)x : (double)x;
  const double r = a < 2.0 ? erf_series(a) : 1.0 - erfc_pos(a);
  return with_sign(r, sign_(x));
}

TM_HD float erfcf(float x) {
  if (isnan_(x)) return x;
  const double d = (double)x;
  if (d >= 0.0) return to_f32(erfc_pos(d));
  const double a = -d;
  return to_f32(a < 2.0 ? 1.0 + erf_series(a) : 2.0 - erfc_pos(a));
}

// the inverse of erf on (-1, 1); +-1: +-inf; beyond: NaN
TM_HD float erfinvf(float y) {
  if (isnan_(y) || y > 1.0f || y < -1.0f) return f32_nan();
  if (y == 1.0f || y == -1.0f) return y == 1.0f ? f32_inf() : -f32_inf();
  if (y == 0.0f) return y;
  const double a = sign_(y) ? -(double)y : (double)y;
  const double q = 1.0 - a;   // exact: y is an f32
  double x;
  if (a <= 0.9) {
    const double a2 = a * a;
    x = 0.886226925452758 * a * (1.0 + a2 * (0.2617993877991494 + a2 * (0.14393173084921979 + a2 * 0.09766361950392055)));
  } else {
    x = sqrt_d(-log_pos(q * kSqrtPi));
    for (int i = 0; i < 2; ++i) x = sqrt_d(-log_pos(q * x * kSqrtPi));
  }
  for (int i = 0; i < 5; ++i) {
    const double d = a < 0.5 ? a - erf_series(x) : erfc_pos(x) - q;
    x = x + d * (kSqrtPi * 0.5) * exp_d(x * x);
  }
  return with_sign(x, sign_(y));
}

// nextafter(x, y) as C's nextafterf: the f32 next to x in the direction of y (an integer step of its bits; from +-0
// the smallest subnormal with y's sign), NaN if either is NaN, y if x == y
TM_HD float nextafterf(float x, float y) {
  if (isnan_(x) || isnan_(y)) return f32_nan();
  if (x == y) return y;
  if (x == 0.0f) return u2f((f2u(y) & 0x80000000u) | 1u);
  const uint32_t b = f2u(x);
  return u2f(((x < y) == (x > 0.0f)) ? b + 1u : b - 1u);
}

// ln|Gamma(x)| in double, the f32 result rounded once.  Regions (every branch in double, IEEE operations only):
//   [1.5, 2.5)   lgamma(2 + t) = (1 - euler_gamma) t + sum_{k=2..31} (-1)^k (zeta(k) - 1) t^k / k, |t| <= 1/2
//                (the Taylor series about 2; its terms fall as 4^-k, truncation below 2e-18 of the first)
//   [0.5, 1.5)   lgamma(1 + t) = lgamma(2 + t) - log1p(t)
//   [2.5, 10)    lgamma(x) = lgamma(x - n) + log((x - 1) ... (x - n)), x - n in [1.5, 2.5)
//   [10, inf)    Stirling: (x - 1/2) log x - x + log(2 pi) / 2 + sum_{k=1..8} B_2k / (2k (2k - 1) x^(2k - 1))
//                (the next term is below 2e-18 at x = 10)
//   (-inf, 0.5)  reflection: log(pi / |sin(pi x)|) - lgamma(1 - x); +inf at 0 and the negative integers
TM_HD double lgamma_series2(double t) {   // lgamma(2 + t), |t| <= 1/2
  double p = -1.5021384080754142e-11;
  p = p * t + 3.104424774732227e-11;
  p = p * t + -6.422964563838102e-11;
  p = p * t + 1.3304764374244491e-10;
  p = p * t + -2.7595228851242334e-10;
  p = p * t + 5.731367241678861e-10;
  p = p * t + -1.1921401405860912e-09;
  p = p * t + 2.4836745438024785e-09;
  p = p * t + -5.183475041970047e-09;
  p = p * t + 1.0838659214896953e-08;
  p = p * t + -2.2711094608943164e-08;
  p = p * t + 4.76981016936398e-08;
  p = p * t + -1.0043224823968102e-07;
  p = p * t + 2.1207184805554667e-07;
  p = p * t + -4.492469198764565e-07;
  p = p * t + 9.551412130407415e-07;
  p = p * t + -2.039215753801366e-06;
  p = p * t + 4.3748667899074865e-06;
  p = p * t + -9.439488275268398e-06;
  p = p * t + 2.0507212775670688e-05;
  p = p * t + -4.4926236738133156e-05;
  p = p * t + 9.945751278180857e-05;
  p = p * t + -0.00022315475845357936;
  p = p * t + 0.0005096695247430426;
  p = p * t + -0.0011927539117032612;
  p = p * t + 0.002890510330741523;
  p = p * t + -0.007385551028673988;
  p = p * t + 0.020580808427784553;
  p = p * t + -0.0673523010531981;
  p = p * t + 0.3224670334241133;
  return t * (0.42278433509846713939 + t * p);   // (1 - euler_gamma)
}

TM_HD double log1p_d(double t) {   // log(1 + t) for t > -1, t from an f32 difference (Goldberg's correction)
  const double u = 1.0 + t;
  if (u == 1.0) return t;
  return log_pos(u) * (t / (u - 1.0));
}

TM_HD double lgamma_pos(double x) {   // x >= 0.5
  if (x < 1.5) return lgamma_series2(x - 1.0) - log1p_d(x - 1.0);
  if (x < 2.5) return lgamma_series2(x - 2.0);
  if (x < 10.0) {
    double p = 1.0, y = x;
    while (y >= 2.5) {
      y = y - 1.0;
      p = p * y;
    }
    return lgamma_series2(y - 2.0) + log_pos(p);
  }
  const double r = 1.0 / x, r2 = r * r;
  double s = -3617.0 / 122400.0;
  s = s * r2 + 1.0 / 156.0;
  s = s * r2 - 691.0 / 360360.0;
  s = s * r2 + 1.0 / 1188.0;
  s = s * r2 - 1.0 / 1680.0;
  s = s * r2 + 1.0 / 1260.0;
  s = s * r2 - 1.0 / 360.0;
  s = s * r2 + 1.0 / 12.0;
  return ((x - 0.5) * log_pos(x) - x) + (0.91893853320467274178 + s * r);
}

TM_HD double sinpi_abs(double r) {   // |sin(pi r)| for |r| <= 1
  double a = r < 0.0 ? -r : r;
  if (a > 0.5) a = 1.0 - a;
  if (a <= 0.25) return sin_core(3.14159265358979311600 * a);
  return cos_core(3.14159265358979311600 * (0.5 - a));
}

TM_HD float lgammaf(float xf) {
  if (isnan_(xf)) return xf;
  if (isinf_(xf)) return f32_inf();
  const double x = (double)xf;
  if (x >= 0.5) return to_f32(lgamma_pos(x));
  // x < 1/2: an integer (every f32 of magnitude 2^23 or more is one) is a pole
  const double h = x * 0.5;
  const double n2 = (double)(long long)(h < 0.0 ? h - 0.5 : h + 0.5);   // nearest integer to x / 2
  const double r = x - 2.0 * n2;                                       // exact: x - 2 n2 in [-1, 1]
  if (r == 0.0 || r == 1.0 || r == -1.0 || !(x > -8388608.0)) return f32_inf();
  return to_f32(log_pos(3.14159265358979311600 / sinpi_abs(r)) - lgamma_pos(1.0 - x));
}

// the shared dispatch of tm_math_eval and the oracle's or_math: fn as tallymap_b200.lower MATH_IDS
TM_HD float eval(int fn, float x, float y) {
  switch (fn) {
    case 0: return logf(x);
    case 1: return expf(x);
    case 2: return sinf(x);
    case 3: return cosf(x);
    case 4: return powf(x, y);
    case 5: return atanf(x);
    case 6: return atan2f(x, y);
    case 7: return asinf(x);
    case 8: return acosf(x);
    case 9: return tanf(x);
    case 10: return sinhf(x);
    case 11: return coshf(x);
    case 12: return asinhf(x);
    case 13: return acoshf(x);
    case 14: return atanhf(x);
    case 15: return exp2f(x);
    case 16: return log2f(x);
    case 17: return cbrtf(x);
    case 18: return erff(x);
    case 19: return erfcf(x);
    case 21: return nextafterf(x, y);
    case 22: return lgammaf(x);
    default: return erfinvf(x);
  }
}
constexpr int kMathFns = 23;

}  // namespace tmm
