// Deterministic scalar math shared bit-for-bit by the sm_100a sampler and the
// host-side checker.
//
// The sampler's random race (sampling.rs:191-213 of the reference) needs
// `f32::exp` and `f64::ln_1p`, and parity is defined as bit-exact token ids given
// identical logits. Platform libm/CUDA implementations differ in the last bit, so
// both sides compile these functions from this one header instead:
//
//   det_expf  : Cody-Waite reduction x = k*ln2 + r (ln2 split in a high part with
//               trailing zero bits and a low correction), Taylor series of e^r to
//               degree 13 evaluated by Horner's rule in double with explicit fma,
//               exact 2^k scaling through the exponent field, then ONE rounding
//               to float. Double evaluation leaves ~1e-16 relative error, so the
//               float result is the correctly rounded e^x except for arguments
//               within ~1e-16 of a float rounding boundary.
//   det_log1p : y = 1 + x; log(y) = e*ln2 + 2*atanh(s), s = (m-1)/(m+1) with
//               y = m*2^e, m in [sqrt(1/2), sqrt(2)) (the classic atanh series,
//               |s| <= 0.1716, 12 odd terms); Kahan's correction -((y-1)-x)/y
//               restores the bits lost in forming 1 + x. Signed zero is returned
//               unchanged, as IEEE log1p does.
//   round_bf16: round-to-nearest-even to bfloat16 kept in a float, NaN quieted
//               with its sign kept (tensor.rs:645-652).
//   powi_f32  : binary exponentiation in float (the integer-power routine that
//               `f32::powi` lowers to for a run-time exponent).
//
// Every operation is a single IEEE-rounded add/mul/div/fma or an exact bit
// manipulation, so host (gcc, -ffp-contract=off) and device (nvcc, explicit
// __fma_rn/__dmul_rn) produce identical bits.
#pragma once
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define DET_HD __host__ __device__ __forceinline__
#else
#define DET_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define DET_FMA(a, b, c) __fma_rn((a), (b), (c))
#define DET_DMUL(a, b) __dmul_rn((a), (b))
#define DET_DADD(a, b) __dadd_rn((a), (b))
#define DET_DDIV(a, b) __ddiv_rn((a), (b))
#else
#include <math.h>
#define DET_FMA(a, b, c) fma((a), (b), (c))
#define DET_DMUL(a, b) ((a) * (b))
#define DET_DADD(a, b) ((a) + (b))
#define DET_DDIV(a, b) ((a) / (b))
#endif

DET_HD uint32_t det_f2u(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}
DET_HD float det_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}
DET_HD uint64_t det_d2u(double d) {
#if defined(__CUDA_ARCH__)
  return (uint64_t)__double_as_longlong(d);
#else
  uint64_t u;
  memcpy(&u, &d, 8);
  return u;
#endif
}
DET_HD double det_u2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)u);
#else
  double d;
  memcpy(&d, &u, 8);
  return d;
#endif
}
DET_HD float det_d2f(double d) {
#if defined(__CUDA_ARCH__)
  return __double2float_rn(d);
#else
  return (float)d;
#endif
}

/* bfloat16 round-to-nearest-even kept in an f32 (tensor.rs:645-652). */
DET_HD float round_bf16(float v) {
  uint32_t b = det_f2u(v);
  if ((b & 0x7fffffffu) > 0x7f800000u) return det_u2f((b & 0xffff0000u) | 0x00400000u);
  return det_u2f((b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u);
}

/* Order-preserving key of Rust's f32::total_cmp: -NaN < -inf < ... < -0 < +0 < ... < +inf < NaN. */
DET_HD uint32_t total_key(float v) {
  uint32_t b = det_f2u(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
DET_HD float total_key_to_float(uint32_t k) {
  return det_u2f((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

/* x^n by binary exponentiation in float; n may be negative. */
DET_HD float powi_f32(float a, int b) {
  const int recip = b < 0;
  float r = 1.0f;
  for (;;) {
    if (b & 1) r = r * a;
    b /= 2;
    if (b == 0) break;
    a = a * a;
  }
  return recip ? 1.0f / r : r;
}

/* e^x for float x, correctly rounded up to the double-evaluation error. */
DET_HD float det_expf(float xf) {
  if (xf != xf) return xf;
  if (xf > 100.0f) return det_u2f(0x7f800000u);
  if (xf < -200.0f) return 0.0f;
  const double x = (double)xf;
  const double LOG2E = 1.4426950408889634074;
  /* ln2 = LN2_HI + LN2_LO; LN2_HI has 32 trailing zero bits so k*LN2_HI is exact for |k| < 2^20. */
  const double LN2_HI = 6.93147180369123816490e-01;
  const double LN2_LO = 1.90821492927058770002e-10;
  double t = DET_DMUL(x, LOG2E);
  /* round half away from zero; k is small so the conversion is exact */
  double k = (double)(long long)(t >= 0.0 ? DET_DADD(t, 0.5) : DET_DADD(t, -0.5));
  double r = DET_FMA(-k, LN2_HI, x);
  r = DET_FMA(-k, LN2_LO, r);
  /* Taylor coefficients 1/n!, n = 13 .. 0 */
  double p = 1.6059043836821614599e-10;     /* 1/13! */
  p = DET_FMA(p, r, 2.0876756987868098979e-09); /* 1/12! */
  p = DET_FMA(p, r, 2.5052108385441718775e-08); /* 1/11! */
  p = DET_FMA(p, r, 2.7557319223985890653e-07); /* 1/10! */
  p = DET_FMA(p, r, 2.7557319223985890653e-06); /* 1/9!  */
  p = DET_FMA(p, r, 2.4801587301587301587e-05); /* 1/8!  */
  p = DET_FMA(p, r, 1.9841269841269841270e-04); /* 1/7!  */
  p = DET_FMA(p, r, 1.3888888888888888889e-03); /* 1/6!  */
  p = DET_FMA(p, r, 8.3333333333333333333e-03); /* 1/5!  */
  p = DET_FMA(p, r, 4.1666666666666666667e-02); /* 1/4!  */
  p = DET_FMA(p, r, 1.6666666666666666667e-01); /* 1/3!  */
  p = DET_FMA(p, r, 0.5);
  p = DET_FMA(p, r, 1.0);
  p = DET_FMA(p, r, 1.0);
  /* 2^k as a double (|k| <= 289 keeps it normal); the product is exact */
  int ki = (int)k;
  double scale = det_u2d((uint64_t)(ki + 1023) << 52);
  return det_d2f(DET_DMUL(p, scale));
}

/* natural log of a positive finite double */
DET_HD double det_log_pos(double y) {
  uint64_t bits = det_d2u(y);
  int e = (int)((bits >> 52) & 0x7ff);
  if (e == 0) { /* subnormal: scale by 2^64 */
    y = DET_DMUL(y, 18446744073709551616.0);
    bits = det_d2u(y);
    e = (int)((bits >> 52) & 0x7ff) - 64;
  }
  e -= 1023;
  double m = det_u2d((bits & 0x000fffffffffffffull) | 0x3ff0000000000000ull); /* [1,2) */
  if (m > 1.4142135623730950488) { m = DET_DMUL(m, 0.5); e += 1; }
  double f = DET_DADD(m, -1.0);                 /* exact (Sterbenz) */
  double s = DET_DDIV(f, DET_DADD(2.0, f));
  double s2 = DET_DMUL(s, s);
  /* 2*atanh(s) = 2*(s + s^3/3 + s^5/5 + ... + s^23/23) */
  double q = 1.0 / 23.0;
  q = DET_FMA(q, s2, 1.0 / 21.0);
  q = DET_FMA(q, s2, 1.0 / 19.0);
  q = DET_FMA(q, s2, 1.0 / 17.0);
  q = DET_FMA(q, s2, 1.0 / 15.0);
  q = DET_FMA(q, s2, 1.0 / 13.0);
  q = DET_FMA(q, s2, 1.0 / 11.0);
  q = DET_FMA(q, s2, 1.0 / 9.0);
  q = DET_FMA(q, s2, 1.0 / 7.0);
  q = DET_FMA(q, s2, 1.0 / 5.0);
  q = DET_FMA(q, s2, 1.0 / 3.0);
  /* log(m) = 2s + 2s*s2*q */
  double two_s = DET_DMUL(2.0, s);
  double logm = DET_FMA(DET_DMUL(two_s, s2), q, two_s);
  const double LN2_HI = 6.93147180369123816490e-01;
  const double LN2_LO = 1.90821492927058770002e-10;
  double de = (double)e;
  return DET_DADD(DET_FMA(de, LN2_HI, DET_FMA(de, LN2_LO, logm)), 0.0);
}

/* log(1 + x) in double. */
DET_HD double det_log1p(double x) {
  if (x == 0.0 || x != x) return x;
  if (x == -1.0) return -det_u2d(0x7ff0000000000000ull);
  if (x < -1.0) return det_u2d(0x7ff8000000000000ull);
  if (x == det_u2d(0x7ff0000000000000ull)) return x;
  double y = DET_DADD(1.0, x);
  double lg = det_log_pos(y);
  /* Kahan: correct for the rounding of 1 + x */
  double corr = DET_DDIV(DET_DADD(DET_DADD(y, -1.0), -x), y);
  return DET_DADD(lg, -corr);
}
