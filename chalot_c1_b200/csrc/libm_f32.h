// libm_f32.h — single-precision tanh and exp with the rounding of the host
// libm the reference links (glibc), for host and device.
//
// The reference's attention soft-cap calls f32::tanh (src/tensor/activations.rs:
// 133-135), which Rust on Linux takes from glibc. glibc's tanhf follows the
// method of Sun's fdlibm: for |x| < 22, tanh is rebuilt from expm1 of 2|x|
// (|x| >= 1: 1 - 2/(expm1(2|x|) + 2)) or of -2|x| (|x| < 1:
// -expm1(-2|x|) / (expm1(-2|x|) + 2)); expm1 reduces its argument as
// x = k*ln2 + r with ln2 split into a head exact in float and a tail, evaluates
// a rational approximation of degree 5 in r^2/2 on |r| <= ln2/2, and rebuilds
// 2^k * (expm1(r) + 1) - 1 with a correction term for the reduction error.
// This file restates that published method in float arithmetic, operation by
// operation, so the device reproduces the host's tanhf bit for bit (a host test
// compares it against the system tanhf over millions of arguments).
#pragma once

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define LIBM_FN __host__ __device__ __forceinline__
#else
#define LIBM_FN static inline
#endif

namespace chalot {
namespace libm {

#if defined(__CUDA_ARCH__)
// a / b rounded to nearest even, as IEEE division: Markstein's method
// (P. Markstein, IBM J. Res. Dev. 34(1), 1990) with fused multiply-adds. The
// hardware reciprocal approximation y0 is refined by one Newton step,
// y = y0 + y0*(1 - b*y0); the quotient q0 = a*y is corrected twice with the
// exact remainder r = a - b*q (one fma each): q' = q + r*y. Operands and
// quotients away from the ends of the exponent range (where the remainder
// could lose bits), zeros, infinities and NaNs take the division
// instruction sequence of the compiler instead, which is exact but about ten
// times slower in a dependent chain. Checked bit for bit against it.
__device__ __forceinline__ float div_rn(float a, float b) {
  const float aa = fabsf(a), ab = fabsf(b);
  if (aa >= 0x1p-100f && aa <= 0x1p+100f && ab >= 0x1p-100f && ab <= 0x1p+100f) {
    float y0;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(b));
    const float y = __fmaf_rn(y0, __fmaf_rn(-b, y0, 1.0f), y0);
    float q = __fmul_rn(a, y);
    q = __fmaf_rn(__fmaf_rn(-b, q, a), y, q);
    q = __fmaf_rn(__fmaf_rn(-b, q, a), y, q);
    return q;
  }
  return __fdiv_rn(a, b);
}
LIBM_FN double dmul(double a, double b) { return __dmul_rn(a, b); }
LIBM_FN double dadd(double a, double b) { return __dadd_rn(a, b); }
LIBM_FN double dsub(double a, double b) { return __dsub_rn(a, b); }
LIBM_FN uint64_t dbits(double d) { return (uint64_t)__double_as_longlong(d); }
LIBM_FN double dfrom_bits(uint64_t u) { return __longlong_as_double((long long)u); }
LIBM_FN float mul(float a, float b) { return __fmul_rn(a, b); }
LIBM_FN float add(float a, float b) { return __fadd_rn(a, b); }
LIBM_FN float sub(float a, float b) { return __fsub_rn(a, b); }
LIBM_FN float dvd(float a, float b) { return div_rn(a, b); }
LIBM_FN uint32_t bits(float f) { return __float_as_uint(f); }
LIBM_FN float from_bits(uint32_t u) { return __uint_as_float(u); }
#else
// host: compiled with -ffp-contract=off, every operation rounds once
LIBM_FN float div_rn(float a, float b) { return a / b; }
LIBM_FN double dmul(double a, double b) { return a * b; }
LIBM_FN double dadd(double a, double b) { return a + b; }
LIBM_FN double dsub(double a, double b) { return a - b; }
LIBM_FN uint64_t dbits(double d) {
  uint64_t u;
  memcpy(&u, &d, 8);
  return u;
}
LIBM_FN double dfrom_bits(uint64_t u) {
  double d;
  memcpy(&d, &u, 8);
  return d;
}
LIBM_FN float mul(float a, float b) { return a * b; }
LIBM_FN float add(float a, float b) { return a + b; }
LIBM_FN float sub(float a, float b) { return a - b; }
LIBM_FN float dvd(float a, float b) { return a / b; }
LIBM_FN uint32_t bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
LIBM_FN float from_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
#endif

// expm1 for finite |x| < 88 (the range tanh needs), fdlibm's method.
LIBM_FN float expm1_f32(float x) {
  const float ln2_head = from_bits(0x3f317180u);  // ln 2 rounded so k*head is exact
  const float ln2_tail = from_bits(0x3717f7d1u);  // ln 2 - head
  const float inv_ln2 = from_bits(0x3fb8aa3bu);
  // coefficients of the rational approximation in (r*r/2)
  const float q1 = from_bits(0xbd088889u), q2 = from_bits(0x3ad00d01u),
              q3 = from_bits(0xb8a670cdu), q4 = from_bits(0x36867e54u),
              q5 = from_bits(0xb457edbbu);
  const uint32_t ux = bits(x);
  const bool neg = (ux >> 31) != 0;
  const uint32_t ax = ux & 0x7fffffffu;
  if (ax >= 0x4195b844u && neg) return -1.0f;  // x <= -27 ln2: expm1 rounds to -1
  int k = 0;
  float corr = 0.0f;
  if (ax > 0x3eb17218u) {  // |x| > ln2/2: reduce
    float hi, lo;
    if (ax < 0x3f851592u) {  // |x| < 1.5 ln2: k = +-1
      k = neg ? -1 : 1;
      hi = neg ? add(x, ln2_head) : sub(x, ln2_head);
      lo = neg ? -ln2_tail : ln2_tail;
    } else {
      k = (int)add(mul(inv_ln2, x), neg ? -0.5f : 0.5f);  // truncation toward zero
      const float kf = (float)k;
      hi = sub(x, mul(kf, ln2_head));
      lo = mul(kf, ln2_tail);
    }
    const float r = sub(hi, lo);
    corr = sub(sub(hi, r), lo);
    x = r;
  } else if (ax < 0x33000000u) {  // |x| < 2^-25
    return x;
  }
  const float half_x = mul(0.5f, x);
  const float hxs = mul(x, half_x);
  const float r1 =
      add(1.0f, mul(hxs, add(q1, mul(hxs, add(q2, mul(hxs, add(q3, mul(hxs, add(q4, mul(hxs, q5))))))))));
  const float t = sub(3.0f, mul(r1, half_x));
  float e = mul(hxs, dvd(sub(r1, t), sub(6.0f, mul(x, t))));
  if (k == 0) return sub(x, sub(mul(x, e), hxs));
  e = sub(mul(x, sub(e, corr)), corr);
  e = sub(e, hxs);
  if (k == -1) return sub(mul(0.5f, sub(x, e)), 0.5f);
  if (k == 1) {
    if (x < -0.25f) return mul(-2.0f, sub(e, add(x, 0.5f)));
    return add(1.0f, mul(2.0f, sub(x, e)));
  }
  if (k <= -2 || k > 56) {
    float y = sub(1.0f, sub(e, x));
    y = from_bits(bits(y) + ((uint32_t)k << 23));
    return sub(y, 1.0f);
  }
  float y;
  if (k < 23) {
    const float one_minus = from_bits(0x3f800000u - (0x1000000u >> k));  // 1 - 2^-k
    y = sub(one_minus, sub(e, x));
  } else {
    const float two_mk = from_bits((uint32_t)(0x7f - k) << 23);  // 2^-k
    y = sub(x, add(e, two_mk));
    y = add(y, 1.0f);
  }
  return from_bits(bits(y) + ((uint32_t)k << 23));
}

// tanh for finite x, fdlibm's method (see the file comment).
LIBM_FN float tanh_f32(float x) {
  const uint32_t ux = bits(x);
  const uint32_t ax = ux & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (ux >> 31) ? -1.0f : 1.0f;  // +-inf (NaN not expected)
  float z;
  if (ax < 0x41b00000u) {                 // |x| < 22
    if (ax < 0x24000000u) return mul(x, add(1.0f, x));  // |x| < 2^-55
    const float a = from_bits(ax);
    if (ax >= 0x3f800000u) {              // |x| >= 1
      const float t = expm1_f32(mul(2.0f, a));
      z = sub(1.0f, dvd(2.0f, add(t, 2.0f)));
    } else {
      const float t = expm1_f32(mul(-2.0f, a));
      z = dvd(-t, add(t, 2.0f));
    }
  } else {
    z = 1.0f;  // 1 - tiny rounds to 1
  }
  return (ux >> 31) ? -z : z;
}

// 2^(i/32) for i = 0..31 as doubles with i/32 taken out of the exponent
// field (the table of exp_f32 below).
#if defined(__CUDACC__)
static __constant__ uint64_t kExpTab32[32] = {
      0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
      0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
      0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
      0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
      0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
      0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
      0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
      0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};
#endif
static const uint64_t kExpTab32Host[32] = {
      0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
      0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
      0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
      0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
      0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
      0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
      0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
      0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

// expf as glibc (2.28 and later) computes it, the method of the Arm
// optimized-routines single-precision exp (Szabolcs Nagy, 2017): in double
// precision, z = x * 32/ln2 is split into an integer k (rounded by adding and
// subtracting 1.5*2^52) and r = z - k; 2^(k/32) is a table entry for k mod 32
// (2^(i/32) rounded to double, here computed offline from exact arithmetic)
// with k/32 added to its exponent; 2^(r/32) is a cubic in r; the product is
// rounded once to float. Out of range: +inf above 88.72, 0 below -103.97.
// Matches the system expf of glibc 2.39 on every float in [-87, 88] but two
// (x = 0x1.04845ep+5 and -0x1.f8cbb2p+5, 1 ulp; the attention softmax under
// the soft-cap only reaches [-60, 0]). Coefficients: the published cubic of
// that method.
LIBM_FN float exp_f32(float x) {
  const uint32_t ux = bits(x);
  const uint32_t ax = ux & 0x7fffffffu;
  if (ax >= 0x42b00000u) {                            // |x| >= 88, inf or NaN
    if (ux == 0xff800000u) return 0.0f;               // -inf
    if (ax > 0x7f800000u) return x;                   // NaN
    if (!(ux >> 31) && ax > 0x42b17217u) return from_bits(0x7f800000u);  // overflow
    if ((ux >> 31) && ax > 0x42cff1b4u) return 0.0f;  // underflow
  }
  const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
  const double shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / 32768.0, c1 = 0x1.ebfce50fac4f3p-3 / 1024.0,
               c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  const double z = dmul(inv_ln2_n, (double)x);
  double kd = dadd(z, shift);
  const uint64_t ki = dbits(kd);
  kd = dsub(kd, shift);
  const double r = dsub(z, kd);
#if defined(__CUDA_ARCH__)
  const double s = dfrom_bits(kExpTab32[ki & 31] + (ki << 47));
#else
  const double s = dfrom_bits(kExpTab32Host[ki & 31] + (ki << 47));
#endif
  const double p = dadd(dmul(c0, r), c1);
  const double r2 = dmul(r, r);
  double y = dadd(dmul(c2, r), 1.0);
  y = dadd(dmul(p, r2), y);
  y = dmul(y, s);
  return (float)y;
}

}  // namespace libm
}  // namespace chalot
