// Portable double-precision math shared bit-for-bit by host and device code.
//
// The GPU trainer computes objective derivatives in Float64 and narrows them
// to Float32, as the reference CPU trainer does (boosting.mojo:676-812 with
// histogram.mojo:462-480).  The logistic and softmax derivatives need exp().
// CUDA's exp() and glibc's exp() are each accurate to about one ulp but are
// not the same function, so a device gradient computed with one and a host
// gradient computed with the other could differ in the last bit.  Every
// integer histogram downstream of a gradient is bit-exact, so this file gives
// both sides ONE exp, written here from a published method and built without
// floating-point contraction on both sides (host: -ffp-contract=off; device:
// nvcc -fmad=false), so host and device produce identical bits.
//
// Method: Cody & Waite (1980) argument reduction, x = k*ln2 + r with ln2 split
// into a 32-bit-exact high part and a low correction, |r| <= ln2/2, followed by
// the degree-13 Taylor polynomial of e^r in Horner form (truncation error below
// 0.5e-17 relative on that interval), and an exact scaling by 2^k through the
// exponent field.  Accuracy is checked against libm in the tests (<= 2 ulp).
#pragma once
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define MT_HD __host__ __device__ __forceinline__
#else
#define MT_HD inline
#endif

MT_HD double mt_bits_to_double(uint64_t u) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)u);
#else
  double d;
  memcpy(&d, &u, sizeof d);
  return d;
#endif
}

MT_HD uint64_t mt_double_to_bits(double d) {
#if defined(__CUDA_ARCH__)
  return (uint64_t)__double_as_longlong(d);
#else
  uint64_t u;
  memcpy(&u, &d, sizeof u);
  return u;
#endif
}

// e^x.  Returns +inf above 709.78, 0 below -745.2, NaN for NaN.
MT_HD double mt_exp(double x) {
  if (x != x) return x;
  if (x > 709.782712893384) return mt_bits_to_double(0x7FF0000000000000ull);
  if (x < -745.2) return 0.0;
  const double inv_ln2 = 1.4426950408889634;
  // ln2 = LN2_HI + LN2_LO, LN2_HI has 32 significant bits so k*LN2_HI is exact
  // for |k| < 2^20.
  const double LN2_HI = 6.93147180369123816490e-01;
  const double LN2_LO = 1.90821492927058770002e-10;
  double kd = x * inv_ln2;
  // round half away from zero to the nearest integer
  kd = kd >= 0.0 ? (double)(long long)(kd + 0.5) : (double)(long long)(kd - 0.5);
  long long k = (long long)kd;
  double hi = x - kd * LN2_HI;
  double r = hi - kd * LN2_LO;
  // Horner evaluation of sum_{i=0}^{13} r^i / i!
  double p = 1.0 / 6227020800.0;      // 1/13!
  p = p * r + 1.0 / 479001600.0;      // 1/12!
  p = p * r + 1.0 / 39916800.0;       // 1/11!
  p = p * r + 1.0 / 3628800.0;        // 1/10!
  p = p * r + 1.0 / 362880.0;         // 1/9!
  p = p * r + 1.0 / 40320.0;          // 1/8!
  p = p * r + 1.0 / 5040.0;           // 1/7!
  p = p * r + 1.0 / 720.0;            // 1/6!
  p = p * r + 1.0 / 120.0;            // 1/5!
  p = p * r + 1.0 / 24.0;             // 1/4!
  p = p * r + 1.0 / 6.0;              // 1/3!
  p = p * r + 0.5;                    // 1/2!
  p = p * r + 1.0;
  p = p * r + 1.0;
  // scale by 2^k in two steps so that subnormal and near-overflow results
  // are formed by exact power-of-two multiplications
  long long k1 = k / 2;
  long long k2 = k - k1;
  double s1 = mt_bits_to_double((uint64_t)(k1 + 1023) << 52);
  double s2 = mt_bits_to_double((uint64_t)(k2 + 1023) << 52);
  return (p * s1) * s2;
}

// The reference's numerically stable logistic (boosting.mojo:261-266).
MT_HD double mt_sigmoid(double x) {
  if (x >= 0.0) {
    double e = mt_exp(-x);
    return 1.0 / (1.0 + e);
  }
  double e = mt_exp(x);
  return e / (1.0 + e);
}

// splitmix64 finalizer and the 53-bit uniform of rng.mojo:35-46.
MT_HD uint64_t mt_splitmix64(uint64_t state) {
  uint64_t z = state + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

MT_HD double mt_uniform(uint64_t counter) {
  return (double)(mt_splitmix64(counter) >> 11) * (1.0 / 9007199254740992.0);
}

#define MT_GOLDEN 0x9E3779B97F4A7C15ull

// Stochastic-rounding stream of quantized_gradient.mojo:475-492.
MT_HD uint64_t mt_quant_stream(long long seed, long long round_index, long long class_index, int plane) {
  const uint64_t mask = 0x7FFFFFFFFFFFFFFFull;
  uint64_t h = mt_splitmix64((uint64_t)seed & mask);
  h = mt_splitmix64(h ^ ((uint64_t)round_index & mask));
  h = mt_splitmix64(h ^ ((uint64_t)(class_index + 1) & mask));
  return mt_splitmix64(h ^ ((uint64_t)plane * MT_GOLDEN));
}

// quantize_scalar of quantized_gradient.mojo:1479-1545 in stochastic mode:
// clamp value*units to [-lim, lim], then |q| = floor(|y| + u), sign kept.
MT_HD long long mt_quantize_stochastic(double value, double units, double lim, uint64_t counter) {
  double y = value * units;
  if (y > lim) y = lim;
  else if (y < -lim) y = -lim;
  double u = mt_uniform(counter);
#if defined(__CUDA_ARCH__)
  if (y >= 0.0) return (long long)floor(y + u);
  return -(long long)floor(-y + u);
#else
  if (y >= 0.0) return (long long)__builtin_floor(y + u);
  return -(long long)__builtin_floor(-y + u);
#endif
}

// Largest power of two <= x for positive normal x (quantized_gradient.mojo:856-887).
MT_HD double mt_pow2_floor(double x) {
  uint64_t bits = mt_double_to_bits(x);
  uint64_t biased = (bits >> 52) & 0x7FF;
  return mt_bits_to_double(biased << 52);
}

// The fixed-point scale rule of quantized_gradient.mojo:908: 2^k <= fl(2^30/T),
// T floored at 1e-12, returned as the Float32 the histogram kernels multiply by.
MT_HD float mt_fixed_point_scale(double total) {
  double t = total < 1e-12 ? 1e-12 : total;
  return (float)mt_pow2_floor(1073741824.0 / t);
}

// The same rule with the bound 2^52 (Int64 cells; every sum of quantized
// values stays below 2^53, so its Float64 dequantization is exact).
MT_HD float mt_fixed_point_scale52(double total) {
  double t = total < 1e-12 ? 1e-12 : total;
  return (float)mt_pow2_floor(4503599627370496.0 / t);
}
