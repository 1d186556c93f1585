/*
 * snai_exp.h - the double-precision exponential of the sampling contract.
 *
 * The PHP samplers (src/snai_inference.php:181, src/tensor_ffi_adapter.php:184)
 * call PHP's exp(), i.e. the platform libm exp() on a double.  A sampled token
 * id is a function of every exp() value in a row (they are summed in vocab
 * order), so for ids to be bit-identical between the GPU kernel and a CPU
 * check, both sides must evaluate the *same* function bit for bit.  libm's exp
 * cannot run on the GPU and CUDA's exp cannot run on the CPU, so the contract
 * fixes this one instead and both sides compile it from this header.
 *
 * Method: Cody & Waite argument reduction (W. J. Cody, W. Waite, "Software
 * Manual for the Elementary Functions", 1980):  x = k*ln2 + r, |r| <= ln2/2,
 * with ln2 split into a head (the double nearest ln2) and a tail, both
 * products formed inside fused multiply-adds.  e^r is the Taylor series of
 * the exponential truncated after r^13/13! (truncation error < 5e-18 for
 * |r| <= 0.3466), evaluated in Horner form with fused multiply-adds; the
 * coefficients are the doubles nearest 1/n!.  The result is scaled by 2^k
 * with exact power-of-two multiplies (two of them when 2^k is not a normal
 * double, so a subnormal result is rounded exactly once).
 *
 * Every step is an IEEE-754 operation with round-to-nearest-even (fma, *,
 * rint) and no step is left to the compiler to contract, so the CPU build
 * (compiled with -ffp-contract=off, fma() from libm) and the GPU build
 * (__fma_rn/__dmul_rn) produce identical bits.  The accuracy against libm
 * exp() is checked by the test-suite (max error 1 ulp over the sampling
 * domain).
 */
#ifndef SNAI_EXP_H
#define SNAI_EXP_H

#include <stdint.h>
#include <string.h>
#include <math.h>

#if defined(__CUDACC__)
#define SNAI_HD __host__ __device__ __forceinline__
#else
#define SNAI_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define SNAI_FMA(a, b, c) __fma_rn((a), (b), (c))
#define SNAI_DMUL(a, b) __dmul_rn((a), (b))
#define SNAI_RINT(a) rint(a)
#else
#define SNAI_FMA(a, b, c) fma((a), (b), (c))
#define SNAI_DMUL(a, b) ((a) * (b))
#define SNAI_RINT(a) rint(a)
#endif

/* 2^e for e in [-1022, 1023], built from its exponent field. */
SNAI_HD double snai_pow2i(int e) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)(e + 1023) << 52);
#else
  uint64_t bits = (uint64_t)(int64_t)(e + 1023) << 52;
  double r;
  memcpy(&r, &bits, sizeof r);
  return r;
#endif
}

SNAI_HD double snai_exp(double x) {
  /* Hex literals are exact: the doubles nearest the named constants. */
  const double kLog2e = 0x1.71547652b82fep+0;  /* 1/ln 2 */
  const double kLn2Hi = 0x1.62e42fefa39efp-1;  /* ln 2 rounded to double */
  const double kLn2Lo = 0x1.abc9e3b39803fp-56; /* ln 2 - kLn2Hi */
  if (x != x) return x;                                 /* NaN */
  if (x > 0x1.62e42fefa39efp+9) return (double)INFINITY; /* > ln(DBL_MAX) */
  if (x < -0x1.74910d52d3052p+9) return 0.0;            /* < ln(2^-1075) */
  double kd = SNAI_RINT(SNAI_DMUL(x, kLog2e));
  int k = (int)kd;
  double r = SNAI_FMA(-kd, kLn2Hi, x);
  r = SNAI_FMA(-kd, kLn2Lo, r);
  /* Taylor coefficients 1/n!, n = 13 .. 2 */
  double p = 0x1.6124613a86d09p-33;
  p = SNAI_FMA(p, r, 0x1.1eed8eff8d898p-29);
  p = SNAI_FMA(p, r, 0x1.ae64567f544e4p-26);
  p = SNAI_FMA(p, r, 0x1.27e4fb7789f5cp-22);
  p = SNAI_FMA(p, r, 0x1.71de3a556c734p-19);
  p = SNAI_FMA(p, r, 0x1.a01a01a01a01ap-16);
  p = SNAI_FMA(p, r, 0x1.a01a01a01a01ap-13);
  p = SNAI_FMA(p, r, 0x1.6c16c16c16c17p-10);
  p = SNAI_FMA(p, r, 0x1.1111111111111p-7);
  p = SNAI_FMA(p, r, 0x1.5555555555555p-5);
  p = SNAI_FMA(p, r, 0x1.5555555555555p-3);
  p = SNAI_FMA(p, r, 0x1.0000000000000p-1);
  p = SNAI_FMA(p, r, 1.0);
  p = SNAI_FMA(p, r, 1.0);
  if (k > 1023) return SNAI_DMUL(SNAI_DMUL(p, snai_pow2i(k - 1)), 2.0);
  if (k < -1021) return SNAI_DMUL(SNAI_DMUL(p, snai_pow2i(k + 64)), 0x1p-64);
  return SNAI_DMUL(p, snai_pow2i(k));
}

#endif /* SNAI_EXP_H */
