/* Deterministic transcendental functions for the oracle.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.c). The CUDA product carries its own
 * implementation of the same formulas; both must give identical bits, which
 * the GPU parity tests check.
 *
 * det_expf: exp(x) for binary32 x, computed in binary64 by Cody-Waite range
 * reduction (x = k*ln2 + r, |r| <= ln2/2, with ln2 split into a 32-bit head and
 * a binary64 tail so that k*head is exact) followed by the degree-11 Taylor
 * polynomial of e^r in Horner form, scaled by 2^k and rounded once to binary32.
 * Every step is an IEEE-754 binary64 operation in a fixed order with no
 * contraction, so any conforming host or device evaluates it to the same bits.
 * The truncation error is below 1e-14 relative, so the result is the correctly
 * rounded exp(x) except within ~1e-14 of a binary32 rounding boundary.
 */
#ifndef XGB_ORACLE_DET_MATH_H
#define XGB_ORACLE_DET_MATH_H
#include <math.h>

/* ln2 = 0.693147180559945309417232121458176568...; the head keeps its first
 * 32 fraction bits, the tail is the binary64 value nearest to the rest. */
#define DET_LN2_HEAD 0x1.62e42feep-1
#define DET_LN2_TAIL 0x1.a39ef35793c76p-33
#define DET_INV_LN2 0x1.71547652b82fep+0

static inline float det_expf(float x) {
  if (x != x) return x;
  if (x > 89.0f) return INFINITY;
  if (x < -104.0f) return 0.0f;
  double xd = (double)x;
  double k = nearbyint(xd * DET_INV_LN2);
  double r = xd - k * DET_LN2_HEAD;
  r = r - k * DET_LN2_TAIL;
  /* Coefficients 1/n!, each the binary64 value nearest to it. */
  double p = 0x1.ae64567f544e4p-26;     /* 1/11! */
  p = p * r + 0x1.27e4fb7789f5cp-22;    /* 1/10! */
  p = p * r + 0x1.71de3a556c734p-19;    /* 1/9!  */
  p = p * r + 0x1.a01a01a01a01ap-16;    /* 1/8!  */
  p = p * r + 0x1.a01a01a01a01ap-13;    /* 1/7!  */
  p = p * r + 0x1.6c16c16c16c17p-10;    /* 1/6!  */
  p = p * r + 0x1.1111111111111p-7;     /* 1/5!  */
  p = p * r + 0x1.5555555555555p-5;     /* 1/4!  */
  p = p * r + 0x1.5555555555555p-3;     /* 1/3!  */
  p = p * r + 0.5;                      /* 1/2!  */
  p = p * r + 1.0;
  p = p * r + 1.0;
  return (float)ldexp(p, (int)k);
}

#endif
