// Device arithmetic with explicit IEEE rounding. Every operation that the
// split, gradient and leaf semantics depend on is spelled with an _rn
// intrinsic, so the compiler can neither contract nor reassociate it.
#pragma once
#include <cuda_runtime.h>
#include <math_constants.h>

#include <cstdint>

namespace xgbb {

// exp(x) for binary32 x in binary64: Cody-Waite reduction x = k*ln2 + r with
// ln2 split into a 32-bit head (k*head exact) and a binary64 tail, the
// degree-11 Taylor polynomial of e^r by Horner's rule, one final rounding to
// binary32. The host trainer's checker evaluates the same sequence of IEEE
// operations, so both give identical bits.
__device__ __forceinline__ float det_expf(float x) {
  if (x != x) return x;
  if (x > 89.0f) return CUDART_INF_F;
  if (x < -104.0f) return 0.0f;
  const double xd = (double)x;
  const double k = rint(__dmul_rn(xd, 0x1.71547652b82fep+0));
  double r = __dsub_rn(xd, __dmul_rn(k, 0x1.62e42feep-1));
  r = __dsub_rn(r, __dmul_rn(k, 0x1.a39ef35793c76p-33));
  double p = 0x1.ae64567f544e4p-26;
  p = __dadd_rn(__dmul_rn(p, r), 0x1.27e4fb7789f5cp-22);
  p = __dadd_rn(__dmul_rn(p, r), 0x1.71de3a556c734p-19);
  p = __dadd_rn(__dmul_rn(p, r), 0x1.a01a01a01a01ap-16);
  p = __dadd_rn(__dmul_rn(p, r), 0x1.a01a01a01a01ap-13);
  p = __dadd_rn(__dmul_rn(p, r), 0x1.6c16c16c16c17p-10);
  p = __dadd_rn(__dmul_rn(p, r), 0x1.1111111111111p-7);
  p = __dadd_rn(__dmul_rn(p, r), 0x1.5555555555555p-5);
  p = __dadd_rn(__dmul_rn(p, r), 0x1.5555555555555p-3);
  p = __dadd_rn(__dmul_rn(p, r), 0.5);
  p = __dadd_rn(__dmul_rn(p, r), 1.0);
  p = __dadd_rn(__dmul_rn(p, r), 1.0);
  return __double2float_rn(scalbn(p, (int)k));
}

// An exact int64 sum in units of 2^-s (s = log2 of the power-of-two scale)
// as binary64: one rounding of the integer, then an exact scaling.
__device__ __forceinline__ double stat_value(long long v, double inv_scale) {
  return v == 0 ? 0.0 : __dmul_rn(__ll2double_rn(v), inv_scale);
}

struct SplitMath {
  double lambda, alpha, alpha2, min_child;
  float max_delta;
};

// Leaf weight RN32(RN64(-T(G)/(H+lambda))) with T the L1 soft threshold,
// clamped to +-max_delta_step; 0 when H <= 0.
__device__ __forceinline__ float leaf_weight(double G, double H, const SplitMath& m) {
  if (!(H > 0.0)) return 0.0f;
  const double t = fabs(G) <= m.alpha ? 0.0 : (G < 0.0 ? __dadd_rn(G, m.alpha) : __dsub_rn(G, m.alpha));
  const double den = __dadd_rn(H, m.lambda);
  float w = __double2float_rn(__ddiv_rn(-t, den));
  if (m.max_delta != 0.0f && fabsf(w) > m.max_delta) w = copysignf(m.max_delta, w);
  return w;
}

// Node gain RN32(-(fma(2*alpha, |w|, fma(2G, w, (H+lambda)*RN32(w*w))))).
__device__ __forceinline__ float node_gain(double G, double H, float w, const SplitMath& m) {
  if (!(H > 0.0)) return 0.0f;
  const double wd = (double)w;
  const double square = (double)__double2float_rn(__dmul_rn(wd, wd));
  const double quadratic = __dmul_rn(__dadd_rn(H, m.lambda), square);
  double sum = __fma_rn(__dadd_rn(G, G), wd, quadratic);
  sum = __fma_rn(m.alpha2, fabs(wd), sum);
  return __double2float_rn(-sum);
}

__device__ __forceinline__ bool valid_hessian(double H, const SplitMath& m) {
  return H > 0.0 && H >= m.min_child;
}

}  // namespace xgbb
