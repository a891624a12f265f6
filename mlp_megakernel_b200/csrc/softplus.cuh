// softplus(z) = log(1 + e^z) with beta = 1, threshold = 20 -- the activation of
// the reference (F.softplus at kernel.py:169-170, written in the fused kernel
// as where(z > 20, z, log(exp(z) + 1)) at kernel.py:108).
//
// Evaluated as max(z, 0) + log1p(e^{-|z|}), which equals the reference form
// for every z (for z > 20 the log1p term is below 2.1e-9, under fp32's
// resolution of z).  One MUFU op (ex2) per element; log1p(t) on t in (0, 1] is
// t*q(t) with q a degree-4 polynomial on the FMA pipe.  The coefficients are
// this project's own minimax fit (Lawson's iteratively reweighted least
// squares on the RELATIVE error) of q(t) = log1p(t)/t on [0, 1]: max relative
// error 5.7e-5 in float32 Horner form, 1/8 of fp16's half-ulp, so the fp16
// value fed to the next GEMM is the correctly rounded softplus in about 97%
// of cases and one ulp away otherwise.  Degree 4 instead of 5 (8.5e-6, 99.5%)
// saves one packed FMA per pair of elements: 4% of the 3L128 forward, whose
// epilogue issue rate bounds it.  Relative (not absolute) error matters
// because h = log1p(e^-|z|) is tiny for very negative z.  Accuracy is checked
// against float64 log1p in tests/test_softplus_poly.py.
#pragma once
#include "ptx.cuh"

namespace mlpk {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kSpC0 = 0.9999432563781738f;
constexpr float kSpC1 = -0.49697771668434143f;
constexpr float kSpC2 = 0.30630072951316833f;
constexpr float kSpC3 = -0.15742707252502441f;
constexpr float kSpC4 = 0.041347306221723557f;

__device__ __forceinline__ float log1p_unit(float t) {  // t in [0, 1]
  float q = kSpC4;
  q = fmaf(q, t, kSpC3);
  q = fmaf(q, t, kSpC2);
  q = fmaf(q, t, kSpC1);
  q = fmaf(q, t, kSpC0);
  return q * t;
}

__device__ __forceinline__ float softplus_f32(float z) {
  const float e = ex2_approx(fabsf(z) * -kLog2e);  // e^{-|z|} in (0, 1]
  return fmaxf(z, 0.0f) + log1p_unit(e);
}

// Two softplus evaluations with packed f32x2 arithmetic (sm_100 FFMA2 /
// FMUL2: one instruction for both lanes); same formula and coefficients as
// softplus_f32, with the last Horner step fused with the relu term:
// h = q(e) * e + max(z, 0).
__device__ __forceinline__ float2 softplus_x2(float2 z) {
  const float2 s = __fmul2_rn(z, make_float2(kLog2e, kLog2e));
  const float2 e = make_float2(ex2_approx(-fabsf(s.x)), ex2_approx(-fabsf(s.y)));  // e^{-|z|}
  float2 q = __ffma2_rn(make_float2(kSpC4, kSpC4), e, make_float2(kSpC3, kSpC3));
  q = __ffma2_rn(q, e, make_float2(kSpC2, kSpC2));
  q = __ffma2_rn(q, e, make_float2(kSpC1, kSpC1));
  q = __ffma2_rn(q, e, make_float2(kSpC0, kSpC0));
  return __ffma2_rn(q, e, make_float2(fmaxf(z.x, 0.0f), fmaxf(z.y, 0.0f)));
}

// d softplus / dz expressed through the post-activation h = softplus(z):
// sigmoid(z) = 1 - e^{-h}  (mlp_fused.md:87-95).
__device__ __forceinline__ float dsoftplus_from_h(float h) {
  return 1.0f - ex2_approx(h * -kLog2e);
}

}  // namespace mlpk
