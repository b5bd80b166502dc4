// GELU of two fp32 values through the fitted erfc form (see elementwise.cu for the fit and its
// accuracy): Phi(x) = 1 - h (x >= 0) or h (x < 0), h = erfc(|x| / sqrt(2)) / 2 = 2^-q(t).
// Shared by the standalone GELU kernel and the fused GEMM epilogue.
#pragma once

#include <cuda_runtime.h>

namespace fa {

// Coefficients of q(t) ~ -log2(erfc(t) / 2), lowest order first (fitted: numpy, Lawson-reweighted
// least squares on [0, 4] with weight sqrt(erfc)). Internal linkage: one copy per translation unit.
static __device__ __constant__ float kGeluQ[10] = {9.999999404e-01f, 1.627912402e+00f, 9.183757305e-01f, 1.486348212e-01f,
                                 -2.850020491e-02f, 9.230164578e-04f, 1.523754443e-03f, -5.291793495e-04f,
                                 8.135833923e-05f, -5.036062703e-06f};
constexpr float kGeluT = 4.0f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float2 splat(float v) { return make_float2(v, v); }

// GELU of two elements (FA_GELU_POLY).
__device__ __forceinline__ float2 gelu2_poly(float2 x) {
  constexpr float kAlpha = 0.70710678118654752440f;
  float2 t = __fmul2_rn(make_float2(fabsf(x.x), fabsf(x.y)), splat(kAlpha));
  const bool in0 = t.x < kGeluT, in1 = t.y < kGeluT;
  t.x = fminf(t.x, kGeluT);
  t.y = fminf(t.y, kGeluT);
  float2 q = splat(kGeluQ[9]);
#pragma unroll
  for (int k = 8; k >= 0; --k) q = __ffma2_rn(q, t, splat(kGeluQ[k]));
  const float2 h = make_float2(in0 ? ex2_approx(-q.x) : 0.f, in1 ? ex2_approx(-q.y) : 0.f);
  const float2 m = __fmul2_rn(x, h);                                   // x * Phi(x), x < 0
  const float2 r = __fmul2_rn(x, __ffma2_rn(h, splat(-1.f), splat(1.f)));  // x * (1 - h), x >= 0
  return make_float2(x.x < 0.f ? m.x : r.x, x.y < 0.f ? m.y : r.y);
}

// GELU of two elements whose result is rounded to bf16 (the GEMM epilogues). Same form with a
// degree-7 q (numpy, Lawson-reweighted least squares of q itself on [0, 4]; relative error of h
// within 7.2e-6 when evaluated in fp32, against 4.1e-6 for the degree-9 q above, both dominated
// by the fp32 Horner rounding) and no cut-off: this q keeps rising past t = 4 (within 0.02 of the
// exact q on [4, 6], then overflowing to +inf, so h goes to 0), which leaves the tiny negative
// tail (x < -5.66) at its value instead of 0. On 2 M normal fp32 sums (sigma 2) the bf16 results
// differ from the rounded exact GELU in 621 cases (one unit each), against 4928 for gelu2_poly.
static __device__ __constant__ float kGeluQ7[8] = {9.999953508e-01f, 1.628112555e+00f, 9.169421196e-01f,
                                                   1.525954902e-01f, -3.400735185e-02f, 5.252912641e-03f,
                                                   -4.904009402e-04f, 2.055818732e-05f};

__device__ __forceinline__ float2 gelu2_bf16out(float2 x) {
  constexpr float kAlpha = 0.70710678118654752440f;
  const float2 t = __fmul2_rn(make_float2(fabsf(x.x), fabsf(x.y)), splat(kAlpha));
  float2 q = splat(kGeluQ7[7]);
#pragma unroll
  for (int k = 6; k >= 0; --k) q = __ffma2_rn(q, t, splat(kGeluQ7[k]));
  const float2 h = make_float2(ex2_approx(-q.x), ex2_approx(-q.y));
  const float2 r = __ffma2_rn(h, splat(-1.f), splat(1.f));  // Phi(x) = 1 - h, x >= 0
  return __fmul2_rn(x, make_float2(x.x < 0.f ? h.x : r.x, x.y < 0.f ? h.y : r.y));
}

}  // namespace fa
