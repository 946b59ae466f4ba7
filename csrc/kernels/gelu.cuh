// GELU and its derivative for the fused epilogues and the standalone GELU kernels.
//
//   gelu(x)  = x * Phi(x),         Phi(x) = (1 + erf(x / sqrt 2)) / 2
//   gelu'(x) = Phi(x) + x * phi(x), phi(x) = exp(-x^2 / 2) / sqrt(2 pi)
//
// erf comes from the rational approximation of Abramowitz & Stegun, Handbook of
// Mathematical Functions (1964), formula 7.1.26 (after C. Hastings):
//   erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2),
//   t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7,
// extended to z < 0 by symmetry.  exp(-z^2) with z = |x| / sqrt 2 is exp(-x^2 / 2),
// the same factor phi needs, so gelu' costs one exponential and one reciprocal
// (both on the special-function unit) plus a handful of FMAs.  The GELU outputs
// are stored as bf16 (8 significant bits), far coarser than the 1.5e-7 error.
#pragma once

namespace mtorus {

struct GeluParts {
  float phi_cdf;  // Phi(x)
  float e;        // exp(-x^2 / 2)
};

__device__ __forceinline__ GeluParts gelu_parts(float x) {
  constexpr float p = 0.3275911f;
  constexpr float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f, a4 = -1.453152027f,
                  a5 = 1.061405429f;
  const float z = fabsf(x) * 0.70710678118654752f;
  const float t = __fdividef(1.f, fmaf(p, z, 1.f));
  const float e = __expf(-0.5f * x * x);
  const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, a5, a4), a3), a2), a1);
  const float half_erfc = 0.5f * poly * e;  // (1 - erf(z)) / 2
  return {x >= 0.f ? 1.f - half_erfc : half_erfc, e};
}

__device__ __forceinline__ float gelu_fwd(float x) { return x * gelu_parts(x).phi_cdf; }

__device__ __forceinline__ float gelu_grad(float x) {
  const GeluParts g = gelu_parts(x);
  return fmaf(x * 0.39894228040143268f, g.e, g.phi_cdf);
}

// The same GELU / GELU' with the exponential and the reciprocal on the FMA and
// integer pipes instead of the special-function unit, for epilogues where that unit
// is the bottleneck (they alternate the two forms over their values):
//   2^y, y <= 0: y = n + f with n = round(y) (adding 1.5 * 2^23), f in [-1/2, 1/2];
//     2^f from a degree-5 polynomial fitted for this file by iteratively reweighted
//     least squares on the relative error (maximum 2.3e-7 in fp32); n goes into the
//     exponent field; y < -125 gives 0.
//   1/d, d >= 1: initial guess from the exponent arithmetic bits(1/d) ~ 2 bits(1) -
//     bits(d) (exact at powers of two, within 12.5 %), then three Newton-Raphson
//     steps r <- r + r (1 - d r) (relative error 1.9e-7).
__device__ __forceinline__ float ex2_fma(float y) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float t = y + kMagic;
  const float f = y - (t - kMagic);
  float p = fmaf(0.0013276462f, f, 0.0096755400f);
  p = fmaf(p, f, 0.0555071346f);
  p = fmaf(p, f, 0.2402212024f);
  p = fmaf(p, f, 0.6931469440f);
  p = fmaf(p, f, 1.0000001192f);
  const float r = __int_as_float(__float_as_int(p) + ((__float_as_int(t) - __float_as_int(kMagic)) << 23));
  return y < -125.f ? 0.f : r;
}

__device__ __forceinline__ float rcp_fma(float d) {
  float r = __int_as_float(0x7F000000 - __float_as_int(d));
#pragma unroll
  for (int i = 0; i < 3; ++i) r = fmaf(r, fmaf(-d, r, 1.f), r);
  return r;
}

__device__ __forceinline__ GeluParts gelu_parts_fma(float x) {
  constexpr float p = 0.3275911f;
  constexpr float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f, a4 = -1.453152027f,
                  a5 = 1.061405429f;
  const float z = fabsf(x) * 0.70710678118654752f;
  const float t = rcp_fma(fmaf(p, z, 1.f));
  const float e = ex2_fma(-0.72134752044448170f * x * x);  // exp(-x^2 / 2) = 2^(-x^2 log2(e) / 2)
  const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, a5, a4), a3), a2), a1);
  const float half_erfc = 0.5f * poly * e;
  return {x >= 0.f ? 1.f - half_erfc : half_erfc, e};
}

__device__ __forceinline__ float gelu_fwd_fma(float x) { return x * gelu_parts_fma(x).phi_cdf; }

__device__ __forceinline__ float gelu_grad_fma(float x) {
  const GeluParts g = gelu_parts_fma(x);
  return fmaf(x * 0.39894228040143268f, g.e, g.phi_cdf);
}

}  // namespace mtorus
