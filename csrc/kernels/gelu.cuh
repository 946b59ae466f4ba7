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

}  // namespace mtorus
