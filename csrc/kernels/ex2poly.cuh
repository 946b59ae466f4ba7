// 2^x for x <= 0 on the FMA / integer pipes.  Softmax-shaped kernels run one
// exponential per element, which keeps the special-function unit (16
// exponentials per clock per SM) the bound; evaluating part of them here moves
// that work to the FP32 pipe (~10 instructions each).
//
// x = n + f with n = round(x) (the round-to-nearest of adding 1.5 * 2^23),
// f in [-1/2, 1/2]; 2^f is a cubic whose coefficients were fitted for this file
// by iteratively reweighted least squares on the relative error over
// [-1/2, 1/2] (maximum 7.5e-5 in fp32, below the 2^-9 relative rounding of a
// bf16 result); n is added to the exponent field.  x < -125 (masked scores
// included) gives 0; x must not be NaN.
#pragma once

namespace mtorus {

__device__ __forceinline__ float ex2_poly(float x) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float t = x + kMagic;
  const float f = x - (t - kMagic);
  const float p = fmaf(fmaf(fmaf(0.055171531f, f, 0.242611006f), f, 0.693260968f), f, 0.999928057f);
  const float y = __int_as_float(__float_as_int(p) + ((__float_as_int(t) - __float_as_int(kMagic)) << 23));
  return x < -125.f ? 0.f : y;
}

}  // namespace mtorus
