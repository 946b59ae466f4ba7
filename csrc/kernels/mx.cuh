// MXFP8 block helpers shared by the quantisers that write block-scaled operands
// (fp8.cu: mx_quantize_rc; layernorm.cu: the LayerNorm that writes MX codes).
//
// mx_block: one 32-element block -> 32 codes (8 packed words) and its UE8M0 scale
// byte.  X = the smallest integer with amax <= fmax * 2^X, from the IEEE-754 fields
// (amax = (1 + ma) 2^ea, fmax = (1 + mf) 2^ef: X = ea - ef + (ma > mf)); codes are
// fp8(v * 2^-X) with the saturating round-to-nearest-even cvt; an all-zero block
// gets X = 0, a block holding a NaN / Inf the NaN scale byte 255 (and X = 0 codes).
// mx_sf_offset: byte of row r, K-block j in the tcgen05 scale atom layout
// [ceil(R/128)][nkb4][512], (r % 32) * 16 + (r % 128 / 32) * 4 + j % 4.
#pragma once

#include "amax_publish.cuh"

namespace mtorus {

// max(a, |b|) that propagates NaN (a NaN anywhere in a block makes its amax NaN)
__device__ __forceinline__ float max_nan_abs(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(fabsf(b)));
  return d;
}

__device__ __forceinline__ void mx_block(const float (&v)[32], int ef, uint32_t mf, int fmt, uint32_t (&w)[8],
                                         uint8_t& sfb) {
  // two independent chains, one NaN-propagating max per value
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    a0 = max_nan_abs(a0, v[i]);
    a1 = max_nan_abs(a1, v[i + 1]);
  }
  float amax;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(amax) : "f"(a0), "f"(a1));
  // a block holding a NaN / Inf: scale byte 255 and codes of the unscaled values
  const bool finite = amax <= 3.402823466e38f;
  int X = 0;
  if (finite && amax > 0.f) {
    const uint32_t ua = __float_as_uint(amax);
    X = (int)((ua >> 23) & 0xFF) - ef + ((ua & 0x7FFFFF) > mf ? 1 : 0);
    X = max(-127, min(127, X));
  }
  const float inv = __uint_as_float((uint32_t)(127 - min(X, 126)) << 23);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float* t = v + 4 * q;
    const uint16_t lo = fmt == 0 ? cvt2_e4m3(t[0] * inv, t[1] * inv) : cvt2_e5m2(t[0] * inv, t[1] * inv);
    const uint16_t hi = fmt == 0 ? cvt2_e4m3(t[2] * inv, t[3] * inv) : cvt2_e5m2(t[2] * inv, t[3] * inv);
    w[q] = (uint32_t)lo | ((uint32_t)hi << 16);
  }
  sfb = finite ? (uint8_t)(X + 127) : (uint8_t)255;
}

__device__ __forceinline__ int64_t mx_sf_offset(int r, int j, int nkb4) {
  const int rr = r & 127;
  return ((int64_t)(r >> 7) * nkb4 + (j >> 2)) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + (j & 3);
}

}  // namespace mtorus
