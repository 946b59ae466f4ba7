// Counter-based random numbers for dropout: Philox4x32-10 (J. K. Salmon, M. A.
// Moraes, R. O. Dror, D. E. Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011): a 128-bit counter and a 64-bit key, ten rounds of two 32 x 32 -> 64-bit
// multiplies with the round constants and key schedule published in that paper.
// The same (key, counter) gives the same bits in any kernel, so a dropout mask
// drawn in a forward epilogue is drawn again, bit for bit, by the backward kernel
// that needs it (and by a recomputed forward under activation checkpointing)
// instead of being stored.
//
// Dropout draw: element e of site `site` (a dropout call site of the model, e.g.
// layer * 8 + role) belongs to the group of 8 consecutive elements e / 8; that
// group's Philox block (counter = {e/8 low, e/8 high, site, 0}, key = the step's
// seed) yields eight 16-bit uniforms, and element e is kept when its uniform is at
// least thr16 = round(p * 65536) (so p is honoured to 2^-16).  Kept values are
// scaled by 1 / (1 - p).
#pragma once

#include <cstdint>

namespace mtorus {

__host__ __device__ __forceinline__ void philox4x32_10(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Keep bits (bit j = element 8 * group + j) of one 8-element group.
__host__ __device__ __forceinline__ uint32_t dropout_keep8(uint32_t seed_lo, uint32_t seed_hi, uint32_t site,
                                                           uint64_t group, uint32_t thr16) {
  uint32_t c[4] = {(uint32_t)group, (uint32_t)(group >> 32), site, 0u};
  philox4x32_10(c, seed_lo, seed_hi);
  uint32_t keep = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t u = (c[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu;
    keep |= (u >= thr16 ? 1u : 0u) << j;
  }
  return keep;
}

// Device-side dropout parameters of one call site; rng points at the step's key
// {seed_lo, seed_hi} in device memory, so a captured CUDA graph draws new masks at
// every replay once the key is advanced on the device.
struct DropoutArgs {
  const uint32_t* rng;
  uint32_t site;
  uint32_t thr16;
  float scale;  // 1 / (1 - p)
};

}  // namespace mtorus
