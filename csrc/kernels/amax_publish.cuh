// Cross-rank amax publication shared by the FP8 producers (quantise kernels,
// LayerNorm with FP8 output): a block's max|x| folds into the tensor role's
// running amax; with an arrival counter, the grid's last block then stores the
// role's amax into every data-parallel peer's table (symmetric memory, one u64
// store per peer: epoch << 32 | float bits, double-buffered by step parity).
#pragma once

#include "common.cuh"

namespace mtorus {

__device__ __forceinline__ void atomic_max_pos(float* addr, float v) {
  // non-negative floats order like their bit patterns
  atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
}

// two floats -> two FP8 codes (low byte = a), round to nearest, saturating
__device__ __forceinline__ uint16_t cvt2_e4m3(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint16_t cvt2_e5m2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
  return r;
}

constexpr int kAmaxMaxPeers = 8;
struct AmaxPeers {
  uint64_t p[kAmaxMaxPeers];
  // device-resident step counter (nullptr: none).  When set, the stamp is
  // epoch + *ep and the parity its low bit, so a captured CUDA graph replays
  // with a new stamp every step.
  const unsigned int* ep;
};

// Block amax -> the slot's running amax (atomic); with a counter, the grid's last
// block then stores the slot's amax into every peer's table (see above).
__device__ __forceinline__ void publish_amax(float m, float* amax, unsigned int* counter, const AmaxPeers& table,
                                             int me, int world, int cap, int slot, int parity, unsigned int epoch,
                                             bool* last) {
  if (threadIdx.x == 0) {
    atomic_max_pos(amax, m);
    if (counter) {
      __threadfence();
      *last = atomicAdd(counter, 1u) == gridDim.x * gridDim.y - 1;
    }
  }
  if (!counter) return;
  __syncthreads();
  if (!*last) return;
  if (threadIdx.x == 0) *counter = 0u;  // ready for the next launch on this slot
  if (threadIdx.x < world) {
    if (table.ep) {
      epoch += *reinterpret_cast<const volatile unsigned int*>(table.ep);
      parity = (int)(epoch & 1u);
    }
    const float a = *reinterpret_cast<volatile float*>(amax);
    const unsigned long long v = ((unsigned long long)epoch << 32) | __float_as_uint(a);
    unsigned long long* t = reinterpret_cast<unsigned long long*>(table.p[threadIdx.x]) +
                            ((size_t)parity * world + me) * cap + slot;
    *reinterpret_cast<volatile unsigned long long*>(t) = v;
    __threadfence_system();
  }
}


}  // namespace mtorus
