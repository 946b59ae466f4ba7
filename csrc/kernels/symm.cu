// Fused data-parallel collectives over NVLink peer memory (NVSwitch full mesh).
//
// Every rank's flat gradient buffer, bf16 weight buffer and a small flag / scalar
// area are allocated as symmetric memory, so kernels receive one pointer per
// peer and move data with plain loads and stores across NVLink.
//
//   rs_bucket      reduce-scatter of one gradient bucket: rank r sums chunk r of
//                  the bucket over all peers' buffers (fp32 accumulate), writes
//                  it into its own buffer and accumulates the squared norm and
//                  a non-finite flag (overflow detection): the reduction half of
//                  the fused data-parallel gradient path;
//   scalars_ar     all-reduce of the per-rank norm partials (tiny);
//   adam_shard_ag  Adam on this rank's shard (skipped on overflow, unscaled and
//                  clipped by the device multiplier) whose new bf16 weights are
//                  stored straight into every peer's weight buffer: the update
//                  and the parameter all-gather in one pass: the optimizer half of
//                  the fused data-parallel path, broadcasting the new weights;
//   wait_flags     makes a stream wait until all peers reached an epoch;
//   allreduce / allgather / broadcast / halo: standalone collectives for the
//                  microbenchmark and the torus neighbour exchange (path d).
//
// Synchronisation: flags[slot * world + src] in each rank's flag area hold an
// epoch; a producer publishes with a system-scope fence + release store into
// every peer's slot, consumers spin with acquire loads.  Every spin is bounded
// by a wall-clock limit (globaltimer); on expiry the kernel records a status
// code, skips the dependent work and returns, so a missing peer never hangs the
// GPU.  No TMA, no cluster launches.
#include <cstring>

#include "common.cuh"
#include "mx.cuh"

namespace mtorus {

constexpr int kMaxPeers = 8;
constexpr uint64_t kSymmSpinLimitNs = 5000000000ull;  // 5 s

struct PeerPtrs {
  uint64_t p[kMaxPeers];
};

__device__ __forceinline__ void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Publish `epoch` into flags[slot * n + me] of every peer.
__device__ __forceinline__ void signal_peers(const PeerPtrs& flags, int me, int n, int slot,
                                             uint32_t epoch) {
  __threadfence_system();
  for (int p = 0; p < n; ++p) {
    uint32_t* f = reinterpret_cast<uint32_t*>(flags.p[p]) + slot * n + me;
    st_release_sys(f, epoch);
  }
}

// Wait until flags[slot * n + p] >= epoch for all p (own flag area).  Bounded.
__device__ __forceinline__ bool wait_peers(const uint32_t* my_flags, int n, int slot,
                                           uint32_t epoch, int* status, int code) {
  const uint64_t t0 = globaltimer_ns();
  for (int p = 0; p < n; ++p) {
    const uint32_t* f = my_flags + slot * n + p;
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if (globaltimer_ns() - t0 > kSymmSpinLimitNs) {
        if (status) atomicExch(status, code);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// Block-wide: thread 0 (optionally) signals, then waits; the result is shared.
__device__ __forceinline__ bool block_barrier(const PeerPtrs& flags, const uint32_t* my_flags,
                                              int me, int n, int slot, uint32_t epoch,
                                              bool do_signal, int* status, int code) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (do_signal) signal_peers(flags, me, n, slot, epoch);
    ok = wait_peers(my_flags, n, slot, epoch, status, code) ? 1 : 0;
  }
  __syncthreads();
  return ok != 0;
}

// ------------------------------------------------------------------ NVLS (multimem) collectives
// The symmetric buffers are also bound to an NVLink multicast object: a
// `multimem.ld_reduce` through the multicast address returns the sum of that
// element over every GPU (the NVSwitch reduces in the switch), a `multimem.st`
// writes one value into every GPU's copy.  All-reduce: each rank reduces its
// 1/N slice in the switch and stores the result back to all ranks (each byte
// crosses its link about twice, independent of N); broadcast: the root stores
// once and the switch replicates.
__device__ __forceinline__ void mc_ld_reduce_f32(uint64_t a, float4& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(a)
               : "memory");
}
__device__ __forceinline__ void mc_ld_reduce_bf16(uint64_t a, uint4& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(a)
               : "memory");
}
__device__ __forceinline__ void mc_st_16(uint64_t a, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}
__device__ __forceinline__ void mc_publish_fence() {
  // multicast stores alias the unicast buffers the consumers read
  asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
}

// A context's device-resident step counter: with ep set, a kernel's effective epoch
// is the host value plus *ep, so a CUDA graph that advances the counter (one
// epoch_advance launch per step) replays with fresh epochs.
__device__ __forceinline__ uint32_t resolve_epoch(uint32_t epoch, const uint32_t* ep) {
  return ep ? epoch + *reinterpret_cast<const volatile uint32_t*>(ep) : epoch;
}

__global__ void epoch_advance_kernel(uint32_t* ep) { *ep += 1u; }

// ------------------------------------------------------------------ reduce-scatter
// Bucket [start, start+len) (elements, fp32).  Chunk c = [start + c*clen, ...).
__global__ void __launch_bounds__(512) rs_bucket_kernel(PeerPtrs grads, PeerPtrs flags,
                                                        uint32_t* my_flags, int me, int n,
                                                        int64_t start, int64_t len, int64_t clen,
                                                        int slot, uint32_t epoch, float inv_n,
                                                        float* st, int* status, const uint32_t* ep) {
  __shared__ float red[32];
  epoch = resolve_epoch(epoch, ep);
  if (!block_barrier(flags, my_flags, me, n, slot, epoch, blockIdx.x == 0, status, 21)) return;
  const int64_t c0 = start + (int64_t)me * clen;
  const int64_t c1 = min(start + len, c0 + clen);
  float* mine = reinterpret_cast<float*>(grads.p[me]);
  float acc2 = 0.f;
  int bad = 0;
  const int64_t nvec = (c1 > c0) ? (c1 - c0) / 4 : 0;
  // two vectors per thread per trip: 2 x n independent 16-byte peer loads in flight
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < nvec; i0 += 2 * stride) {
    float4 s[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) s[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p) {
      if (p < n) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int64_t i = i0 + u * stride;
          if (i < nvec) {
            const float4 v =
                *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(grads.p[p]) + c0 + i * 4);
            s[u].x += v.x; s[u].y += v.y; s[u].z += v.z; s[u].w += v.w;
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= nvec) continue;
      float4 t = s[u];
      t.x *= inv_n; t.y *= inv_n; t.z *= inv_n; t.w *= inv_n;
      *reinterpret_cast<float4*>(mine + c0 + i * 4) = t;
      acc2 += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
      bad |= !(isfinite(t.x) && isfinite(t.y) && isfinite(t.z) && isfinite(t.w));
    }
  }
  // scalar tail (len not a multiple of 4)
  for (int64_t off = c0 + nvec * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; off < c1;
       off += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int p = 0; p < n; ++p) s += reinterpret_cast<const float*>(grads.p[p])[off];
    s *= inv_n;
    mine[off] = s;
    acc2 += s * s;
    bad |= !isfinite(s);
  }
  acc2 = block_sum(acc2, red);
  const int anybad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    atomicAdd(st + 0, acc2);  // kStSumSq
    if (anybad) atomicAdd(st + 1, 1.f);
  }
}

// ------------------------------------------------------------------ scalars all-reduce
// scal[me * 2 + k] of every peer <- st[k] (k = 0: Σg², 1: non-finite count); then sum.
__global__ void scalars_ar_kernel(PeerPtrs scal, PeerPtrs flags, uint32_t* my_flags, int me, int n,
                                  int slot, uint32_t epoch, float* st, int* status, const uint32_t* ep) {
  if (threadIdx.x != 0) return;
  epoch = resolve_epoch(epoch, ep);
  for (int p = 0; p < n; ++p) {
    float* d = reinterpret_cast<float*>(scal.p[p]) + me * 2;
    d[0] = st[0];
    d[1] = st[1];
  }
  signal_peers(flags, me, n, slot, epoch);
  if (!wait_peers(my_flags, n, slot, epoch, status, 22)) {
    st[1] += 1.f;  // treat a missing peer as an overflow: the step is skipped
    return;
  }
  const float* mine = reinterpret_cast<const float*>(scal.p[me]);
  float s0 = 0.f, s1 = 0.f;
  for (int p = 0; p < n; ++p) {
    s0 += mine[p * 2];
    s1 += mine[p * 2 + 1];
  }
  st[0] = s0;
  st[1] = s1;
}

// ------------------------------------------------------------------ sharded Adam + all-gather
// ranges[r] = {flat offset, length, compact (m/v) offset}; blockIdx.y = range.
// w16_mc (non-zero): the multicast address of the bf16 weight buffer; each new weight
// vector is then stored once through the switch, which writes it into every rank's copy
// (one store instead of n, so the all-gather costs 1/n of the NVLink bytes).
__global__ void __launch_bounds__(256) adam_shard_ag_kernel(
    const int64_t* __restrict__ ranges, float* __restrict__ master, float* __restrict__ m,
    float* __restrict__ v, const float* __restrict__ grad, PeerPtrs w16, int n,
    const float* __restrict__ st, float lr, float beta1, float beta2, float eps, float wd, uint64_t w16_mc) {
  const int64_t off = ranges[blockIdx.y * 3], len = ranges[blockIdx.y * 3 + 1],
                moff = ranges[blockIdx.y * 3 + 2];
  const bool skip = st[5] > 0.f;  // kStSkip
  const float gm = st[4];         // kStGradMul
  const float step = st[7];       // kStStep
  const float bc1 = 1.f - powf(beta1, step), bc2 = 1.f - powf(beta2, step);
  const float step_size = lr / bc1, inv_sqrt_bc2 = rsqrtf(bc2);
  const int64_t nv = len / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = off + i * 8, mo = moff + i * 8;
    float pf[8];
    *reinterpret_cast<float4*>(pf) = *reinterpret_cast<const float4*>(master + o);
    *reinterpret_cast<float4*>(pf + 4) = *reinterpret_cast<const float4*>(master + o + 4);
    if (!skip) {
      float gf[8], mf[8], vf[8];
      *reinterpret_cast<float4*>(gf) = *reinterpret_cast<const float4*>(grad + o);
      *reinterpret_cast<float4*>(gf + 4) = *reinterpret_cast<const float4*>(grad + o + 4);
      *reinterpret_cast<float4*>(mf) = *reinterpret_cast<const float4*>(m + mo);
      *reinterpret_cast<float4*>(mf + 4) = *reinterpret_cast<const float4*>(m + mo + 4);
      *reinterpret_cast<float4*>(vf) = *reinterpret_cast<const float4*>(v + mo);
      *reinterpret_cast<float4*>(vf + 4) = *reinterpret_cast<const float4*>(v + mo + 4);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float g = gf[k] * gm;
        if (wd != 0.f) g += wd * pf[k];
        mf[k] = beta1 * mf[k] + (1.f - beta1) * g;
        vf[k] = beta2 * vf[k] + (1.f - beta2) * g * g;
        pf[k] -= step_size * mf[k] / (sqrtf(vf[k]) * inv_sqrt_bc2 + eps);
      }
      *reinterpret_cast<float4*>(master + o) = *reinterpret_cast<float4*>(pf);
      *reinterpret_cast<float4*>(master + o + 4) = *reinterpret_cast<float4*>(pf + 4);
      *reinterpret_cast<float4*>(m + mo) = *reinterpret_cast<float4*>(mf);
      *reinterpret_cast<float4*>(m + mo + 4) = *reinterpret_cast<float4*>(mf + 4);
      *reinterpret_cast<float4*>(v + mo) = *reinterpret_cast<float4*>(vf);
      *reinterpret_cast<float4*>(v + mo + 4) = *reinterpret_cast<float4*>(vf + 4);
    }
    const bf16x8 w = pack8(pf);
    if (w16_mc) {
      mc_st_16(w16_mc + (uint64_t)o * 2, *reinterpret_cast<const uint4*>(&w));
    } else {
#pragma unroll
      for (int p = 0; p < kMaxPeers; ++p)
        if (p < n) reinterpret_cast<bf16x8*>(reinterpret_cast<bf16*>(w16.p[p]) + o)[0] = w;
    }
  }
  if (w16_mc) mc_publish_fence();  // the multicast stores before the barrier that publishes them
}

// Signal (this rank finished writing into peers) then wait for everyone.
__global__ void barrier_kernel(PeerPtrs flags, uint32_t* my_flags, int me, int n, int slot,
                               uint32_t epoch, int* status, int code, const uint32_t* ep) {
  if (threadIdx.x != 0) return;
  epoch = resolve_epoch(epoch, ep);
  signal_peers(flags, me, n, slot, epoch);
  wait_peers(my_flags, n, slot, epoch, status, code);
  // peers may have written this rank's buffers through a multicast alias: order those
  // before the unicast reads of the kernels that follow
  asm volatile("fence.proxy.alias;" ::: "memory");
}

// ------------------------------------------------------------------ standalone collectives
// out (own buffer) = sum over peers of buf[p] (fp32 or bf16), every rank computes all
// elements it owns (chunk me), then all-gathers them with peer stores.
template <typename T>
__global__ void __launch_bounds__(512) allreduce_kernel(PeerPtrs bufs, PeerPtrs flags,
                                                        uint32_t* my_flags, int me, int n,
                                                        int64_t numel, int slot, uint32_t epoch,
                                                        int* status) {
  constexpr int V = 16 / sizeof(T);
  if (!block_barrier(flags, my_flags, me, n, slot, epoch, blockIdx.x == 0, status, 31)) return;
  const int64_t nvec = numel / V;
  const int64_t per = (nvec + n - 1) / n;
  const int64_t v0 = (int64_t)me * per, v1 = min(nvec, v0 + per);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = v0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < v1; i0 += 2 * stride) {
    uint4 raw[2][kMaxPeers];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int p = 0; p < kMaxPeers; ++p)
        if (p < n && i0 + u * stride < v1) raw[u][p] = reinterpret_cast<const uint4*>(bufs.p[p])[i0 + u * stride];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= v1) continue;
      float acc[V];
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] = 0.f;
#pragma unroll
      for (int p = 0; p < kMaxPeers; ++p) {
        if (p < n) {
          const T* e = reinterpret_cast<const T*>(&raw[u][p]);
#pragma unroll
          for (int k = 0; k < V; ++k) acc[k] += to_f(e[k]);
        }
      }
      uint4 outv;
      T* o = reinterpret_cast<T*>(&outv);
#pragma unroll
      for (int k = 0; k < V; ++k) o[k] = from_f<T>(acc[k]);
#pragma unroll
      for (int p = 0; p < kMaxPeers; ++p)
        if (p < n) reinterpret_cast<uint4*>(bufs.p[p])[i] = outv;
    }
  }
}

// Each rank copies its `bytes` from src (local) into slot me of every peer's dst.
__global__ void __launch_bounds__(512) allgather_kernel(const uint4* __restrict__ src,
                                                        PeerPtrs dst, int me, int n,
                                                        int64_t nvec) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = src[i];
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p)
      if (p < n) reinterpret_cast<uint4*>(dst.p[p])[(int64_t)me * nvec + i] = v;
  }
}

// Root pushes its buffer into every peer's buffer.
__global__ void __launch_bounds__(512) broadcast_kernel(PeerPtrs bufs, int root, int n,
                                                        int64_t nvec) {
  const uint4* src = reinterpret_cast<const uint4*>(bufs.p[root]);
  constexpr int U = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < nvec; i0 += U * stride) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + u * stride < nvec) v[u] = src[i0 + u * stride];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int p = 0; p < kMaxPeers; ++p)
        if (p < n && p != root && i0 + u * stride < nvec)
          reinterpret_cast<uint4*>(bufs.p[p])[i0 + u * stride] = v[u];
  }
}

// Torus neighbour exchange: this rank stores its send buffer into slot k of
// neighbour k's receive area (slots = 2 * axes, one per direction), so a 2-wide
// axis whose + and - neighbour coincide still gets two distinct slots.
__global__ void __launch_bounds__(512) halo_kernel(const uint4* __restrict__ src, PeerPtrs recv,
                                                   const int* __restrict__ nbr_rank,
                                                   const int* __restrict__ nbr_slot, int nslots,
                                                   int64_t nvec) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = src[i];
    for (int k = 0; k < nslots; ++k) {
      uint4* d = reinterpret_cast<uint4*>(recv.p[nbr_rank[k]]);
      d[(int64_t)nbr_slot[k] * nvec + i] = v;
    }
  }
}


template <int DT>  // 0: fp32, 1: bf16
__global__ void __launch_bounds__(512) allreduce_mc_kernel(uint64_t mc, PeerPtrs flags, uint32_t* my_flags,
                                                           int me, int n, int64_t numel, int slot,
                                                           uint32_t epoch, int* status) {
  if (!block_barrier(flags, my_flags, me, n, slot, epoch, blockIdx.x == 0, status, 33)) return;
  asm volatile("fence.proxy.alias;" ::: "memory");  // peers' unicast writes, read through the multicast alias
  const int64_t nvec = numel / (DT == 0 ? 4 : 8);
  const int64_t per = (nvec + n - 1) / n;
  const int64_t v0 = (int64_t)me * per, v1 = min(nvec, v0 + per);
  // four vectors per thread per trip: the switch round trip is long, keep many in flight
  constexpr int U = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = v0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < v1; i0 += U * stride) {
    uint4 r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < v1) {
        const uint64_t a = mc + (uint64_t)i * 16;
        if (DT == 0) {
          float4 f;
          mc_ld_reduce_f32(a, f);
          r[u] = make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z),
                            __float_as_uint(f.w));
        } else {
          mc_ld_reduce_bf16(a, r[u]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < v1) mc_st_16(mc + (uint64_t)i * 16, r[u]);
    }
  }
  mc_publish_fence();
}

// Only the root stores; every rank's buffer receives the data.
__global__ void __launch_bounds__(512) broadcast_mc_kernel(const uint4* __restrict__ src, uint64_t mc,
                                                           int64_t nvec) {
  constexpr int U = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < nvec; i0 += U * stride) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + u * stride < nvec) v[u] = src[i0 + u * stride];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + u * stride < nvec) mc_st_16(mc + (uint64_t)(i0 + u * stride) * 16, v[u]);
  }
  mc_publish_fence();
}

// ------------------------------------------------------------------ NVLS reduce-scatter (DP buckets)
// rs_bucket with the per-peer loads replaced by one multimem.ld_reduce through the
// gradient buffer's multicast address: the switch sums this rank's chunk over all
// ranks, so each rank receives its chunk once instead of from n peers.  Same
// outputs as rs_bucket (averaged chunk in the own buffer, sum of squares and the
// non-finite count into st).
__global__ void __launch_bounds__(512) rs_bucket_mc_kernel(uint64_t grads_mc, float* mine, PeerPtrs flags,
                                                           uint32_t* my_flags, int me, int n, int64_t start,
                                                           int64_t len, int64_t clen, int slot, uint32_t epoch,
                                                           float inv_n, float* st, int* status, const uint32_t* ep) {
  __shared__ float red[32];
  epoch = resolve_epoch(epoch, ep);
  if (!block_barrier(flags, my_flags, me, n, slot, epoch, blockIdx.x == 0, status, 25)) return;
  asm volatile("fence.proxy.alias;" ::: "memory");  // peers' unicast writes, read through the multicast alias
  const int64_t c0 = start + (int64_t)me * clen;
  const int64_t c1 = min(start + len, c0 + clen);
  float acc2 = 0.f;
  int bad = 0;
  const int64_t nvec = (c1 > c0) ? (c1 - c0) / 4 : 0;
  constexpr int U = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i0 < nvec; i0 += U * stride) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + u * stride < nvec) mc_ld_reduce_f32(grads_mc + (uint64_t)(c0 + (i0 + u * stride) * 4) * 4, v[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= nvec) continue;
      float4 t = v[u];
      t.x *= inv_n; t.y *= inv_n; t.z *= inv_n; t.w *= inv_n;
      *reinterpret_cast<float4*>(mine + c0 + i * 4) = t;
      acc2 += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
      bad |= !(isfinite(t.x) && isfinite(t.y) && isfinite(t.z) && isfinite(t.w));
    }
  }
  acc2 = block_sum(acc2, red);
  const int anybad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    atomicAdd(st + 0, acc2);
    if (anybad) atomicAdd(st + 1, 1.f);
  }
}

// ------------------------------------------------------------------ FP8 all-reduce (peer loads)
// E4M3 / E5M2 codes: decode each peer's 16 codes to fp32, sum, re-encode with
// saturation, store the result into every peer (reduce-scatter + all-gather).
__device__ __forceinline__ void dec8x2(uint16_t c, int fmt, float& a, float& b) {
  uint32_t h;
  if (fmt == 0)
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(c));
  else
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h) : "h"(c));
  const __half2 hh = *reinterpret_cast<__half2*>(&h);
  a = __low2float(hh);
  b = __high2float(hh);
}
__device__ __forceinline__ uint16_t enc8x2(float a, float b, int fmt) {
  uint16_t r;
  if (fmt == 0)
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
  else
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
  return r;
}

__global__ void __launch_bounds__(512) allreduce_fp8_kernel(PeerPtrs bufs, PeerPtrs flags, uint32_t* my_flags,
                                                            int me, int n, int64_t numel, int fmt, int slot,
                                                            uint32_t epoch, int* status) {
  if (!block_barrier(flags, my_flags, me, n, slot, epoch, blockIdx.x == 0, status, 34)) return;
  const int64_t nvec = numel / 16;
  const int64_t per = (nvec + n - 1) / n;
  const int64_t v0 = (int64_t)me * per, v1 = min(nvec, v0 + per);
  for (int64_t i = v0 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < v1;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) acc[k] = 0.f;
    uint4 raw[kMaxPeers];
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p)
      if (p < n) raw[p] = reinterpret_cast<const uint4*>(bufs.p[p])[i];
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p) {
      if (p < n) {
        const uint16_t* c = reinterpret_cast<const uint16_t*>(&raw[p]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float a, b;
          dec8x2(c[k], fmt, a, b);
          acc[2 * k] += a;
          acc[2 * k + 1] += b;
        }
      }
    }
    uint4 outv;
    uint16_t* o = reinterpret_cast<uint16_t*>(&outv);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = enc8x2(acc[2 * k], acc[2 * k + 1], fmt);
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p)
      if (p < n) reinterpret_cast<uint4*>(bufs.p[p])[i] = outv;
  }
}

// ------------------------------------------------------------------ host side
static PeerPtrs to_peers(const std::vector<int64_t>& v) {
  MT_CHECK(v.size() <= (size_t)kMaxPeers, "at most 8 peers");
  PeerPtrs p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = (uint64_t)v[i];
  return p;
}

static int* symm_status_ptr() {
  static int* s = nullptr;
  if (!s) {
    C10_CUDA_CHECK(cudaMalloc(&s, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(s, 0, sizeof(int)));
  }
  return s;
}

// ------------------------------------------------------------------ E5M2 gradient transport (DP buckets)
// Opt-in variant of rs_bucket that moves gradients over NVLink as E5M2 codes with
// one power-of-two scale per 32 values (the MX block rule of mx.cuh: the block's
// amax maps to at most the format maximum, 57344, so nothing saturates): 33 bytes
// per 32 gradients instead of 128.  dp_quant_e5m2_kernel encodes this rank's
// finished bucket into its symmetric code / scale buffers; rs_bucket_e5m2_kernel
// then decodes chunk me of every peer's bucket, sums in fp32, averages, writes the
// result into this rank's fp32 gradient buffer and accumulates the squared norm
// and the non-finite count exactly like rs_bucket.  A block holding a NaN / Inf
// carries the NaN scale byte and decodes to NaN, so overflow detection still sees it.
__global__ void __launch_bounds__(256) dp_quant_e5m2_kernel(const float* __restrict__ g, uint8_t* __restrict__ codes,
                                                            uint8_t* __restrict__ sf, int64_t nblocks,
                                                            uint32_t fmax_bits) {
  const int ef = (int)((fmax_bits >> 23) & 0xFF);
  const uint32_t mf = fmax_bits & 0x7FFFFF;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nblocks;
       b += (int64_t)gridDim.x * blockDim.x) {
    float v[32];
    const float4* src = reinterpret_cast<const float4*>(g + b * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 t = src[q];
      v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
    }
    uint32_t w[8];
    uint8_t sfb;
    mx_block(v, ef, mf, 1, w, sfb);
    uint4* dst = reinterpret_cast<uint4*>(codes + b * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    sf[b] = sfb;
  }
}

// 2^(s - 127) for a UE8M0 scale byte (0: 2^-127, a subnormal; 255: NaN).
__device__ __forceinline__ float ue8m0_value(uint32_t s) {
  if (s == 255u) return __uint_as_float(0x7FC00000u);
  if (s == 0u) return __uint_as_float(0x00400000u);
  return __uint_as_float(s << 23);
}

__global__ void __launch_bounds__(512) rs_bucket_e5m2_kernel(PeerPtrs codes, PeerPtrs sfs, PeerPtrs flags,
                                                             uint32_t* my_flags, int me, int n, int64_t start,
                                                             int64_t len, int64_t clen, int slot, uint32_t epoch,
                                                             float inv_n, float* __restrict__ mine, float* st,
                                                             int* status, const uint32_t* ep) {
  __shared__ float red[32];
  epoch = resolve_epoch(epoch, ep);
  if (!block_barrier(flags, my_flags, me, n, slot, epoch, blockIdx.x == 0, status, 26)) return;
  const int64_t c0 = start + (int64_t)me * clen;
  const int64_t c1 = min(start + len, c0 + clen);
  const int64_t nb = (c1 > c0) ? (c1 - c0) / 32 : 0;
  float acc2 = 0.f;
  int bad = 0;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = c0 + b * 32;
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p) {
      if (p < n) {
        const uint4* cp = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(codes.p[p]) + e0);
        const uint4 c0v = cp[0], c1v = cp[1];
        const uint32_t words[8] = {c0v.x, c0v.y, c0v.z, c0v.w, c1v.x, c1v.y, c1v.z, c1v.w};
        const float scale = ue8m0_value(reinterpret_cast<const uint8_t*>(sfs.p[p])[e0 / 32]);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          float a, bb;
          dec8x2((uint16_t)(words[k >> 1] >> ((k & 1) * 16)), 1, a, bb);
          acc[2 * k] += a * scale;
          acc[2 * k + 1] += bb * scale;
        }
      }
    }
    float4* dst = reinterpret_cast<float4*>(mine + e0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 t = make_float4(acc[4 * q] * inv_n, acc[4 * q + 1] * inv_n, acc[4 * q + 2] * inv_n, acc[4 * q + 3] * inv_n);
      dst[q] = t;
      acc2 += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
      bad |= !(isfinite(t.x) && isfinite(t.y) && isfinite(t.z) && isfinite(t.w));
    }
  }
  acc2 = block_sum(acc2, red);
  const int anybad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    atomicAdd(st + 0, acc2);
    if (anybad) atomicAdd(st + 1, 1.f);
  }
}

// E5M2 transport on the NCCL reducer: after an all-to-all, row p of codes / sf holds
// this rank's chunk of rank p's encoded bucket.  out[i] = bf16(inv_n * sum_p decode(p, i)),
// summed in rank order in fp32 (the same order and rounding as the CPU path).
__global__ void __launch_bounds__(256) dp_decode_mean_e5m2_kernel(const uint8_t* __restrict__ codes,
                                                                  const uint8_t* __restrict__ sf, int n, int64_t c,
                                                                  float inv_n, bf16* __restrict__ out) {
  const int64_t nb = c / 32;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    for (int p = 0; p < n; ++p) {
      const uint4* cp = reinterpret_cast<const uint4*>(codes + (int64_t)p * c + b * 32);
      const uint4 c0v = cp[0], c1v = cp[1];
      const uint32_t words[8] = {c0v.x, c0v.y, c0v.z, c0v.w, c1v.x, c1v.y, c1v.z, c1v.w};
      const float scale = ue8m0_value(sf[(int64_t)p * nb + b]);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        float a, bb;
        dec8x2((uint16_t)(words[k >> 1] >> ((k & 1) * 16)), 1, a, bb);
        acc[2 * k] += a * scale;
        acc[2 * k + 1] += bb * scale;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] *= inv_n;
    bf16x8* dst = reinterpret_cast<bf16x8*>(out + b * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q) dst[q] = pack8(acc + 8 * q);
  }
}

int64_t symm_status(bool reset) {
  int h = 0;
  C10_CUDA_CHECK(cudaMemcpy(&h, symm_status_ptr(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) C10_CUDA_CHECK(cudaMemset(symm_status_ptr(), 0, sizeof(int)));
  return h;
}

void symm_rs_bucket(const std::vector<int64_t>& grads, const std::vector<int64_t>& flags,
                    int64_t me, int64_t start, int64_t len, int64_t clen, int64_t slot,
                    int64_t epoch, at::Tensor st, int64_t ctas, double inv_n, int64_t ep_ptr) {
  const int n = grads.size();
  rs_bucket_kernel<<<(int)ctas, 512, 0, cur_stream()>>>(
      to_peers(grads), to_peers(flags), reinterpret_cast<uint32_t*>(flags[me]), (int)me, n, start,
      len, clen, (int)slot, (uint32_t)epoch, (float)inv_n, st.data_ptr<float>(), symm_status_ptr(),
      reinterpret_cast<const uint32_t*>(ep_ptr));
  MT_LAUNCH_CHECK();
}

// NVLS variant of symm_rs_bucket (grads_mc: multicast address of the gradient buffer).
void symm_rs_bucket_mc(int64_t grads_mc, const std::vector<int64_t>& grads, const std::vector<int64_t>& flags,
                       int64_t me, int64_t start, int64_t len, int64_t clen, int64_t slot, int64_t epoch,
                       at::Tensor st, int64_t ctas, double inv_n, int64_t ep_ptr) {
  MT_CHECK(grads_mc != 0 && grads_mc % 16 == 0, "rs_bucket_mc: no multicast address");
  MT_CHECK(start % 4 == 0 && clen % 4 == 0 && len % 4 == 0, "rs_bucket_mc: 16-byte aligned bucket and chunks");
  const int n = flags.size();
  rs_bucket_mc_kernel<<<(int)ctas, 512, 0, cur_stream()>>>(
      (uint64_t)grads_mc, reinterpret_cast<float*>(grads[me]), to_peers(flags),
      reinterpret_cast<uint32_t*>(flags[me]), (int)me, n, start, len, clen, (int)slot, (uint32_t)epoch,
      (float)inv_n, st.data_ptr<float>(), symm_status_ptr(), reinterpret_cast<const uint32_t*>(ep_ptr));
  MT_LAUNCH_CHECK();
}

// E5M2 gradient transport: encode this rank's bucket (fp32 at grad, nelem a multiple of 32)
// into codes / sf (one scale byte per 32 values) on the current stream.
void dp_quant_e5m2(int64_t grad, int64_t codes, int64_t sf, int64_t nelem) {
  MT_CHECK(nelem % 32 == 0 && grad % 16 == 0 && codes % 16 == 0, "dp_quant_e5m2: 32-element blocks, aligned buffers");
  if (nelem == 0) return;
  const float fm = 57344.f;  // E5M2 largest finite value
  uint32_t fbits;
  std::memcpy(&fbits, &fm, 4);
  const int64_t nblocks = nelem / 32;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((nblocks + 255) / 256, (int64_t)num_sms() * 8));
  dp_quant_e5m2_kernel<<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<const float*>(grad),
                                                       reinterpret_cast<uint8_t*>(codes), reinterpret_cast<uint8_t*>(sf),
                                                       nblocks, fbits);
  MT_LAUNCH_CHECK();
}

// rs_bucket over E5M2-encoded buckets: codes / sfs are every rank's code and scale
// buffers (element and block offsets match the fp32 gradient buffer), mine this
// rank's fp32 gradient buffer that receives the averaged chunk.
void symm_rs_bucket_e5m2(const std::vector<int64_t>& codes, const std::vector<int64_t>& sfs,
                         const std::vector<int64_t>& flags, int64_t me, int64_t start, int64_t len, int64_t clen,
                         int64_t slot, int64_t epoch, at::Tensor st, int64_t ctas, double inv_n, int64_t mine,
                         int64_t ep_ptr) {
  MT_CHECK(start % 32 == 0 && len % 32 == 0 && clen % 32 == 0, "rs_bucket_e5m2: 32-element aligned bucket and chunks");
  MT_CHECK(codes.size() == flags.size() && sfs.size() == flags.size(), "rs_bucket_e5m2: one buffer per rank");
  rs_bucket_e5m2_kernel<<<(int)ctas, 512, 0, cur_stream()>>>(
      to_peers(codes), to_peers(sfs), to_peers(flags), reinterpret_cast<uint32_t*>(flags[me]), (int)me,
      (int)flags.size(), start, len, clen, (int)slot, (uint32_t)epoch, (float)inv_n, reinterpret_cast<float*>(mine),
      st.data_ptr<float>(), symm_status_ptr(), reinterpret_cast<const uint32_t*>(ep_ptr));
  MT_LAUNCH_CHECK();
}

// codes [n, c] and sf [n, c / 32] (uint8, contiguous, c a multiple of 32) -> out bf16 [c].
void dp_decode_mean_e5m2(const at::Tensor& codes, const at::Tensor& sf, at::Tensor out) {
  MT_CHECK(codes.dim() == 2 && codes.element_size() == 1 && codes.is_contiguous(), "dp_decode_mean_e5m2: codes [n, c]");
  const int64_t n = codes.size(0), c = codes.size(1);
  MT_CHECK(c % 32 == 0 && sf.numel() == n * (c / 32) && sf.is_contiguous() && sf.element_size() == 1,
           "dp_decode_mean_e5m2: sf [n, c / 32]");
  MT_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == c, "dp_decode_mean_e5m2: out");
  MT_CHECK(reinterpret_cast<uintptr_t>(codes.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "dp_decode_mean_e5m2: 16-byte aligned buffers");
  if (c == 0) return;
  const int64_t nb = c / 32;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((nb + 255) / 256, (int64_t)num_sms() * 8));
  dp_decode_mean_e5m2_kernel<<<grid, 256, 0, cur_stream()>>>(
      reinterpret_cast<const uint8_t*>(codes.data_ptr()), reinterpret_cast<const uint8_t*>(sf.data_ptr()), (int)n, c,
      1.f / (float)n, reinterpret_cast<bf16*>(out.data_ptr()));
  MT_LAUNCH_CHECK();
}

void symm_scalars_ar(const std::vector<int64_t>& scal, const std::vector<int64_t>& flags,
                     int64_t me, int64_t slot, int64_t epoch, at::Tensor st, int64_t ep_ptr) {
  scalars_ar_kernel<<<1, 32, 0, cur_stream()>>>(to_peers(scal), to_peers(flags),
                                                reinterpret_cast<uint32_t*>(flags[me]), (int)me,
                                                (int)scal.size(), (int)slot, (uint32_t)epoch,
                                                st.data_ptr<float>(), symm_status_ptr(),
                                                reinterpret_cast<const uint32_t*>(ep_ptr));
  MT_LAUNCH_CHECK();
}

void symm_adam_shard_ag(const at::Tensor& ranges, at::Tensor master, at::Tensor m, at::Tensor v,
                        const at::Tensor& grad, const std::vector<int64_t>& w16, const at::Tensor& st,
                        double lr, double beta1, double beta2, double eps, double wd, int64_t w16_mc) {
  MT_CHECK(w16_mc % 16 == 0, "symm_adam_shard_ag: 16-byte aligned multicast address");
  const int nr = ranges.size(0);
  if (nr == 0) return;
  dim3 grid(std::max(1, num_sms() * 4 / std::max(nr, 1)), nr);
  adam_shard_ag_kernel<<<grid, 256, 0, cur_stream()>>>(
      ranges.data_ptr<int64_t>(), master.data_ptr<float>(), m.data_ptr<float>(),
      v.data_ptr<float>(), grad.data_ptr<float>(), to_peers(w16), (int)w16.size(),
      st.data_ptr<float>(), (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd, (uint64_t)w16_mc);
  MT_LAUNCH_CHECK();
}

// Copy-engine copy of `bytes` from src (any address in this process's unified
// space: a peer's symmetric buffer included) to dst on the current stream: one
// cudaMemcpyAsync per call, no SM involved, so it overlaps with kernels on other
// streams.
void copy_async(int64_t dst, int64_t src, int64_t bytes) {
  MT_CHECK(bytes >= 0, "copy_async: bytes >= 0");
  if (bytes == 0) return;
  C10_CUDA_CHECK(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), (size_t)bytes,
                                 cudaMemcpyDeviceToDevice, cur_stream()));
}

void symm_barrier(const std::vector<int64_t>& flags, int64_t me, int64_t slot, int64_t epoch,
                  int64_t code, int64_t ep_ptr) {
  barrier_kernel<<<1, 32, 0, cur_stream()>>>(to_peers(flags), reinterpret_cast<uint32_t*>(flags[me]),
                                             (int)me, (int)flags.size(), (int)slot, (uint32_t)epoch,
                                             symm_status_ptr(), (int)code, reinterpret_cast<const uint32_t*>(ep_ptr));
  MT_LAUNCH_CHECK();
}

// Advance a device-resident step counter (uint32 [1]) on the current stream.
void symm_epoch_advance(at::Tensor ep) {
  MT_CHECK(ep.is_cuda() && ep.element_size() == 4 && ep.numel() >= 1, "symm_epoch_advance: int32 [1] on the GPU");
  epoch_advance_kernel<<<1, 1, 0, cur_stream()>>>(reinterpret_cast<uint32_t*>(ep.data_ptr()));
  MT_LAUNCH_CHECK();
}

void symm_allreduce(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t me,
                    int64_t numel, int64_t dtype, int64_t slot, int64_t epoch, int64_t ctas) {
  const int n = bufs.size();
  if (dtype == 0)
    allreduce_kernel<float><<<(int)ctas, 512, 0, cur_stream()>>>(
        to_peers(bufs), to_peers(flags), reinterpret_cast<uint32_t*>(flags[me]), (int)me, n, numel,
        (int)slot, (uint32_t)epoch, symm_status_ptr());
  else
    allreduce_kernel<bf16><<<(int)ctas, 512, 0, cur_stream()>>>(
        to_peers(bufs), to_peers(flags), reinterpret_cast<uint32_t*>(flags[me]), (int)me, n, numel,
        (int)slot, (uint32_t)epoch, symm_status_ptr());
  MT_LAUNCH_CHECK();
}

// NVLS all-reduce through the multicast address `mc` (fp32: dtype 0, bf16: 1), or
// the FP8 all-reduce over peer loads (dtype 2: E4M3, 3: E5M2; `mc` unused).
void symm_allreduce_mc(int64_t mc, const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags,
                       int64_t me, int64_t numel, int64_t dtype, int64_t slot, int64_t epoch, int64_t ctas) {
  const int n = flags.size();
  auto* my = reinterpret_cast<uint32_t*>(flags[me]);
  if (dtype == 0 || dtype == 1) {
    MT_CHECK(mc != 0, "allreduce_mc: no multicast address");
    MT_CHECK(mc % 16 == 0 && numel % (dtype == 0 ? 4 : 8) == 0, "allreduce_mc: 16-byte granularity");
    if (dtype == 0)
      allreduce_mc_kernel<0><<<(int)ctas, 512, 0, cur_stream()>>>((uint64_t)mc, to_peers(flags), my, (int)me, n,
                                                                  numel, (int)slot, (uint32_t)epoch,
                                                                  symm_status_ptr());
    else
      allreduce_mc_kernel<1><<<(int)ctas, 512, 0, cur_stream()>>>((uint64_t)mc, to_peers(flags), my, (int)me, n,
                                                                  numel, (int)slot, (uint32_t)epoch,
                                                                  symm_status_ptr());
  } else {
    MT_CHECK(numel % 16 == 0 && bufs.size() == flags.size(), "allreduce fp8: numel % 16, one buffer per rank");
    allreduce_fp8_kernel<<<(int)ctas, 512, 0, cur_stream()>>>(to_peers(bufs), to_peers(flags), my, (int)me, n,
                                                              numel, (int)(dtype - 2), (int)slot, (uint32_t)epoch,
                                                              symm_status_ptr());
  }
  MT_LAUNCH_CHECK();
}

void symm_broadcast_mc(int64_t src, int64_t mc, int64_t bytes, int64_t ctas) {
  MT_CHECK(bytes % 16 == 0 && mc % 16 == 0 && mc != 0, "broadcast_mc: 16-byte granularity, multicast address");
  broadcast_mc_kernel<<<(int)ctas, 512, 0, cur_stream()>>>(reinterpret_cast<const uint4*>(src), (uint64_t)mc,
                                                           bytes / 16);
  MT_LAUNCH_CHECK();
}

void symm_allgather(int64_t src, const std::vector<int64_t>& dst, int64_t me, int64_t bytes,
                    int64_t ctas) {
  MT_CHECK(bytes % 16 == 0, "allgather: bytes must be a multiple of 16");
  allgather_kernel<<<(int)ctas, 512, 0, cur_stream()>>>(reinterpret_cast<const uint4*>(src),
                                                        to_peers(dst), (int)me, (int)dst.size(),
                                                        bytes / 16);
  MT_LAUNCH_CHECK();
}

void symm_broadcast(const std::vector<int64_t>& bufs, int64_t root, int64_t bytes, int64_t ctas) {
  MT_CHECK(bytes % 16 == 0, "broadcast: bytes must be a multiple of 16");
  broadcast_kernel<<<(int)ctas, 512, 0, cur_stream()>>>(to_peers(bufs), (int)root,
                                                        (int)bufs.size(), bytes / 16);
  MT_LAUNCH_CHECK();
}

void symm_halo(int64_t src, const std::vector<int64_t>& recv, const at::Tensor& nbr_rank,
               const at::Tensor& nbr_slot, int64_t bytes, int64_t ctas) {
  MT_CHECK(bytes % 16 == 0, "halo: bytes must be a multiple of 16");
  halo_kernel<<<(int)ctas, 512, 0, cur_stream()>>>(
      reinterpret_cast<const uint4*>(src), to_peers(recv), nbr_rank.data_ptr<int>(),
      nbr_slot.data_ptr<int>(), (int)nbr_rank.numel(), bytes / 16);
  MT_LAUNCH_CHECK();
}


// ------------------------------------------------------------------ byte-message communicator
// Kernels behind the device Communicator (mtorus.comm.device.SymmCommunicator):
// messages of any length live in symmetric byte buffers as [int64 length | 8 pad |
// payload], and every collective is a pull of whole messages over NVLink.
//
//   pull_msgs        copies the messages of a list of peers (their staging buffers)
//                    into local slots: all_gather (every peer), broadcast (the
//                    root), the neighbour exchange (the torus neighbours) and a
//                    point-to-point receive (one sender);
//   allreduce_msgs   reads every peer's staged message and reduces it element by
//                    element in rank order (Sum / Product / Min / Max / Mean over
//                    u64, i64, f32, f64, i32, u8), which is the order the host
//                    reduce_buffers uses, so float results agree bit for bit;
//   flag_kernel      release-stores one flag into a peer and / or waits (bounded)
//                    for one of its own flags: the handshake of point-to-point
//                    messages.
constexpr int kMaxMsgs = 16;
constexpr int64_t kMsgHeader = 16;

struct MsgList {
  int peer[kMaxMsgs];
  int slot[kMaxMsgs];
  int n;
};

__global__ void __launch_bounds__(256) pull_msgs_kernel(PeerPtrs src, int64_t src_off, uint8_t* dst,
                                                        int64_t slot_bytes, MsgList msgs, int* status) {
  const int per_msg = gridDim.x / msgs.n;
  const int k = blockIdx.x / per_msg, part = blockIdx.x % per_msg;
  if (k >= msgs.n) return;
  const uint8_t* s = reinterpret_cast<const uint8_t*>(src.p[msgs.peer[k]]) + src_off;
  uint8_t* d = dst + (int64_t)msgs.slot[k] * slot_bytes;
  int64_t len = *reinterpret_cast<const volatile int64_t*>(s);
  if (len < 0 || len > slot_bytes - kMsgHeader) {
    if (threadIdx.x == 0 && part == 0) atomicExch(status, 51);
    len = 0;
  }
  const int64_t nvec = (kMsgHeader + len + 15) / 16;
  const uint4* sv = reinterpret_cast<const uint4*>(s);
  uint4* dv = reinterpret_cast<uint4*>(d);
  for (int64_t i = (int64_t)part * blockDim.x + threadIdx.x; i < nvec; i += (int64_t)per_msg * blockDim.x)
    dv[i] = sv[i];
}

template <typename T>
__device__ __forceinline__ T reduce_one(int op, T a, T b) {
  switch (op) {
    case 1: return a * b;
    case 2: return b < a ? b : a;
    case 3: return a < b ? b : a;
    default: return a + b;  // Sum, Mean
  }
}

template <typename T>
__global__ void __launch_bounds__(256) allreduce_msgs_kernel(PeerPtrs src, int64_t src_off, uint8_t* dst, int n,
                                                             int op, int64_t cap, int* status) {
  // element count from rank 0's message (reference semantics); shorter messages read as zeros
  const int64_t len0 = *reinterpret_cast<const volatile int64_t*>(reinterpret_cast<const uint8_t*>(src.p[0]) + src_off);
  if (len0 < 0 || len0 > cap) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(status, 52);
    return;
  }
  const int64_t count = len0 / (int64_t)sizeof(T);
  if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<int64_t*>(dst) = count * (int64_t)sizeof(T);
  __shared__ int64_t lens[kMaxPeers];
  if (threadIdx.x < n)
    lens[threadIdx.x] =
        *reinterpret_cast<const volatile int64_t*>(reinterpret_cast<const uint8_t*>(src.p[threadIdx.x]) + src_off);
  __syncthreads();
  T* out = reinterpret_cast<T*>(dst + kMsgHeader);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const T* s0 = reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(src.p[0]) + src_off + kMsgHeader);
    T acc = s0[i];
    for (int p = 1; p < n; ++p) {
      const T* sp = reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(src.p[p]) + src_off + kMsgHeader);
      const T x = (i + 1) * (int64_t)sizeof(T) <= lens[p] ? sp[i] : T(0);
      acc = reduce_one<T>(op, acc, x);
    }
    if (op == 4) acc = static_cast<T>(acc / static_cast<T>(n));
    out[i] = acc;
  }
}

__global__ void flag_kernel(uint32_t* signal_addr, uint32_t signal_value, const uint32_t* wait_addr,
                            uint32_t wait_value, int* status, int code) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (signal_addr) {
    __threadfence_system();
    st_release_sys(signal_addr, signal_value);
  }
  if (wait_addr) {
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(wait_addr) - wait_value) < 0) {
      if (globaltimer_ns() - t0 > kSymmSpinLimitNs) {
        atomicExch(status, code);
        return;
      }
      __nanosleep(128);
    }
  }
}

void symm_pull_msgs(const std::vector<int64_t>& src, int64_t src_off, int64_t dst, int64_t slot_bytes,
                    const std::vector<int64_t>& peers, const std::vector<int64_t>& slots, int64_t ctas_per_msg) {
  MT_CHECK(!peers.empty() && peers.size() == slots.size() && peers.size() <= (size_t)kMaxMsgs,
           "pull_msgs: 1..16 (peer, slot) pairs");
  MT_CHECK(slot_bytes % 16 == 0 && src_off % 16 == 0 && dst % 16 == 0, "pull_msgs: 16-byte alignment");
  MsgList m{};
  m.n = (int)peers.size();
  for (int i = 0; i < m.n; ++i) {
    MT_CHECK(peers[i] >= 0 && peers[i] < (int64_t)src.size(), "pull_msgs: peer out of range");
    m.peer[i] = (int)peers[i];
    m.slot[i] = (int)slots[i];
  }
  const int per = (int)std::max<int64_t>(1, ctas_per_msg);
  pull_msgs_kernel<<<per * m.n, 256, 0, cur_stream()>>>(to_peers(src), src_off, reinterpret_cast<uint8_t*>(dst),
                                                       slot_bytes, m, symm_status_ptr());
  MT_LAUNCH_CHECK();
}

// dtype: 0 U64, 1 I64, 2 F32, 3 F64, 4 I32, 5 U8 (the host DType order); op: 0 Sum, 1 Product,
// 2 Min, 3 Max, 4 Mean (the host ReduceOp order).
void symm_allreduce_msgs(const std::vector<int64_t>& src, int64_t src_off, int64_t dst, int64_t dtype, int64_t op,
                         int64_t cap, int64_t ctas) {
  MT_CHECK(op >= 0 && op <= 4, "allreduce_msgs: op 0..4");
  MT_CHECK(src_off % 16 == 0 && dst % 16 == 0, "allreduce_msgs: 16-byte alignment");
  const int n = (int)src.size();
  auto* d = reinterpret_cast<uint8_t*>(dst);
  const PeerPtrs pp = to_peers(src);
  const int g = (int)std::max<int64_t>(1, ctas);
  switch (dtype) {
    case 0: allreduce_msgs_kernel<uint64_t><<<g, 256, 0, cur_stream()>>>(pp, src_off, d, n, (int)op, cap, symm_status_ptr()); break;
    case 1: allreduce_msgs_kernel<int64_t><<<g, 256, 0, cur_stream()>>>(pp, src_off, d, n, (int)op, cap, symm_status_ptr()); break;
    case 2: allreduce_msgs_kernel<float><<<g, 256, 0, cur_stream()>>>(pp, src_off, d, n, (int)op, cap, symm_status_ptr()); break;
    case 3: allreduce_msgs_kernel<double><<<g, 256, 0, cur_stream()>>>(pp, src_off, d, n, (int)op, cap, symm_status_ptr()); break;
    case 4: allreduce_msgs_kernel<int32_t><<<g, 256, 0, cur_stream()>>>(pp, src_off, d, n, (int)op, cap, symm_status_ptr()); break;
    case 5: allreduce_msgs_kernel<uint8_t><<<g, 256, 0, cur_stream()>>>(pp, src_off, d, n, (int)op, cap, symm_status_ptr()); break;
    default: MT_CHECK(false, "allreduce_msgs: unknown dtype");
  }
  MT_LAUNCH_CHECK();
}

void symm_flag(int64_t signal_addr, int64_t signal_value, int64_t wait_addr, int64_t wait_value, int64_t code) {
  flag_kernel<<<1, 32, 0, cur_stream()>>>(reinterpret_cast<uint32_t*>(signal_addr), (uint32_t)signal_value,
                                          reinterpret_cast<const uint32_t*>(wait_addr), (uint32_t)wait_value,
                                          symm_status_ptr(), (int)code);
  MT_LAUNCH_CHECK();
}

}  // namespace mtorus
