// LayerNorm forward / backward for the GPT blocks (pre-LN, eps = 1e-5).
//
// Reference semantics: Burn's LayerNorm as used by the GPT example
// (examples/gpt-1b/src/transformer.rs:134-135,146,152 and model.rs:88,127):
//   y = (x - mean) / sqrt(var + eps) * gamma + beta, biased variance.
//
// Design (B200): one warp per row, the row held in registers as 16-byte bf16x8
// vectors (NCH chunks of 256 columns), so a row is read from HBM exactly once.
// gamma/beta are the fp32 master parameters.  The backward writes dx and
// accumulates dgamma/dbeta in per-warp shared-memory slices, reduced per block
// into a [blocks, 2, d] partial buffer and finished by a column-sum kernel.
#include "common.cuh"

namespace mtorus {

template <int NCH>
__global__ void __launch_bounds__(256) ln_fwd_vec(const bf16* __restrict__ x,
                                                  const float* __restrict__ gamma,
                                                  const float* __restrict__ beta,
                                                  bf16* __restrict__ y, float* __restrict__ mean_out,
                                                  float* __restrict__ rstd_out, int rows, int d,
                                                  float eps) {
  const int lane = threadIdx.x & 31;
  const int warps_per_block = blockDim.x >> 5;
  const int row0 = blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int stride = gridDim.x * warps_per_block;
  for (int row = row0; row < rows; row += stride) {
    const bf16* xr = x + (size_t)row * d;
    float v[NCH][8];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
      if (col < d) {
        bf16x8 t = *reinterpret_cast<const bf16x8*>(xr + col);
        unpack8(t, v[c]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[c][i];
    }
    const float mean = warp_sum(s) / d;
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
      if (col < d) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float t = v[c][i] - mean;
          q += t * t;
        }
      }
    }
    const float rstd = rsqrtf(warp_sum(q) / d + eps);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
      if (col < d) {
        const float4 g0 = *reinterpret_cast<const float4*>(gamma + col);
        const float4 g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
        const float4 b0 = *reinterpret_cast<const float4*>(beta + col);
        const float4 b1 = *reinterpret_cast<const float4*>(beta + col + 4);
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = (v[c][i] - mean) * rstd * g[i] + b[i];
        *reinterpret_cast<bf16x8*>(y + (size_t)row * d + col) = pack8(o);
      }
    }
    if (lane == 0) {
      if (mean_out) mean_out[row] = mean;
      if (rstd_out) rstd_out[row] = rstd;
    }
  }
}

// Generic fallback (any d): warp per row, three passes over the row.
__global__ void ln_fwd_generic(const bf16* __restrict__ x, const float* __restrict__ gamma,
                               const float* __restrict__ beta, bf16* __restrict__ y,
                               float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows,
                               int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bf16* xr = x + (size_t)row * d;
  float s = 0.f;
  for (int i = lane; i < d; i += 32) s += __bfloat162float(xr[i]);
  const float mean = warp_sum(s) / d;
  float q = 0.f;
  for (int i = lane; i < d; i += 32) {
    const float t = __bfloat162float(xr[i]) - mean;
    q += t * t;
  }
  const float rstd = rsqrtf(warp_sum(q) / d + eps);
  for (int i = lane; i < d; i += 32)
    y[(size_t)row * d + i] =
        __float2bfloat16_rn((__bfloat162float(xr[i]) - mean) * rstd * gamma[i] + beta[i]);
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
}

// Backward: dx per row; dgamma/dbeta partials per block -> part[blockIdx][2][d].
template <int NCH>
__global__ void __launch_bounds__(128) ln_bwd_vec(const bf16* __restrict__ dy,
                                                  const bf16* __restrict__ x,
                                                  const float* __restrict__ gamma,
                                                  const float* __restrict__ mean_in,
                                                  const float* __restrict__ rstd_in,
                                                  bf16* __restrict__ dx, float* __restrict__ part,
                                                  int rows, int d) {
  extern __shared__ float sm[];  // [warps][2][d]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float* sdg = sm + (size_t)wid * 2 * d;
  float* sdb = sdg + d;
  for (int i = lane; i < 2 * d; i += 32) sdg[i] = 0.f;
  __syncwarp();
  for (int row = blockIdx.x * nw + wid; row < rows; row += gridDim.x * nw) {
    const float mean = mean_in[row], rstd = rstd_in[row];
    float xh[NCH][8], g[NCH][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
      if (col < d) {
        float xv[8], dv[8];
        unpack8(*reinterpret_cast<const bf16x8*>(x + (size_t)row * d + col), xv);
        unpack8(*reinterpret_cast<const bf16x8*>(dy + (size_t)row * d + col), dv);
        const float4 g0 = *reinterpret_cast<const float4*>(gamma + col);
        const float4 g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          xh[c][i] = (xv[i] - mean) * rstd;
          g[c][i] = dv[i] * gg[i];  // dxhat
          s1 += g[c][i];
          s2 += g[c][i] * xh[c][i];
          sdg[col + i] += dv[i] * xh[c][i];
          sdb[col + i] += dv[i];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) xh[c][i] = g[c][i] = 0.f;
      }
    }
    const float c2 = warp_sum(s1) / d;
    const float c1 = warp_sum(s2) / d;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
      if (col < d) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = (g[c][i] - xh[c][i] * c1 - c2) * rstd;
        *reinterpret_cast<bf16x8*>(dx + (size_t)row * d + col) = pack8(o);
      }
    }
  }
  __syncthreads();
  float* out = part + (size_t)blockIdx.x * 2 * d;
  for (int i = threadIdx.x; i < 2 * d; i += blockDim.x) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += sm[(size_t)w * 2 * d + i];
    out[i] = t;
  }
}

__global__ void ln_bwd_generic(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                               const float* __restrict__ gamma, const float* __restrict__ mean_in,
                               const float* __restrict__ rstd_in, bf16* __restrict__ dx,
                               float* __restrict__ part, int rows, int d) {
  // One block per row group; partial sums accumulated directly per block row.
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float* out = part + (size_t)blockIdx.x * 2 * d;
  for (int row = blockIdx.x * nw + wid; row < rows; row += gridDim.x * nw) {
    const float mean = mean_in[row], rstd = rstd_in[row];
    float s1 = 0.f, s2 = 0.f;
    for (int i = lane; i < d; i += 32) {
      const float xh = (__bfloat162float(x[(size_t)row * d + i]) - mean) * rstd;
      const float g = __bfloat162float(dy[(size_t)row * d + i]) * gamma[i];
      s1 += g;
      s2 += g * xh;
    }
    const float c2 = warp_sum(s1) / d, c1 = warp_sum(s2) / d;
    for (int i = lane; i < d; i += 32) {
      const float dv = __bfloat162float(dy[(size_t)row * d + i]);
      const float xh = (__bfloat162float(x[(size_t)row * d + i]) - mean) * rstd;
      const float g = dv * gamma[i];
      dx[(size_t)row * d + i] = __float2bfloat16_rn((g - xh * c1 - c2) * rstd);
      atomicAdd(out + i, dv * xh);
      atomicAdd(out + d + i, dv);
    }
  }
}

// Sum partials over blocks: dg[i] (+)= sum_b part[b][0][i]; db likewise.
__global__ void ln_bwd_finish(const float* __restrict__ part, float* __restrict__ dgamma,
                              float* __restrict__ dbeta, int nblocks, int d, int accumulate) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * d) return;
  float t = 0.f;
  for (int b = 0; b < nblocks; ++b) t += part[(size_t)b * 2 * d + i];
  float* dst = i < d ? dgamma + i : dbeta + (i - d);
  *dst = accumulate ? *dst + t : t;
}

static int pick_nch(int d) {
  if (d % 8 != 0) return 0;
  if (d <= 256) return 1;
  if (d <= 512) return 2;
  if (d <= 1024) return 4;
  if (d <= 2048) return 8;
  if (d <= 4096) return 16;
  return 0;
}

std::vector<at::Tensor> layernorm_fwd(const at::Tensor& x, const at::Tensor& gamma,
                                      const at::Tensor& beta, double eps) {
  MT_CHECK_CUDA(x);
  MT_CHECK(x.scalar_type() == at::kBFloat16, "layernorm_fwd: x must be bf16");
  MT_CHECK(gamma.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat,
           "layernorm_fwd: gamma/beta must be fp32");
  MT_CHECK_CONTIG(x);
  const int d = x.size(-1);
  const int rows = x.numel() / d;
  auto y = at::empty_like(x);
  auto opts = x.options().dtype(at::kFloat);
  auto mean = at::empty({rows}, opts), rstd = at::empty({rows}, opts);
  if (rows == 0) return {y, mean, rstd};
  const int nch = pick_nch(d);
  const auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* yp = reinterpret_cast<bf16*>(y.data_ptr());
  const bool aligned = (reinterpret_cast<uintptr_t>(xp) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(gamma.data_ptr()) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(beta.data_ptr()) % 16 == 0);
  const int wpb = 8;
  int grid = std::min((rows + wpb - 1) / wpb, num_sms() * 8);
  auto st = cur_stream();
#define LNF(N)                                                                              \
  ln_fwd_vec<N><<<grid, wpb * 32, 0, st>>>(xp, gamma.data_ptr<float>(), beta.data_ptr<float>(), \
                                           yp, mean.data_ptr<float>(), rstd.data_ptr<float>(), \
                                           rows, d, (float)eps)
  if (nch && aligned) {
    switch (nch) {
      case 1: LNF(1); break;
      case 2: LNF(2); break;
      case 4: LNF(4); break;
      case 8: LNF(8); break;
      case 16: LNF(16); break;
    }
  } else {
    ln_fwd_generic<<<(rows + 3) / 4, 128, 0, st>>>(xp, gamma.data_ptr<float>(),
                                                   beta.data_ptr<float>(), yp,
                                                   mean.data_ptr<float>(),
                                                   rstd.data_ptr<float>(), rows, d, (float)eps);
  }
#undef LNF
  MT_LAUNCH_CHECK();
  return {y, mean, rstd};
}

// Returns dx; writes (or accumulates into) dgamma/dbeta (fp32, length d).
at::Tensor layernorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& gamma,
                         const at::Tensor& mean, const at::Tensor& rstd, at::Tensor dgamma,
                         at::Tensor dbeta, bool accumulate) {
  MT_CHECK_CONTIG(dy);
  MT_CHECK_CONTIG(x);
  MT_CHECK(dy.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16,
           "layernorm_bwd: bf16 expected");
  const int d = x.size(-1);
  const int rows = x.numel() / d;
  auto dx = at::empty_like(x);
  if (rows == 0) return dx;
  const int nch = pick_nch(d);
  auto st = cur_stream();
  const int wpb = 4;
  const bool aligned = (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(dy.data_ptr()) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(gamma.data_ptr()) % 16 == 0);
  const size_t smem = (size_t)wpb * 2 * d * sizeof(float);
  int grid = std::min((rows + wpb - 1) / wpb, num_sms() * (smem <= 64 * 1024 ? 3 : 1));
  auto part = at::empty({grid, 2, d}, x.options().dtype(at::kFloat));
  const auto* dyp = reinterpret_cast<const bf16*>(dy.data_ptr());
  const auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* dxp = reinterpret_cast<bf16*>(dx.data_ptr());
#define LNB(N)                                                                                \
  do {                                                                                        \
    cudaFuncSetAttribute(ln_bwd_vec<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    ln_bwd_vec<N><<<grid, wpb * 32, smem, st>>>(dyp, xp, gamma.data_ptr<float>(),             \
                                                mean.data_ptr<float>(), rstd.data_ptr<float>(), \
                                                dxp, part.data_ptr<float>(), rows, d);        \
  } while (0)
  if (nch && aligned && smem <= 200 * 1024) {
    switch (nch) {
      case 1: LNB(1); break;
      case 2: LNB(2); break;
      case 4: LNB(4); break;
      case 8: LNB(8); break;
      case 16: LNB(16); break;
    }
  } else {
    part.zero_();
    ln_bwd_generic<<<grid, wpb * 32, 0, st>>>(dyp, xp, gamma.data_ptr<float>(),
                                              mean.data_ptr<float>(), rstd.data_ptr<float>(), dxp,
                                              part.data_ptr<float>(), rows, d);
  }
#undef LNB
  MT_LAUNCH_CHECK();
  ln_bwd_finish<<<(2 * d + 255) / 256, 256, 0, st>>>(part.data_ptr<float>(),
                                                      dgamma.data_ptr<float>(),
                                                      dbeta.data_ptr<float>(), grid, d,
                                                      accumulate ? 1 : 0);
  MT_LAUNCH_CHECK();
  return dx;
}

}  // namespace mtorus

// ---------------------------------------------------------------------------
// Allocation-free variant of layernorm_bwd for callers that cannot allocate
// device memory (declared in layernorm_noalloc.h, which describes the limits).
// It launches the same ln_bwd_vec / ln_bwd_finish kernels with their partial-sum
// scratch in a file-scope device array instead of a torch allocation.
#include <mutex>

#include "layernorm_noalloc.h"

namespace mtorus {
namespace {

constexpr int kNoAllocMaxDevices = 64;
constexpr size_t kNoAllocFloats =
    (size_t)MTORUS_LN_NOALLOC_MAX_BLOCKS * 2 * MTORUS_LN_NOALLOC_MAX_D;

static __device__ __align__(256) float g_ln_noalloc_scratch[kNoAllocFloats];

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Once per device, with that device current: the device address of the array
// (the host-side name g_ln_noalloc_scratch is only a stand-in, not a device
// address) and the shared-memory opt-in of the kernels it launches.
float* noalloc_setup(int dev) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev]) return g_noalloc_ptr[dev];
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_ln_noalloc_scratch) != cudaSuccess || p == nullptr) return nullptr;
  const int smem = 4 * 2 * MTORUS_LN_NOALLOC_MAX_D * (int)sizeof(float);
  if (cudaFuncSetAttribute(ln_bwd_vec<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(ln_bwd_vec<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(ln_bwd_vec<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(ln_bwd_vec<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(ln_bwd_vec<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return nullptr;
  g_noalloc_ptr[dev] = static_cast<float*>(p);
  return g_noalloc_ptr[dev];
}

}  // namespace
}  // namespace mtorus

extern "C" int mtorus_layernorm_bwd_noalloc(const uint16_t* dy, const uint16_t* x,
                                            const float* gamma, const float* mean,
                                            const float* rstd, uint16_t* dx, float* dgamma,
                                            float* dbeta, int rows, int d, int accumulate,
                                            cudaStream_t stream) {
  using namespace mtorus;
  if (!dy || !x || !gamma || !mean || !rstd || !dx || !dgamma || !dbeta || rows <= 0 || d <= 0 ||
      d % 8 != 0)
    return MTORUS_NOALLOC_EARG;
  for (const void* p : {(const void*)dy, (const void*)x, (const void*)gamma, (const void*)dx})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return MTORUS_NOALLOC_EARG;
  if (d > MTORUS_LN_NOALLOC_MAX_D) return MTORUS_NOALLOC_ESIZE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
    return MTORUS_NOALLOC_ESETUP;
  float* part = noalloc_setup(dev);
  if (!part) return MTORUS_NOALLOC_ESETUP;
  const int nch = pick_nch(d);
  const int wpb = 4;
  const size_t smem = (size_t)wpb * 2 * d * sizeof(float);
  const int grid = std::min((rows + wpb - 1) / wpb, MTORUS_LN_NOALLOC_MAX_BLOCKS);
  const auto* dyp = reinterpret_cast<const bf16*>(dy);
  const auto* xp = reinterpret_cast<const bf16*>(x);
  auto* dxp = reinterpret_cast<bf16*>(dx);
  switch (nch) {
    case 1: ln_bwd_vec<1><<<grid, wpb * 32, smem, stream>>>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d); break;
    case 2: ln_bwd_vec<2><<<grid, wpb * 32, smem, stream>>>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d); break;
    case 4: ln_bwd_vec<4><<<grid, wpb * 32, smem, stream>>>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d); break;
    case 8: ln_bwd_vec<8><<<grid, wpb * 32, smem, stream>>>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d); break;
    case 16: ln_bwd_vec<16><<<grid, wpb * 32, smem, stream>>>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d); break;
    default: return MTORUS_NOALLOC_ESIZE;
  }
  if (cudaGetLastError() != cudaSuccess) return MTORUS_NOALLOC_ELAUNCH;
  ln_bwd_finish<<<(2 * d + 255) / 256, 256, 0, stream>>>(part, dgamma, dbeta, grid, d,
                                                         accumulate ? 1 : 0);
  if (cudaGetLastError() != cudaSuccess) return MTORUS_NOALLOC_ELAUNCH;
  return MTORUS_NOALLOC_OK;
}
