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
#include <cstring>

#include "amax_publish.cuh"
#include "mx.cuh"

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

// ---------------------------------------------------------------------------
// Block-per-row kernels: one CTA of d/8 threads (8 columns per thread) walks a
// strided set of rows, so each thread holds only 8 values of a row, and the
// dgamma/dbeta partial sums of its 8 columns stay in registers across rows.
// Row reductions use a parity-double-buffered shared array: one __syncthreads
// per reduction.

__device__ __forceinline__ float2 block_sum2(float a, float b, float (*red)[32], int par) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  if (lane == 0) {
    red[par * 2][wid] = a;
    red[par * 2 + 1][wid] = b;
  }
  __syncthreads();
  float ta = 0.f, tb = 0.f;
  for (int w = 0; w < nw; ++w) {
    ta += red[par * 2][w];
    tb += red[par * 2 + 1][w];
  }
  return make_float2(ta, tb);
}

__global__ void __launch_bounds__(1024) ln_fwd_row(const bf16* __restrict__ x,
                                                   const float* __restrict__ gamma,
                                                   const float* __restrict__ beta,
                                                   bf16* __restrict__ y, float* __restrict__ mean_out,
                                                   float* __restrict__ rstd_out, int rows, int d,
                                                   float eps) {
  __shared__ float red[4][32];
  const int col = threadIdx.x * 8;
  float g[8], b[8];
  {
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + col);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
    const float4 b0 = *reinterpret_cast<const float4*>(beta + col);
    const float4 b1 = *reinterpret_cast<const float4*>(beta + col + 4);
    g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w; g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
    b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
  }
  int par = 0;
  bf16x8 nxt;
  if (blockIdx.x < rows) nxt = *reinterpret_cast<const bf16x8*>(x + (size_t)blockIdx.x * d + col);
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    float v[8];
    unpack8(nxt, v);
    if (row + gridDim.x < rows)  // prefetch the next row while this one is reduced
      nxt = *reinterpret_cast<const bf16x8*>(x + (size_t)(row + gridDim.x) * d + col);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[i];
    const float mean = block_sum2(s, 0.f, red, par).x / d;
    par ^= 1;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float t = v[i] - mean;
      q += t * t;
    }
    const float rstd = rsqrtf(block_sum2(q, 0.f, red, par).x / d + eps);
    par ^= 1;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (v[i] - mean) * rstd * g[i] + b[i];
    *reinterpret_cast<bf16x8*>(y + (size_t)row * d + col) = pack8(o);
    if (threadIdx.x == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

// LayerNorm whose output goes straight to FP8 codes (the input of the next FP8
// GEMM): y = LN(x) is rounded to bf16 as in the bf16 path, multiplied by the tensor
// role's delayed scale and stored as E4M3 / E5M2; max|y| folds into the role's amax
// (and, with a counter, is published to the data-parallel peers).  Saves the bf16
// write of y and the separate quantise pass that would read it back.
template <int FMT>
__global__ void __launch_bounds__(1024) ln_fwd_row_fp8(const bf16* __restrict__ x,
                                                       const float* __restrict__ gamma,
                                                       const float* __restrict__ beta,
                                                       uint8_t* __restrict__ y8, float* __restrict__ mean_out,
                                                       float* __restrict__ rstd_out, int rows, int d, float eps,
                                                       const float* __restrict__ scale, float* __restrict__ amax,
                                                       unsigned int* counter, AmaxPeers table, int me, int world,
                                                       int cap, int slot, int parity, unsigned int epoch) {
  __shared__ float red[4][32];
  __shared__ float redm[32];
  __shared__ bool last;
  const int col = threadIdx.x * 8;
  const float sc = *scale;
  float g[8], b[8];
  {
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + col);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
    const float4 b0 = *reinterpret_cast<const float4*>(beta + col);
    const float4 b1 = *reinterpret_cast<const float4*>(beta + col + 4);
    g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w; g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
    b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
  }
  float m = 0.f;
  int par = 0;
  bf16x8 nxt;
  if (blockIdx.x < rows) nxt = *reinterpret_cast<const bf16x8*>(x + (size_t)blockIdx.x * d + col);
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    float v[8];
    unpack8(nxt, v);
    if (row + gridDim.x < rows)
      nxt = *reinterpret_cast<const bf16x8*>(x + (size_t)(row + gridDim.x) * d + col);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[i];
    const float mean = block_sum2(s, 0.f, red, par).x / d;
    par ^= 1;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float t = v[i] - mean;
      q += t * t;
    }
    const float rstd = rsqrtf(block_sum2(q, 0.f, red, par).x / d + eps);
    par ^= 1;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (v[i] - mean) * rstd * g[i] + b[i];
    float r[8];
    unpack8(pack8(o), r);  // the bf16 value the unfused path would quantise
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
#pragma unroll
      for (int j = 0; j < 4; ++j) m = fmaxf(m, fabsf(r[4 * k + j]));
      const uint16_t lo = FMT == 0 ? cvt2_e4m3(r[4 * k] * sc, r[4 * k + 1] * sc)
                                   : cvt2_e5m2(r[4 * k] * sc, r[4 * k + 1] * sc);
      const uint16_t hi = FMT == 0 ? cvt2_e4m3(r[4 * k + 2] * sc, r[4 * k + 3] * sc)
                                   : cvt2_e5m2(r[4 * k + 2] * sc, r[4 * k + 3] * sc);
      w[k] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint2*>(y8 + (size_t)row * d + col) = make_uint2(w[0], w[1]);
    if (threadIdx.x == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
  m = block_max(m, redm);
  publish_amax(m, amax, counter, table, me, world, cap, slot, parity, epoch, &last);
}

// dx = LN backward (+ dres, the gradient of a residual branch that reads x);
// part[block][0][:] / part[block][1][:] = this block's dgamma / dbeta sums.
__global__ void __launch_bounds__(1024) ln_bwd_row(const bf16* __restrict__ dy,
                                                   const bf16* __restrict__ x,
                                                   const float* __restrict__ gamma,
                                                   const float* __restrict__ mean_in,
                                                   const float* __restrict__ rstd_in,
                                                   const bf16* __restrict__ dres,
                                                   bf16* __restrict__ dx, float* __restrict__ part,
                                                   int rows, int d) {
  __shared__ float red[4][32];
  const int col = threadIdx.x * 8;
  float gm[8], dg[8], db[8];
  {
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + col);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + col + 4);
    gm[0] = g0.x; gm[1] = g0.y; gm[2] = g0.z; gm[3] = g0.w; gm[4] = g1.x; gm[5] = g1.y; gm[6] = g1.z; gm[7] = g1.w;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) dg[i] = db[i] = 0.f;
  int par = 0;
  bf16x8 nx, ndy;
  if (blockIdx.x < rows) {
    nx = *reinterpret_cast<const bf16x8*>(x + (size_t)blockIdx.x * d + col);
    ndy = *reinterpret_cast<const bf16x8*>(dy + (size_t)blockIdx.x * d + col);
  }
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    float xv[8], dv[8];
    unpack8(nx, xv);
    unpack8(ndy, dv);
    const int nrow = row + gridDim.x;
    if (nrow < rows) {
      nx = *reinterpret_cast<const bf16x8*>(x + (size_t)nrow * d + col);
      ndy = *reinterpret_cast<const bf16x8*>(dy + (size_t)nrow * d + col);
    }
    const float mean = mean_in[row], rstd = rstd_in[row];
    float xh[8], g[8], s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xh[i] = (xv[i] - mean) * rstd;
      g[i] = dv[i] * gm[i];
      s1 += g[i];
      s2 += g[i] * xh[i];
      dg[i] += dv[i] * xh[i];
      db[i] += dv[i];
    }
    const float2 s = block_sum2(s1, s2, red, par);
    par ^= 1;
    const float c2 = s.x / d, c1 = s.y / d;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (g[i] - xh[i] * c1 - c2) * rstd;
    if (dres) {
      float r8[8];
      unpack8(*reinterpret_cast<const bf16x8*>(dres + (size_t)row * d + col), r8);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += r8[i];
    }
    *reinterpret_cast<bf16x8*>(dx + (size_t)row * d + col) = pack8(o);
  }
  float* out = part + (size_t)blockIdx.x * 2 * d + col;
  *reinterpret_cast<float4*>(out) = make_float4(dg[0], dg[1], dg[2], dg[3]);
  *reinterpret_cast<float4*>(out + 4) = make_float4(dg[4], dg[5], dg[6], dg[7]);
  *reinterpret_cast<float4*>(out + d) = make_float4(db[0], db[1], db[2], db[3]);
  *reinterpret_cast<float4*>(out + d + 4) = make_float4(db[4], db[5], db[6], db[7]);
}

// out[c] (+)= sum_r part[r * ld + c], c < ncols (fp32 column sums of the partials).
__global__ void __launch_bounds__(256) colsum_f32_kernel(const float* __restrict__ part, int nrows,
                                                         int ncols, int ld, float* __restrict__ out,
                                                         int rows_per_block) {
  __shared__ float red[8][257];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 256 + tx * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(nrows, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (c0 < ncols) {
    for (int r = r0 + ty; r < r1; r += 8) {
      const float4 a = *reinterpret_cast<const float4*>(part + (size_t)r * ld + c0);
      const float4 b = *reinterpret_cast<const float4*>(part + (size_t)r * ld + c0 + 4);
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) red[ty][tx * 8 + k] = acc[k];
  __syncthreads();
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < ncols) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][threadIdx.x];
    atomicAdd(out + c, t);
  }
}

static void colsum_f32(const float* part, int nrows, int ncols, int ld, float* out, cudaStream_t st) {
  const int rpb = 32;
  dim3 grid((ncols + 255) / 256, (nrows + rpb - 1) / rpb);
  colsum_f32_kernel<<<grid, 256, 0, st>>>(part, nrows, ncols, ld, out, rpb);
  MT_LAUNCH_CHECK();
}

static bool row_kernel_ok(int d, const void* a, const void* b, const void* c) {
  return d % 8 == 0 && d / 8 <= 1024 && d / 8 >= 32 && (d / 8) % 32 == 0 &&
         reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(c) % 16 == 0;
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

// LayerNorm straight to FP8 codes (see ln_fwd_row_fp8) -> (mean, rstd); y8 is the
// uint8 [rows, d] output.  table_ptrs empty: local amax only.
std::vector<at::Tensor> layernorm_fwd_fp8(const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta,
                                          double eps, at::Tensor y8, const at::Tensor& scale, at::Tensor amax,
                                          int64_t fmt, const c10::optional<at::Tensor>& counter,
                                          const std::vector<int64_t>& table_ptrs, int64_t me, int64_t cap,
                                          int64_t slot, int64_t parity, int64_t epoch, int64_t ep_ptr) {
  MT_CHECK_CUDA(x);
  MT_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "layernorm_fwd_fp8: contiguous bf16 x");
  MT_CHECK(gamma.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat, "layernorm_fwd_fp8: fp32 params");
  const int d = x.size(-1);
  const int rows = x.numel() / d;
  MT_CHECK(y8.element_size() == 1 && y8.numel() == x.numel() && y8.is_contiguous(), "layernorm_fwd_fp8: y8");
  const auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  MT_CHECK(row_kernel_ok(d, xp, gamma.data_ptr(), beta.data_ptr()) &&
               reinterpret_cast<uintptr_t>(y8.data_ptr()) % 16 == 0,
           "layernorm_fwd_fp8: d must be a multiple of 8 up to 8192 with aligned buffers");
  auto opts = x.options().dtype(at::kFloat);
  auto mean = at::empty({rows}, opts), rstd = at::empty({rows}, opts);
  if (rows == 0) return {mean, rstd};
  const int world = (int)table_ptrs.size();
  MT_CHECK(world <= kAmaxMaxPeers && (world == 0 || counter.has_value()), "layernorm_fwd_fp8: peers");
  AmaxPeers t{};
  for (int i = 0; i < world; ++i) t.p[i] = (uint64_t)table_ptrs[i];
  t.ep = reinterpret_cast<const unsigned int*>(ep_ptr);
  unsigned int* cp = world ? reinterpret_cast<unsigned int*>(counter->data_ptr()) : nullptr;
  const int threads = d / 8;
  const int grid = std::min(rows, num_sms() * std::max(1, 2048 / threads));
  auto* yp = reinterpret_cast<uint8_t*>(y8.data_ptr());
  if (fmt == 0)
    ln_fwd_row_fp8<0><<<grid, threads, 0, cur_stream()>>>(
        xp, gamma.data_ptr<float>(), beta.data_ptr<float>(), yp, mean.data_ptr<float>(), rstd.data_ptr<float>(),
        rows, d, (float)eps, scale.data_ptr<float>(), amax.data_ptr<float>(), cp, t, (int)me, world, (int)cap,
        (int)slot, (int)parity, (unsigned int)epoch);
  else
    ln_fwd_row_fp8<1><<<grid, threads, 0, cur_stream()>>>(
        xp, gamma.data_ptr<float>(), beta.data_ptr<float>(), yp, mean.data_ptr<float>(), rstd.data_ptr<float>(),
        rows, d, (float)eps, scale.data_ptr<float>(), amax.data_ptr<float>(), cp, t, (int)me, world, (int)cap,
        (int)slot, (int)parity, (unsigned int)epoch);
  MT_LAUNCH_CHECK();
  return {mean, rstd};
}

// LayerNorm straight to MXFP8, row-wise and column-wise (the operands of the
// forward GEMM and of the wgrad GEMM under the MX recipe); the bf16 output itself
// is never written.  Two launches: ln_row_stats (one warp per row: sum, then the
// centred sum of squares, fp32, over a second, cache-resident read of the row)
// writes mean / rstd, which the backward needs anyway; then the 128 x 128 tile
// quantiser (mx_rc_tile_kernel in fp8.cu) normalises each tile on load and
// quantises it along its rows and down its columns.
__global__ void __launch_bounds__(256) ln_row_stats_kernel(const bf16* __restrict__ x, float* __restrict__ mean_out,
                                                           float* __restrict__ rstd_out, int R, int d, float eps) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= R) return;
  const bf16* row = x + (int64_t)warp * d;
  float s = 0.f;
  for (int c = lane * 8; c < d; c += 256) {
    float f[8];
    unpack8(*reinterpret_cast<const bf16x8*>(row + c), f);
#pragma unroll
    for (int k = 0; k < 8; ++k) s += f[k];
  }
  s = warp_sum(s);
  const float mu = s / (float)d;
  float q = 0.f;
  for (int c = lane * 8; c < d; c += 256) {
    float f[8];
    unpack8(*reinterpret_cast<const bf16x8*>(row + c), f);
#pragma unroll
    for (int k = 0; k < 8; ++k) q += (f[k] - mu) * (f[k] - mu);
  }
  q = warp_sum(q);
  if (lane == 0) {
    mean_out[warp] = mu;
    rstd_out[warp] = rsqrtf(q / (float)d + eps);
  }
}

// x bf16 [R, d] contiguous (R % 32 == 0, d % 256 == 0, d <= 2048) -> row codes rc [R, d] +
// rsf, column codes cc [d, R] + csf (scale atoms as mx_quantize_rc), mean / rstd [R].
void mx_rc_tiles(const bf16* x, int64_t ldx, int64_t R, int64_t C, int64_t fmt, double fmax, const float* ln_mean,
                 const float* ln_rstd, const float* ln_gamma, const float* ln_beta, float* colsum, uint8_t* rc,
                 uint8_t* rsf, uint8_t* cc, uint8_t* csf, cudaStream_t st, const float* xq, int64_t ldq,
                 int64_t qcols, int act, const bf16* aux, int64_t ldaux);

void layernorm_fwd_mx_rc(const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta, double eps,
                         at::Tensor rc, at::Tensor rsf, at::Tensor cc, at::Tensor csf, at::Tensor mean,
                         at::Tensor rstd, int64_t fmt, double fmax) {
  MT_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(), "ln_mx: contiguous bf16 [R, d]");
  const int64_t R = x.size(0), d = x.size(1);
  MT_CHECK(R % 32 == 0 && d % 32 == 0, "ln_mx: R and d multiples of 32");
  MT_CHECK(gamma.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat && gamma.numel() == d &&
               beta.numel() == d && reinterpret_cast<uintptr_t>(gamma.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(beta.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
           "ln_mx: fp32 gamma / beta [d], 16-byte aligned");
  auto chk = [](const at::Tensor& t, int64_t n, const char* what) {
    MT_CHECK(t.element_size() == 1 && t.is_contiguous() && t.numel() == n &&
                 reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
             what);
  };
  chk(rc, R * d, "ln_mx: rc must be 16-byte aligned contiguous uint8 [R, d]");
  chk(cc, R * d, "ln_mx: cc must be 16-byte aligned contiguous uint8 [d, R]");
  chk(rsf, (R + 127) / 128 * ((d + 127) / 128) * 512, "ln_mx: rsf size");
  chk(csf, (d + 127) / 128 * ((R + 127) / 128) * 512, "ln_mx: csf size");
  MT_CHECK(mean.scalar_type() == at::kFloat && rstd.scalar_type() == at::kFloat && mean.numel() == R &&
               rstd.numel() == R,
           "ln_mx: fp32 mean / rstd [R]");
  MT_CHECK((fmt == 0 || fmt == 1) && fmax > 0.0, "ln_mx: fmt 0 / 1, fmax > 0");
  if (R == 0) return;
  auto st = cur_stream();
  ln_row_stats_kernel<<<(unsigned)((R + 7) / 8), 256, 0, st>>>(reinterpret_cast<const bf16*>(x.data_ptr()),
                                                               mean.data_ptr<float>(), rstd.data_ptr<float>(),
                                                               (int)R, (int)d, (float)eps);
  MT_LAUNCH_CHECK();
  mx_rc_tiles(reinterpret_cast<const bf16*>(x.data_ptr()), d, R, d, fmt, fmax, mean.data_ptr<float>(),
              rstd.data_ptr<float>(), gamma.data_ptr<float>(), beta.data_ptr<float>(), nullptr,
              reinterpret_cast<uint8_t*>(rc.data_ptr()), reinterpret_cast<uint8_t*>(rsf.data_ptr()),
              reinterpret_cast<uint8_t*>(cc.data_ptr()), reinterpret_cast<uint8_t*>(csf.data_ptr()), st, nullptr, 0,
              0, 0, nullptr, 0);
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
  auto st = cur_stream();
  if (row_kernel_ok(d, xp, gamma.data_ptr(), beta.data_ptr())) {
    const int threads = d / 8;
    const int grid = std::min(rows, num_sms() * std::max(1, 2048 / threads));
    ln_fwd_row<<<grid, threads, 0, st>>>(xp, gamma.data_ptr<float>(), beta.data_ptr<float>(), yp,
                                         mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, d,
                                         (float)eps);
    MT_LAUNCH_CHECK();
    return {y, mean, rstd};
  }
  const int wpb = 8;
  int grid = std::min((rows + wpb - 1) / wpb, num_sms() * 8);
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
                         at::Tensor dbeta, bool accumulate, const c10::optional<at::Tensor>& dres) {
  MT_CHECK_CONTIG(dy);
  MT_CHECK_CONTIG(x);
  MT_CHECK(dy.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16,
           "layernorm_bwd: bf16 expected");
  const int d = x.size(-1);
  const int rows = x.numel() / d;
  auto dx = at::empty_like(x);
  if (rows == 0) return dx;
  auto st = cur_stream();
  if (dres.has_value()) {
    MT_CHECK(dres->is_contiguous() && dres->scalar_type() == at::kBFloat16 && dres->numel() == x.numel(),
             "layernorm_bwd: dres must be a contiguous bf16 tensor shaped like x");
  }
  if (row_kernel_ok(d, x.data_ptr(), dy.data_ptr(), gamma.data_ptr()) &&
      (!dres.has_value() || reinterpret_cast<uintptr_t>(dres->data_ptr()) % 16 == 0)) {
    const int threads = d / 8;
    const int grid = std::min(rows, num_sms() * std::max(1, 2048 / threads));
    auto part = at::empty({grid, 2, d}, x.options().dtype(at::kFloat));
    ln_bwd_row<<<grid, threads, 0, st>>>(
        reinterpret_cast<const bf16*>(dy.data_ptr()), reinterpret_cast<const bf16*>(x.data_ptr()),
        gamma.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
        dres.has_value() ? reinterpret_cast<const bf16*>(dres->data_ptr()) : nullptr,
        reinterpret_cast<bf16*>(dx.data_ptr()), part.data_ptr<float>(), rows, d);
    MT_LAUNCH_CHECK();
    float* dg = dgamma.data_ptr<float>();
    float* dbp = dbeta.data_ptr<float>();
    if (!accumulate) {
      C10_CUDA_CHECK(cudaMemsetAsync(dg, 0, d * sizeof(float), st));
      C10_CUDA_CHECK(cudaMemsetAsync(dbp, 0, d * sizeof(float), st));
    }
    if (dbp == dg + d) {
      colsum_f32(part.data_ptr<float>(), grid, 2 * d, 2 * d, dg, st);
    } else {
      colsum_f32(part.data_ptr<float>(), grid, d, 2 * d, dg, st);
      colsum_f32(part.data_ptr<float>() + d, grid, d, 2 * d, dbp, st);
    }
    return dx;
  }
  MT_CHECK(!dres.has_value(), "layernorm_bwd: dres needs d % 256 == 0 and 16-byte aligned tensors");
  const int nch = pick_nch(d);
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
// address).
float* noalloc_setup(int dev) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev]) return g_noalloc_ptr[dev];
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_ln_noalloc_scratch) != cudaSuccess || p == nullptr) return nullptr;
  g_noalloc_ptr[dev] = static_cast<float*>(p);
  return g_noalloc_ptr[dev];
}

// The dynamic shared-memory limit is a per-function attribute that other code
// (the torch-facing layernorm_bwd sets it to each call's own size) may have
// lowered since the last call, so every call raises it for the kernel it is about
// to launch.  Setting an attribute allocates nothing.
template <int N>
int noalloc_launch_vec(const bf16* dyp, const bf16* xp, const float* gamma, const float* mean,
                       const float* rstd, bf16* dxp, float* part, int rows, int d, int grid,
                       int wpb, size_t smem, cudaStream_t stream) {
  if (cudaFuncSetAttribute(ln_bwd_vec<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess) {
    (void)cudaGetLastError();  // the failed call's own (non-sticky) error
    return MTORUS_NOALLOC_ESETUP;
  }
  ln_bwd_vec<N><<<grid, wpb * 32, smem, stream>>>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d);
  return cudaGetLastError() == cudaSuccess ? MTORUS_NOALLOC_OK : MTORUS_NOALLOC_ELAUNCH;
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
  // An error left pending by earlier work belongs to the caller: report it without
  // launching, and leave it in place for whoever owns it.
  if (cudaPeekAtLastError() != cudaSuccess) return MTORUS_NOALLOC_EPENDING;
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
  int rc;
  switch (nch) {
    case 1: rc = noalloc_launch_vec<1>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d, grid, wpb, smem, stream); break;
    case 2: rc = noalloc_launch_vec<2>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d, grid, wpb, smem, stream); break;
    case 4: rc = noalloc_launch_vec<4>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d, grid, wpb, smem, stream); break;
    case 8: rc = noalloc_launch_vec<8>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d, grid, wpb, smem, stream); break;
    case 16: rc = noalloc_launch_vec<16>(dyp, xp, gamma, mean, rstd, dxp, part, rows, d, grid, wpb, smem, stream); break;
    default: return MTORUS_NOALLOC_ESIZE;
  }
  if (rc != MTORUS_NOALLOC_OK) return rc;
  ln_bwd_finish<<<(2 * d + 255) / 256, 256, 0, stream>>>(part, dgamma, dbeta, grid, d,
                                                         accumulate ? 1 : 0);
  if (cudaGetLastError() != cudaSuccess) return MTORUS_NOALLOC_ELAUNCH;
  return MTORUS_NOALLOC_OK;
}
