// Embedding gather/scatter and bias+GELU kernels for the GPT blocks.
//
// Reference semantics:
//   * token + learned position embedding: x = wte[ids] + wpe[pos]
//     (examples/gpt-1b/src/model.rs:113-118)
//   * FFN activation: GELU, erf form (examples/gpt-1b/src/transformer.rs:107)
//
// Design (B200): 16-byte vectors; the embedding backward scatters token rows
// straight into the fp32 master-gradient buffer with vectorised fp32 atomics
// (red.global.add.v4.f32) and sums position rows over the batch without atomics.
#include "common.cuh"

#include <cuda_fp16.h>
#include "gelu.cuh"
#include "philox.cuh"

namespace mtorus {

// x[t, :] = wte[ids[t], :] + wpe[t % S, :]   (bf16 tables, bf16 output)
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ wte,
                                 const bf16* __restrict__ wpe, bf16* __restrict__ out, int T,
                                 int S, int d, int V, DropoutArgs drop) {
  const uint32_t k0 = drop.rng ? drop.rng[0] : 0u, k1 = drop.rng ? drop.rng[1] : 0u;
  const int nv = d / 8;
  const size_t total = (size_t)T * nv;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int t = i / nv, c = i % nv;
    int64_t id = ids[t];
    id = id < 0 ? 0 : (id >= V ? V - 1 : id);
    float a[8], b[8];
    unpack8(reinterpret_cast<const bf16x8*>(wte + (size_t)id * d)[c], a);
    unpack8(reinterpret_cast<const bf16x8*>(wpe + (size_t)(t % S) * d)[c], b);
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] += b[k];
    if (drop.rng) {  // embedding dropout (element t * d + 8c + k; its 8-group is (t * d) / 8 + c)
      const uint32_t keep = dropout_keep8(k0, k1, drop.site, (uint64_t)t * (d / 8) + c, drop.thr16);
#pragma unroll
      for (int k = 0; k < 8; ++k) a[k] = (keep >> k & 1u) ? a[k] * drop.scale : 0.f;
    }
    reinterpret_cast<bf16x8*>(out + (size_t)t * d)[c] = pack8(a);
  }
}

// out = x * keep * scale over the site's mask (the backward of a dropout: the same
// mask applied to the incoming gradient); out may alias x.  n a multiple of 8.
__global__ void dropout_apply_kernel(const bf16* __restrict__ x, bf16* __restrict__ out, size_t n8,
                                     DropoutArgs drop) {
  const uint32_t k0 = drop.rng[0], k1 = drop.rng[1];
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    float a[8];
    unpack8(reinterpret_cast<const bf16x8*>(x)[i], a);
    const uint32_t keep = dropout_keep8(k0, k1, drop.site, i, drop.thr16);
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = (keep >> k & 1u) ? a[k] * drop.scale : 0.f;
    reinterpret_cast<bf16x8*>(out)[i] = pack8(a);
  }
}

// rng = {key lo, key hi, step lo, step hi}: step += 1, key = SplitMix64 finaliser
// (G. L. Steele, D. Lea, C. H. Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014) of base * golden-ratio increment + step + 1.
__global__ void dropout_advance_kernel(int32_t* rng, uint64_t base) {
  if (threadIdx.x || blockIdx.x) return;
  const uint64_t step = ((uint64_t)(uint32_t)rng[2] | ((uint64_t)(uint32_t)rng[3] << 32)) + 1;
  uint64_t z = base * 0x9E3779B97F4A7C15ull + step + 1;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  rng[0] = (int32_t)(uint32_t)z;
  rng[1] = (int32_t)(uint32_t)(z >> 32);
  rng[2] = (int32_t)(uint32_t)step;
  rng[3] = (int32_t)(uint32_t)(step >> 32);
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// dwte[ids[t], :] += dy[t, :]
__global__ void embed_bwd_tok_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ dy,
                                     float* __restrict__ dwte, int T, int d, int V) {
  const int nv = d / 8;
  const size_t total = (size_t)T * nv;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int t = i / nv, c = i % nv;
    int64_t id = ids[t];
    id = id < 0 ? 0 : (id >= V ? V - 1 : id);
    float g[8];
    unpack8(reinterpret_cast<const bf16x8*>(dy + (size_t)t * d)[c], g);
    float* dst = dwte + (size_t)id * d + c * 8;
    red_add_v4(dst, g[0], g[1], g[2], g[3]);
    red_add_v4(dst + 4, g[4], g[5], g[6], g[7]);
  }
}

// dwpe[s, :] (+)= sum_b dy[b*S + s, :]
__global__ void embed_bwd_pos_kernel(const bf16* __restrict__ dy, float* __restrict__ dwpe, int B,
                                     int S, int d, int accumulate) {
  const size_t total = (size_t)S * d;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int s = i / d, c = i % d;
    float acc = 0.f;
    for (int b = 0; b < B; ++b) acc += __bfloat162float(dy[((size_t)b * S + s) * d + c]);
    dwpe[i] = accumulate ? dwpe[i] + acc : acc;
  }
}

__device__ __forceinline__ float gelu_erf(float x) { return gelu_fwd(x); }
__device__ __forceinline__ float gelu_erf_grad(float x) { return gelu_grad(x); }

// pre[t, j] += bias[j] (in place, optional); act = gelu(pre)
__global__ void bias_gelu_fwd_kernel(bf16* __restrict__ pre, const float* __restrict__ bias,
                                     bf16* __restrict__ act, size_t rows, int F) {
  const int nv = F / 8;
  const size_t total = rows * nv;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = i % nv;
    float x[8], y[8];
    unpack8(reinterpret_cast<const bf16x8*>(pre)[i], x);
    if (bias) {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] += bias[c * 8 + k];
      reinterpret_cast<bf16x8*>(pre)[i] = pack8(x);
      // use the rounded pre-activation so backward sees the same value
      unpack8(reinterpret_cast<const bf16x8*>(pre)[i], x);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) y[k] = gelu_erf(x[k]);
    reinterpret_cast<bf16x8*>(act)[i] = pack8(y);
  }
}

// dpre = dact * gelu'(pre)   (written in place over dact)
__global__ void gelu_bwd_kernel(bf16* __restrict__ dact, const bf16* __restrict__ pre, size_t n8) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8;
       i += (size_t)gridDim.x * blockDim.x) {
    float g[8], x[8];
    unpack8(reinterpret_cast<const bf16x8*>(dact)[i], g);
    unpack8(reinterpret_cast<const bf16x8*>(pre)[i], x);
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] *= gelu_erf_grad(x[k]);
    reinterpret_cast<bf16x8*>(dact)[i] = pack8(g);
  }
}

// Column sums of a [rows, F] bf16 matrix into fp32 (bias gradients), (+)= into out.
// Block = 32 column groups of 8 (16-byte loads, 512 contiguous bytes per warp per
// row) x 8 row lanes; each block reduces its row slice in registers, then across
// row lanes in shared memory, and adds into out with one atomic per column.
__global__ void __launch_bounds__(256) colsum_vec_kernel(const bf16* __restrict__ x,
                                                         float* __restrict__ out, const float* scale,
                                                         int rows, int F, int rows_per_block) {
  __shared__ float red[8][257];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 256 + tx * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (c0 < F) {
    for (int r = r0 + ty; r < r1; r += 8) {
      float f[8];
      unpack8(*reinterpret_cast<const bf16x8*>(x + (size_t)r * F + c0), f);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += f[k];
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) red[ty][tx * 8 + k] = acc[k];
  __syncthreads();
  const int col = threadIdx.x;  // 256 columns of this block
  if (blockIdx.x * 256 + col < F) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][col];
    if (scale) t *= *scale;
    atomicAdd(out + blockIdx.x * 256 + col, t);
  }
}

// Column sums of E5M2 codes [rows, F] (F % 8 == 0): an E5M2 code is the high byte of the
// fp16 with the same value, so decoding is a shift.  out (+)= sum * (*scale) * (*scale2).
__global__ void __launch_bounds__(256) colsum_e5m2_kernel(const uint8_t* __restrict__ x, float* __restrict__ out,
                                                          const float* scale, const float* scale2, int rows, int F,
                                                          int rows_per_block) {
  __shared__ float red[8][257];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 256 + tx * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (c0 < F) {
    for (int r = r0 + ty; r < r1; r += 8) {
      const uint2 w = *reinterpret_cast<const uint2*>(x + (size_t)r * F + c0);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t code = ((k < 4 ? w.x : w.y) >> (8 * (k & 3))) & 0xFFu;
        acc[k] += __half2float(__ushort_as_half((unsigned short)(code << 8)));
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) red[ty][tx * 8 + k] = acc[k];
  __syncthreads();
  const int col = threadIdx.x;
  if (blockIdx.x * 256 + col < F) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][col];
    if (scale) t *= *scale;
    if (scale2) t *= *scale2;
    atomicAdd(out + blockIdx.x * 256 + col, t);
  }
}

// Generic fallback (F % 8 != 0).
__global__ void colsum_kernel(const bf16* __restrict__ x, float* __restrict__ out, const float* scale,
                              int rows, int F, int rows_per_block) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= F) return;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  float acc = 0.f;
  for (int r = r0; r < r1; ++r) acc += __bfloat162float(x[(size_t)r * F + c]);
  if (scale) acc *= *scale;
  atomicAdd(out + c, acc);
}

static int ew_grid(size_t n) {
  return (int)std::max<size_t>(1, std::min<size_t>((n + 255) / 256, (size_t)num_sms() * 16));
}

DropoutArgs make_dropout_args(const c10::optional<at::Tensor>& rng, int64_t site, int64_t thr16, double scale) {
  DropoutArgs a{};
  if (rng.has_value()) {
    MT_CHECK(rng->is_cuda() && rng->scalar_type() == at::kInt && rng->numel() >= 2, "dropout: int32 rng key on the GPU");
    MT_CHECK(thr16 >= 0 && thr16 < 65536 && scale >= 1.0, "dropout: 0 <= p < 1");
    a.rng = reinterpret_cast<const uint32_t*>(rng->data_ptr<int32_t>());
    a.site = (uint32_t)site;
    a.thr16 = (uint32_t)thr16;
    a.scale = (float)scale;
  }
  return a;
}

void dropout_apply(const at::Tensor& x, at::Tensor out, const at::Tensor& rng, int64_t site, int64_t thr16,
                   double scale) {
  MT_CHECK(x.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16 && x.is_contiguous() &&
               out.is_contiguous() && x.numel() == out.numel() && x.numel() % 8 == 0,
           "dropout_apply: contiguous bf16 of equal size, numel % 8 == 0");
  const size_t n8 = x.numel() / 8;
  if (n8 == 0) return;
  dropout_apply_kernel<<<ew_grid(n8), 256, 0, cur_stream()>>>(reinterpret_cast<const bf16*>(x.data_ptr()),
                                                              reinterpret_cast<bf16*>(out.data_ptr()), n8,
                                                              make_dropout_args(rng, site, thr16, scale));
  MT_LAUNCH_CHECK();
}

void dropout_advance(at::Tensor rng, int64_t base) {
  MT_CHECK(rng.is_cuda() && rng.scalar_type() == at::kInt && rng.numel() == 4, "dropout_advance: int32 [4] on the GPU");
  dropout_advance_kernel<<<1, 32, 0, cur_stream()>>>(rng.data_ptr<int32_t>(), (uint64_t)base);
  MT_LAUNCH_CHECK();
}

at::Tensor embed_fwd(const at::Tensor& ids, const at::Tensor& wte, const at::Tensor& wpe,
                     int64_t S, const c10::optional<at::Tensor>& drop_rng, int64_t drop_site, int64_t drop_thr16,
                     double drop_scale) {
  MT_CHECK(ids.scalar_type() == at::kLong, "embed: ids must be int64");
  MT_CHECK(wte.scalar_type() == at::kBFloat16 && wpe.scalar_type() == at::kBFloat16,
           "embed: bf16 tables");
  const int d = wte.size(1), V = wte.size(0);
  MT_CHECK(d % 8 == 0, "embed: d must be a multiple of 8");
  const int T = ids.numel();
  auto out = at::empty({T, d}, wte.options());
  if (T == 0) return out;
  embed_fwd_kernel<<<ew_grid((size_t)T * d / 8), 256, 0, cur_stream()>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const bf16*>(wte.data_ptr()),
      reinterpret_cast<const bf16*>(wpe.data_ptr()), reinterpret_cast<bf16*>(out.data_ptr()), T,
      (int)S, d, V, make_dropout_args(drop_rng, drop_site, drop_thr16, drop_scale));
  MT_LAUNCH_CHECK();
  return out;
}

void embed_bwd(const at::Tensor& ids, const at::Tensor& dy, at::Tensor dwte, at::Tensor dwpe,
               int64_t S, bool accumulate) {
  MT_CHECK_CONTIG(dy);
  MT_CHECK(dwte.scalar_type() == at::kFloat && dwpe.scalar_type() == at::kFloat,
           "embed_bwd: fp32 grads");
  const int d = dy.size(-1);
  const int T = ids.numel();
  const int V = dwte.size(0);
  auto st = cur_stream();
  if (!accumulate) dwte.zero_();
  if (T == 0) return;
  embed_bwd_tok_kernel<<<ew_grid((size_t)T * d / 8), 256, 0, st>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const bf16*>(dy.data_ptr()),
      dwte.data_ptr<float>(), T, d, V);
  MT_LAUNCH_CHECK();
  const int B = T / S;
  embed_bwd_pos_kernel<<<ew_grid((size_t)S * d), 256, 0, st>>>(
      reinterpret_cast<const bf16*>(dy.data_ptr()), dwpe.data_ptr<float>(), B, (int)S, d,
      accumulate ? 1 : 0);
  MT_LAUNCH_CHECK();
}

at::Tensor bias_gelu_fwd(at::Tensor pre, const c10::optional<at::Tensor>& bias) {
  MT_CHECK_CONTIG(pre);
  MT_CHECK(pre.scalar_type() == at::kBFloat16, "gelu: bf16");
  const int F = pre.size(-1);
  MT_CHECK(F % 8 == 0, "gelu: F % 8");
  const size_t rows = pre.numel() / F;
  auto act = at::empty_like(pre);
  if (rows == 0) return act;
  bias_gelu_fwd_kernel<<<ew_grid(rows * F / 8), 256, 0, cur_stream()>>>(
      reinterpret_cast<bf16*>(pre.data_ptr()),
      bias.has_value() ? bias->data_ptr<float>() : nullptr,
      reinterpret_cast<bf16*>(act.data_ptr()), rows, F);
  MT_LAUNCH_CHECK();
  return act;
}

void gelu_bwd_(at::Tensor dact, const at::Tensor& pre) {
  MT_CHECK(dact.numel() % 8 == 0, "gelu_bwd: numel % 8");
  const size_t n8 = dact.numel() / 8;
  if (n8 == 0) return;
  gelu_bwd_kernel<<<ew_grid(n8), 256, 0, cur_stream()>>>(
      reinterpret_cast<bf16*>(dact.data_ptr()), reinterpret_cast<const bf16*>(pre.data_ptr()), n8);
  MT_LAUNCH_CHECK();
}

void colsum_e5m2_(const at::Tensor& codes, at::Tensor out, bool accumulate, const c10::optional<at::Tensor>& scale,
                  const c10::optional<at::Tensor>& scale2) {
  MT_CHECK_CONTIG(codes);
  MT_CHECK(codes.element_size() == 1, "colsum_e5m2: uint8 codes");
  MT_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous(), "colsum_e5m2: fp32 contiguous out");
  const int F = codes.size(-1);
  const int rows = codes.numel() / F;
  MT_CHECK(F % 8 == 0 && reinterpret_cast<uintptr_t>(codes.data_ptr()) % 8 == 0 && out.numel() == F,
           "colsum_e5m2: F % 8 == 0, 8-byte aligned codes, out [F]");
  if (!accumulate) out.zero_();
  if (rows == 0) return;
  const int col_blocks = (F + 255) / 256;
  int row_blocks = std::max(1, std::min((rows + 63) / 64, (num_sms() * 8 + col_blocks - 1) / col_blocks));
  const int rpb = (rows + row_blocks - 1) / row_blocks;
  row_blocks = (rows + rpb - 1) / rpb;
  colsum_e5m2_kernel<<<dim3(col_blocks, row_blocks), 256, 0, cur_stream()>>>(
      reinterpret_cast<const uint8_t*>(codes.data_ptr()), out.data_ptr<float>(),
      scale.has_value() ? scale->data_ptr<float>() : nullptr, scale2.has_value() ? scale2->data_ptr<float>() : nullptr,
      rows, F, rpb);
  MT_LAUNCH_CHECK();
}

void colsum_(const at::Tensor& x, at::Tensor out, bool accumulate,
             const c10::optional<at::Tensor>& scale) {
  MT_CHECK_CONTIG(x);
  MT_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous(), "colsum: fp32 contiguous out");
  const int F = x.size(-1);
  const int rows = x.numel() / F;
  if (!accumulate) out.zero_();
  if (rows == 0) return;
  const float* sp = scale.has_value() ? scale->data_ptr<float>() : nullptr;
  const bool vec = F % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0;
  if (vec) {
    const int col_blocks = (F + 255) / 256;
    // enough blocks to fill the GPU several times over, >= 64 rows each
    int row_blocks = std::max(1, std::min((rows + 63) / 64, (num_sms() * 8 + col_blocks - 1) / col_blocks));
    const int rpb = (rows + row_blocks - 1) / row_blocks;
    row_blocks = (rows + rpb - 1) / rpb;
    colsum_vec_kernel<<<dim3(col_blocks, row_blocks), 256, 0, cur_stream()>>>(
        reinterpret_cast<const bf16*>(x.data_ptr()), out.data_ptr<float>(), sp, rows, F, rpb);
  } else {
    const int rpb = 256;
    dim3 grid((F + 255) / 256, (rows + rpb - 1) / rpb);
    colsum_kernel<<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<const bf16*>(x.data_ptr()),
                                                  out.data_ptr<float>(), sp, rows, F, rpb);
  }
  MT_LAUNCH_CHECK();
}

}  // namespace mtorus
