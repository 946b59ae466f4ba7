// Device-resident optimizer step: gradient norm + overflow detection, loss-scaler
// update, global-norm clipping and fused Adam / SGD over flat parameter buffers.
//
// Reference semantics:
//   * overflow  = non-finite gradient norm -> skip the step, halve the dynamic
//     loss scale (floor 1.0), reset the growth counter
//     (crates/mt-training/src/step.rs:128-139, crates/mt-core/src/precision/loss_scale.rs:34-51)
//   * growth    = double the scale after `growth_interval` clean steps (loss_scale.rs:41-48)
//   * clip      = g *= max_norm / norm when norm > max_norm (step.rs:61-70,84-98)
//   * Adam      = burn-optim Adam (beta1 0.9, beta2 0.999, eps 1e-5), bias-corrected
//   * SGD       = w - lr * dequant(g) (crates/mt-burn/src/optim_ext.rs:44-63)
//
// Design (B200): no host synchronisation anywhere.  The state lives in a small
// fp32 device block `st` (layout kSt* below); the norm kernel reduces Σg² and a
// non-finite flag into it, a one-thread finalize kernel runs the loss-scaler
// state machine and computes the combined gradient multiplier, and the Adam
// kernel reads that multiplier and the skip flag.  Buffers are streamed once
// with 16-byte vectors.
#include "common.cuh"

namespace mtorus {

// device state block (fp32 slots)
enum : int {
  kStSumSq = 0,      // Σ g² of the raw (scaled) gradients, accumulated by the norm kernel
  kStNonFinite = 1,  // > 0 when a NaN/Inf was seen
  kStScale = 2,      // current loss scale
  kStGrowthCounter = 3,
  kStGradMul = 4,    // multiplier applied to raw grads in the update (unscale * clip)
  kStSkip = 5,       // 1 when this step is skipped (overflow)
  kStGradNorm = 6,   // unscaled global grad norm (NaN/Inf on overflow)
  kStStep = 7,       // number of optimizer steps taken (for bias correction)
  kStOverflowCount = 8,
  kStLast = 16
};

template <typename G>
__global__ void grad_sumsq_kernel(const G* __restrict__ g, size_t n, float* __restrict__ st) {
  __shared__ float red[32];
  float acc = 0.f;
  int bad = 0;
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if constexpr (sizeof(G) == 2) {
    const size_t nv = n / 8;
    for (size_t i = tid; i < nv; i += stride) {
      float f[8];
      unpack8(reinterpret_cast<const bf16x8*>(g)[i], f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        acc += f[k] * f[k];
        bad |= !isfinite(f[k]);
      }
    }
    for (size_t i = nv * 8 + tid; i < n; i += stride) {
      const float f = to_f(g[i]);
      acc += f * f;
      bad |= !isfinite(f);
    }
  } else {
    const size_t nv = n / 4;
    for (size_t i = tid; i < nv; i += stride) {
      const float4 f = reinterpret_cast<const float4*>(g)[i];
      acc += f.x * f.x + f.y * f.y + f.z * f.z + f.w * f.w;
      bad |= !(isfinite(f.x) && isfinite(f.y) && isfinite(f.z) && isfinite(f.w));
    }
    for (size_t i = nv * 4 + tid; i < n; i += stride) {
      const float f = to_f(g[i]);
      acc += f * f;
      bad |= !isfinite(f);
    }
  }
  acc = block_sum(acc, red);
  const int anybad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    atomicAdd(st + kStSumSq, acc);
    if (anybad) atomicAdd(st + kStNonFinite, 1.f);
  }
}

// One thread: loss scaler state machine + clip factor.
// dynamic: 1 = dynamic scaler, 0 = static (updates ignored).
__global__ void optim_finalize_kernel(float* st, int dynamic, int growth_interval,
                                      float max_norm, int unscale) {
  const float scale = st[kStScale];
  const bool overflow = st[kStNonFinite] > 0.f || !isfinite(st[kStSumSq]);
  const float inv = unscale ? 1.f / scale : 1.f;
  const float norm = sqrtf(st[kStSumSq]) * inv;
  st[kStGradNorm] = overflow ? __int_as_float(0x7fc00000) : norm;
  float mul = inv;
  if (!overflow && max_norm > 0.f && norm > max_norm) mul *= max_norm / norm;
  st[kStGradMul] = mul;
  st[kStSkip] = overflow ? 1.f : 0.f;
  if (overflow) st[kStOverflowCount] += 1.f;
  else st[kStStep] += 1.f;
  if (dynamic) {
    if (overflow) {
      st[kStScale] = fmaxf(scale * 0.5f, 1.f);
      st[kStGrowthCounter] = 0.f;
    } else {
      float c = st[kStGrowthCounter] + 1.f;
      if (c >= (float)growth_interval) {
        st[kStScale] = scale * 2.f;
        c = 0.f;
      }
      st[kStGrowthCounter] = c;
    }
  }
  // reset accumulators for the next step
  st[kStSumSq] = 0.f;
  st[kStNonFinite] = 0.f;
}

// Adam over a flat range. p/m/v fp32, g bf16 or fp32; w16 (optional) gets the bf16 copy.
template <typename G>
__global__ void adam_kernel(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                            const G* __restrict__ g, bf16* __restrict__ w16, size_t n,
                            const float* __restrict__ st, float lr, float beta1, float beta2,
                            float eps, float weight_decay, float step_override) {
  if (st[kStSkip] > 0.f) return;
  const float gm = st[kStGradMul];
  const float step = step_override > 0.f ? step_override : st[kStStep];
  const float bc1 = 1.f - powf(beta1, step);
  const float bc2 = 1.f - powf(beta2, step);
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t nv = n / 8;
  for (size_t i = tid; i < nv; i += stride) {
    float gf[8];
    if constexpr (sizeof(G) == 2) {
      unpack8(reinterpret_cast<const bf16x8*>(g)[i], gf);
    } else {
      const float4 a = reinterpret_cast<const float4*>(g)[2 * i];
      const float4 b = reinterpret_cast<const float4*>(g)[2 * i + 1];
      gf[0] = a.x; gf[1] = a.y; gf[2] = a.z; gf[3] = a.w;
      gf[4] = b.x; gf[5] = b.y; gf[6] = b.z; gf[7] = b.w;
    }
    float4* p4 = reinterpret_cast<float4*>(p) + 2 * i;
    float4* m4 = reinterpret_cast<float4*>(m) + 2 * i;
    float4* v4 = reinterpret_cast<float4*>(v) + 2 * i;
    float pf[8], mf[8], vf[8];
    *reinterpret_cast<float4*>(pf) = p4[0];
    *reinterpret_cast<float4*>(pf + 4) = p4[1];
    *reinterpret_cast<float4*>(mf) = m4[0];
    *reinterpret_cast<float4*>(mf + 4) = m4[1];
    *reinterpret_cast<float4*>(vf) = v4[0];
    *reinterpret_cast<float4*>(vf + 4) = v4[1];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float gg = gf[k] * gm;
      if (weight_decay != 0.f) gg += weight_decay * pf[k];
      mf[k] = beta1 * mf[k] + (1.f - beta1) * gg;
      vf[k] = beta2 * vf[k] + (1.f - beta2) * gg * gg;
      const float denom = sqrtf(vf[k]) * inv_sqrt_bc2 + eps;
      pf[k] -= step_size * mf[k] / denom;
    }
    p4[0] = *reinterpret_cast<float4*>(pf);
    p4[1] = *reinterpret_cast<float4*>(pf + 4);
    m4[0] = *reinterpret_cast<float4*>(mf);
    m4[1] = *reinterpret_cast<float4*>(mf + 4);
    v4[0] = *reinterpret_cast<float4*>(vf);
    v4[1] = *reinterpret_cast<float4*>(vf + 4);
    if (w16) reinterpret_cast<bf16x8*>(w16)[i] = pack8(pf);
  }
  for (size_t i = nv * 8 + tid; i < n; i += stride) {
    float gg = to_f(g[i]) * gm;
    if (weight_decay != 0.f) gg += weight_decay * p[i];
    m[i] = beta1 * m[i] + (1.f - beta1) * gg;
    v[i] = beta2 * v[i] + (1.f - beta2) * gg * gg;
    p[i] -= step_size * m[i] / (sqrtf(v[i]) * inv_sqrt_bc2 + eps);
    if (w16) w16[i] = __float2bfloat16_rn(p[i]);
  }
}

template <typename G>
__global__ void sgd_kernel(float* __restrict__ p, const G* __restrict__ g, bf16* __restrict__ w16,
                           size_t n, const float* __restrict__ st, float lr) {
  if (st[kStSkip] > 0.f) return;
  const float gm = st[kStGradMul];
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    p[i] -= lr * to_f(g[i]) * gm;
    if (w16) w16[i] = __float2bfloat16_rn(p[i]);
  }
}

static int grid_for(size_t n, int per_thread) {
  const size_t blocks = (n / per_thread + 255) / 256;
  return (int)std::max<size_t>(1, std::min<size_t>(blocks, (size_t)num_sms() * 8));
}

void optim_grad_sumsq(const at::Tensor& g, at::Tensor st) {
  MT_CHECK_CONTIG(g);
  const size_t n = g.numel();
  if (n == 0) return;
  auto s = cur_stream();
  if (g.scalar_type() == at::kBFloat16) {
    MT_CHECK(reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0, "grad buffer must be 16B aligned");
    grad_sumsq_kernel<bf16><<<grid_for(n, 8), 256, 0, s>>>(
        reinterpret_cast<const bf16*>(g.data_ptr()), n, st.data_ptr<float>());
  } else {
    MT_CHECK(g.scalar_type() == at::kFloat, "grad must be bf16 or fp32");
    MT_CHECK(reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0, "grad buffer must be 16B aligned");
    grad_sumsq_kernel<float><<<grid_for(n, 4), 256, 0, s>>>(g.data_ptr<float>(), n,
                                                              st.data_ptr<float>());
  }
  MT_LAUNCH_CHECK();
}

void optim_finalize(at::Tensor st, bool dynamic, int64_t growth_interval, double max_norm,
                    bool unscale) {
  optim_finalize_kernel<<<1, 1, 0, cur_stream()>>>(st.data_ptr<float>(), dynamic ? 1 : 0,
                                                   (int)growth_interval, (float)max_norm,
                                                   unscale ? 1 : 0);
  MT_LAUNCH_CHECK();
}

void adam_step(at::Tensor p, at::Tensor m, at::Tensor v, const at::Tensor& g,
               c10::optional<at::Tensor> w16, const at::Tensor& st, double lr, double beta1,
               double beta2, double eps, double weight_decay, double step_override) {
  MT_CHECK(p.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat &&
               v.scalar_type() == at::kFloat,
           "adam: p/m/v must be fp32");
  const size_t n = p.numel();
  MT_CHECK(m.numel() == (int64_t)n && v.numel() == (int64_t)n && g.numel() == (int64_t)n,
           "adam: size mismatch");
  for (auto* t : {&p, &m, &v})
    MT_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "adam: buffers must be 16B aligned");
  bf16* w = nullptr;
  if (w16.has_value()) {
    MT_CHECK(w16->scalar_type() == at::kBFloat16 && w16->numel() == (int64_t)n, "adam: w16");
    MT_CHECK(reinterpret_cast<uintptr_t>(w16->data_ptr()) % 16 == 0, "adam: w16 alignment");
    w = reinterpret_cast<bf16*>(w16->data_ptr());
  }
  auto s = cur_stream();
  if (n == 0) return;
  if (g.scalar_type() == at::kBFloat16)
    adam_kernel<bf16><<<grid_for(n, 8), 256, 0, s>>>(
        p.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
        reinterpret_cast<const bf16*>(g.data_ptr()), w, n, st.data_ptr<float>(), (float)lr,
        (float)beta1, (float)beta2, (float)eps, (float)weight_decay, (float)step_override);
  else
    adam_kernel<float><<<grid_for(n, 8), 256, 0, s>>>(
        p.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), g.data_ptr<float>(), w,
        n, st.data_ptr<float>(), (float)lr, (float)beta1, (float)beta2, (float)eps,
        (float)weight_decay, (float)step_override);
  MT_LAUNCH_CHECK();
}

void sgd_step(at::Tensor p, const at::Tensor& g, c10::optional<at::Tensor> w16,
              const at::Tensor& st, double lr) {
  const size_t n = p.numel();
  bf16* w = w16.has_value() ? reinterpret_cast<bf16*>(w16->data_ptr()) : nullptr;
  auto s = cur_stream();
  if (n == 0) return;
  if (g.scalar_type() == at::kBFloat16)
    sgd_kernel<bf16><<<grid_for(n, 1), 256, 0, s>>>(p.data_ptr<float>(),
                                                    reinterpret_cast<const bf16*>(g.data_ptr()),
                                                    w, n, st.data_ptr<float>(), (float)lr);
  else
    sgd_kernel<float><<<grid_for(n, 1), 256, 0, s>>>(p.data_ptr<float>(), g.data_ptr<float>(), w,
                                                     n, st.data_ptr<float>(), (float)lr);
  MT_LAUNCH_CHECK();
}

}  // namespace mtorus
