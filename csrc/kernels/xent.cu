// Fused softmax cross-entropy: loss and dlogits in one kernel.
//
// Reference: cross_entropy_loss = -mean(gather(log_softmax(logits), targets))
// (examples/gpt-1b/src/main.rs:32-41).
//
// Design (B200): one CTA per row of the [T, V] bf16 logits.  Pass 1 streams the
// row once with 16-byte loads and an online max / sum-exp (one rescale per
// 8-value vector, base-2 exponentials of pre-scaled logits); pass 2 re-reads the
// row (an L2 hit: the row was touched microseconds earlier) and overwrites it
// in place with dlogits = grad_scale * (softmax - onehot).  Half of the
// exponentials of the 16-byte vectors run as ex2_poly on the FMA pipe, so the
// special-function unit (two exponentials per logit) does not bound the kernel.  grad_scale is a
// device scalar (1/T times the loss scale), so the backward needs no host sync
// and fp32 logits are never materialised.
#include "common.cuh"
#include "ex2poly.cuh"
#include "amax_publish.cuh"

namespace mtorus {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void online_update(float& m, float& s, float x) {
  if (x > m) {
    s = s * __expf(m - x) + 1.f;
    m = x;
  } else {
    s += __expf(x - m);
  }
}

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = s * __expf(m - mm) + s2 * __expf(m2 - mm);
  m = mm;
}

template <bool VEC>
__global__ void __launch_bounds__(512) xent_fwd_bwd(bf16* __restrict__ logits,
                                                    const int64_t* __restrict__ targets,
                                                    float* __restrict__ loss_rows,
                                                    const float* __restrict__ grad_scale,
                                                    float scale_mul, int V, int write_grad,
                                                    uint8_t* __restrict__ out8, const float* __restrict__ out8_scale,
                                                    float* __restrict__ out8_amax) {
  // out8 (VEC only): dlogits leave as E5M2 codes of the bf16-rounded values times *out8_scale
  // (the LM-head backward's operand) instead of overwriting the logits, and max|dlogit|
  // folds into *out8_amax -- the separate quantise pass and the bf16 dlogits disappear
  __shared__ float red_m[32], red_s[32];
  const int row = blockIdx.x;
  bf16* lr = logits + (size_t)row * V;
  float m = -INFINITY, s = 0.f;
  if (VEC) {
    // m, s in log2 units of the scaled logits x * log2e
    const int nv = V / 8;
    for (int j = threadIdx.x; j < nv; j += blockDim.x) {
      float f[8];
      unpack8(reinterpret_cast<const bf16x8*>(lr)[j], f);
      float vm = f[0];
#pragma unroll
      for (int i = 1; i < 8; ++i) vm = fmaxf(vm, f[i]);
      vm *= kLog2e;
      if (vm > m) {
        s *= exp2f(m - vm);
        m = vm;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xe = fmaf(f[i], kLog2e, -m);
        s += i < 4 ? exp2f(xe) : ex2_poly(xe);
      }
    }
    m *= 1.f / kLog2e;  // back to natural units for the merge below
  } else {
    for (int j = threadIdx.x; j < V; j += blockDim.x) online_update(m, s, __bfloat162float(lr[j]));
  }
  // block reduce of (m, s)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) {
    red_m[wid] = m;
    red_s[wid] = s;
  }
  __syncthreads();
  m = lane < nw ? red_m[lane] : -INFINITY;
  s = lane < nw ? red_s[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  const int64_t tgt = targets[row];
  const float lse = m + logf(s);
  if (threadIdx.x == 0) {
    const float xt = (tgt >= 0 && tgt < V) ? __bfloat162float(lr[tgt]) : lse;
    loss_rows[row] = lse - xt;
  }
  if (!write_grad) return;
  __syncthreads();  // thread 0 read lr[tgt] before it is overwritten
  const float gs = (grad_scale ? *grad_scale : 1.f) * scale_mul;
  const float inv_s = 1.f / s;
  if (VEC) {
    const int nv = V / 8;
    const float nm = -m * kLog2e, ps = gs * inv_s;
    const float q = out8 ? *out8_scale : 0.f;
    float am = 0.f;
    for (int j = threadIdx.x; j < nv; j += blockDim.x) {
      float f[8];
      unpack8(reinterpret_cast<const bf16x8*>(lr)[j], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xe = fmaf(f[i], kLog2e, nm);
        float g = (i < 4 ? exp2f(xe) : ex2_poly(xe)) * ps;
        if (j * 8 + i == tgt) g -= gs;
        f[i] = g;
      }
      if (out8) {
        float r[8];
        unpack8(pack8(f), r);  // the bf16 dlogits the separate quantiser would read
        uint32_t w[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
#pragma unroll
          for (int i = 0; i < 4; ++i) am = fmaxf(am, fabsf(r[4 * k + i]));
          const uint16_t lo = cvt2_e5m2(r[4 * k] * q, r[4 * k + 1] * q);
          const uint16_t hi = cvt2_e5m2(r[4 * k + 2] * q, r[4 * k + 3] * q);
          w[k] = (uint32_t)lo | ((uint32_t)hi << 16);
        }
        reinterpret_cast<uint2*>(out8 + (size_t)row * V)[j] = make_uint2(w[0], w[1]);
      } else {
        reinterpret_cast<bf16x8*>(lr)[j] = pack8(f);
      }
    }
    if (out8) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
      if ((threadIdx.x & 31) == 0) atomic_max_pos(out8_amax, am);
    }
  } else {
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      float p = __expf(__bfloat162float(lr[j]) - m) * inv_s;
      if (j == tgt) p -= 1.f;
      lr[j] = __float2bfloat16_rn(p * gs);
    }
  }
}

// logits [T, V] bf16 (overwritten with dlogits when write_grad); returns per-row loss fp32.
// out8 (uint8 [T, V], with out8_scale / out8_amax fp32 [1]): the dlogits go there as E5M2
// codes instead (the logits are left as they were), their max |value| into out8_amax.
at::Tensor xent_fused(at::Tensor logits, const at::Tensor& targets,
                      const c10::optional<at::Tensor>& grad_scale, double scale_mul,
                      bool write_grad, const c10::optional<at::Tensor>& out8,
                      const c10::optional<at::Tensor>& out8_scale, const c10::optional<at::Tensor>& out8_amax) {
  MT_CHECK_CUDA(logits);
  MT_CHECK_CONTIG(logits);
  MT_CHECK(logits.scalar_type() == at::kBFloat16, "xent: logits must be bf16");
  MT_CHECK(targets.scalar_type() == at::kLong, "xent: targets must be int64");
  const int V = logits.size(-1);
  const int T = logits.numel() / V;
  auto loss = at::empty({T}, logits.options().dtype(at::kFloat));
  if (T == 0) return loss;
  const float* gsp = nullptr;
  if (grad_scale.has_value()) {
    MT_CHECK(grad_scale->scalar_type() == at::kFloat, "grad_scale must be fp32");
    gsp = grad_scale->data_ptr<float>();
  }
  auto* lp = reinterpret_cast<bf16*>(logits.data_ptr());
  const bool vec = (V % 8 == 0) && (reinterpret_cast<uintptr_t>(lp) % 16 == 0);
  uint8_t* o8 = nullptr;
  const float* o8s = nullptr;
  float* o8a = nullptr;
  if (out8.has_value()) {
    MT_CHECK(vec && write_grad, "xent: E5M2 dlogits need V % 8 == 0, 16-byte aligned logits and write_grad");
    MT_CHECK(out8->is_cuda() && out8->element_size() == 1 && out8->is_contiguous() && out8->numel() == logits.numel() &&
                 reinterpret_cast<uintptr_t>(out8->data_ptr()) % 8 == 0,
             "xent: out8 must be contiguous uint8 shaped like the logits");
    MT_CHECK(out8_scale.has_value() && out8_amax.has_value() && out8_scale->scalar_type() == at::kFloat &&
                 out8_amax->scalar_type() == at::kFloat,
             "xent: out8 needs fp32 out8_scale and out8_amax");
    o8 = reinterpret_cast<uint8_t*>(out8->data_ptr());
    o8s = out8_scale->data_ptr<float>();
    o8a = out8_amax->data_ptr<float>();
  }
  auto st = cur_stream();
  if (vec)
    xent_fwd_bwd<true><<<T, 512, 0, st>>>(lp, targets.data_ptr<int64_t>(), loss.data_ptr<float>(),
                                          gsp, (float)scale_mul, V, write_grad, o8, o8s, o8a);
  else
    xent_fwd_bwd<false><<<T, 512, 0, st>>>(lp, targets.data_ptr<int64_t>(),
                                           loss.data_ptr<float>(), gsp, (float)scale_mul, V,
                                           write_grad, nullptr, nullptr, nullptr);
  MT_LAUNCH_CHECK();
  return loss;
}

}  // namespace mtorus
