// Causal multi-head attention (flash attention) on tcgen05 for the fused GPT path.
//
// Reference semantics: scores = Q K^T / sqrt(d_head) + causal mask -> softmax -> P V
// (examples/gpt-1b/src/transformer.rs:51-85, mask :163-171); dropout is not applied.
// Layout: one [T, 3*H*128] bf16 matrix holds q | k | v for T = B*S tokens (heads
// contiguous inside each third), the output is [T, H*128]; S is a multiple of 128.
//
// Forward, one CTA per (128-query tile, batch, head), heaviest tiles first:
//   warp 0      TMA producer: Q once, then K_j / V_j into a 2-stage ring
//   warp 1      MMA issuer: S_j = Q K_j^T into one of two TMEM buffers (issued one
//               tile ahead), then O += P_j V_j into the TMEM accumulator
//   warps 2..5  softmax: one query row per thread, read from TMEM; running max
//               with lazy rescaling (O is rescaled only when a row max grows by
//               more than 2^8), P written as bf16 into shared memory in the
//               128B-swizzled K-major layout the MMA reads; the epilogue divides
//               by the row sum and stores O and the log-sum-exp.
// Backward, one CTA per (128-key tile, batch, head), looping over query tiles i >= j:
//   S^T = K Q^T and dP^T = V dO^T into TMEM; P^T = exp(S^T*scale - lse) and
//   dS^T = P^T (dP^T - D) * scale written to shared memory; dV += P^T dO,
//   dK += dS^T Q accumulate in TMEM; dQ_i = dS K lands in TMEM (reusing the S^T
//   columns) and is added to an fp32 dQ buffer with vector atomics.
// D = rowsum(dO * O) comes from a small pre-kernel; a post-kernel casts dQ to bf16.
//
// Every wait is bounded (2 s); on a timeout the kernel records a status code,
// lets its in-flight copies and MMAs land, frees TMEM and returns.
#include "common.cuh"
#include "sm100.cuh"

#include <ATen/ops/zeros.h>

namespace mtorus {

CUtensorMap make_tma_2d(const void* ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                        uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swz);
void ensure_context();

namespace {
using namespace sm100;

constexpr int kD = 128;                 // head dim
constexpr int kTile = 128;              // query / key tile
constexpr int kTileBytes = kTile * kD * 2;  // 32 KB: two 64-column halves of [128 x 128 B]
constexpr int kHalf = kTile * 128;          // 16 KB
constexpr int kThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;        // lazy rescale threshold (log2 units)

int* attn_status_ptr() {
  static int* p = nullptr;
  if (!p) {
    C10_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  }
  return p;
}

// Byte offset of element (row, col) of a [128 x 128] bf16 tile stored as two
// K-major SW128 halves (cols 0-63, 64-127), 8 elements per 16-byte chunk.
__device__ __forceinline__ uint32_t sw128_chunk(int row, int chunk16) {
  const int half = chunk16 >> 3, c = chunk16 & 7;
  return half * kHalf + row * 128 + ((c ^ (row & 7)) << 4);
}

// K-major descriptor for MMA k-step k (16 elements) of a [128 x 128] SW128 tile.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int k) {
  return make_sdesc(base + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024, kSwizzle128B);
}
// MN-major descriptor for k-step k: the tile's rows are the K dimension, its
// 128 columns (two 64-element halves) the M or N dimension.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int k) {
  return make_sdesc(base + k * 2048, kHalf, 1024, kSwizzle128B);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  bf162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void bounded_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(smem_u32(bar), parity) && globaltimer_ns() - t0 < 100000000ull) {
  }
}

__device__ __forceinline__ void named_sync_compute() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// ================================================================== forward
struct FwdCtl {
  uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], p_full, o_done, drain;
  uint32_t tmem_base;
  int abort;
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tma_qkv, bf16* __restrict__ out, int ld_out,
                    float* __restrict__ lse, int B, int H, int S, float scale, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + kTileBytes;             // stage s: K at +2s*32K, V at +(2s+1)*32K
  uint8_t* sP = smem + 5 * kTileBytes;
  FwdCtl* ctl = reinterpret_cast<FwdCtl*>(smem + 6 * kTileBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = S / kTile;
  const int bh = blockIdx.x % (B * H);
  const int qt = nq - 1 - blockIdx.x / (B * H);  // heaviest query tiles first
  const int b = bh / H, h = bh % H;
  const int nkv = qt + 1;
  const int row0 = b * S + qt * kTile;

  if (threadIdx.x == 0) {
    mbar_init(&ctl->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ctl->kv_full[s], 1);
      mbar_init(&ctl->kv_empty[s], 1);
      mbar_init(&ctl->s_full[s], 1);
    }
    mbar_init(&ctl->p_full, 128);
    mbar_init(&ctl->o_done, 1);
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_qkv);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;
  volatile int* abort = &ctl->abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      const int qcol = h * kD, kcol = H * kD + h * kD, vcol = 2 * H * kD + h * kD;
      mbar_arrive_expect_tx(&ctl->q_full, kTileBytes);
      tma_load_2d(sQ, &tma_qkv, &ctl->q_full, qcol, row0);
      tma_load_2d(sQ + kHalf, &tma_qkv, &ctl->q_full, qcol + 64, row0);
      uint32_t issued = 0, par = 0;
      for (int j = 0; j < nkv && !*abort; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&ctl->kv_empty[st], ((j >> 1) - 1) & 1, abort, status, 11)) break;
        uint8_t* k = sKV + (2 * st) * kTileBytes;
        uint8_t* v = k + kTileBytes;
        const int kr = b * S + j * kTile;
        issued |= 1u << st;
        par = (par & ~(1u << st)) | (((uint32_t)(j >> 1) & 1u) << st);
        mbar_arrive_expect_tx(&ctl->kv_full[st], 2 * kTileBytes);
        tma_load_2d(k, &tma_qkv, &ctl->kv_full[st], kcol, kr);
        tma_load_2d(k + kHalf, &tma_qkv, &ctl->kv_full[st], kcol + 64, kr);
        tma_load_2d(v, &tma_qkv, &ctl->kv_full[st], vcol, kr);
        tma_load_2d(v + kHalf, &tma_qkv, &ctl->kv_full[st], vcol + 64, kr);
      }
      if (*abort) {
        bounded_drain(&ctl->q_full, 0);
        for (int s = 0; s < 2; ++s)
          if (issued >> s & 1u) bounded_drain(&ctl->kv_full[s], (par >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t idS = make_idesc_bf16(kTile, kTile, 0, 0);
      const uint32_t idO = make_idesc_bf16(kTile, kD, 0, 1);
      const uint32_t q = smem_u32(sQ), p = smem_u32(sP);
      bool issued_any = false, ok = mbar_wait(&ctl->q_full, 0, abort, status, 12);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&ctl->kv_full[st], (j >> 1) & 1, abort, status, 13)) return false;
        tc_fence_after();
        const uint32_t k = smem_u32(sKV + (2 * st) * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_f16(tS[st], desc_kmajor(q, kk), desc_kmajor(k, kk), idS, kk > 0 ? 1u : 0u);
        umma_commit(&ctl->s_full[st]);
        issued_any = true;
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv && !issue_s(j + 1)) break;
        if (!mbar_wait(&ctl->p_full, j & 1, abort, status, 14)) break;
        tc_fence_after();
        const uint32_t v = smem_u32(sKV + (2 * (j & 1) + 1) * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_f16(tO, desc_kmajor(p, kk), desc_mnmajor(v, kk), idO, (j | kk) != 0 ? 1u : 0u);
        umma_commit(&ctl->o_done);
        umma_commit(&ctl->kv_empty[j & 1]);
      }
      if (*abort && issued_any) {
        umma_commit(&ctl->drain);
        bounded_drain(&ctl->drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&ctl->s_full[st], (j >> 1) & 1, abort, status, 15)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float t[kTile];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tS[st] + lane_off + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) t[c * 32 + e] = __uint_as_float(v[e]) * sl2;
      }
      if (j == qt) {  // diagonal tile: keys after the query are masked
#pragma unroll
        for (int e = 0; e < kTile; ++e)
          if (e > r) t[e] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < kTile; ++e) mx = fmaxf(mx, t[e]);
      float alpha = 1.f;
      if (j == 0) {
        m_ref = mx;
      } else if (mx > m_ref + kRescale) {
        alpha = exp2f(m_ref - mx);
        m_ref = mx;
      }
      // O and the P buffer are free once the previous P V product has completed
      if (j > 0) {
        if (!mbar_wait(&ctl->o_done, (j - 1) & 1, abort, status, 16)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(tO + lane_off + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            tmem_st32(tO + lane_off + c * 32, v);
          }
          tmem_wait_st();
        }
      }
      l *= alpha;
      float sum = 0.f;
#pragma unroll
      for (int c16 = 0; c16 < kTile / 8; ++c16) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pv[e] = exp2f(t[c16 * 8 + e] - m_ref);
          sum += pv[e];
        }
        uint4 w;
        w.x = pack_bf16x2(pv[0], pv[1]);
        w.y = pack_bf16x2(pv[2], pv[3]);
        w.z = pack_bf16x2(pv[4], pv[5]);
        w.w = pack_bf16x2(pv[6], pv[7]);
        *reinterpret_cast<uint4*>(sP + sw128_chunk(r, c16)) = w;
      }
      l += sum;
      fence_async_shared();
      tc_fence_before();
      mbar_arrive(&ctl->p_full);
    }
    if (ok && mbar_wait(&ctl->o_done, (nkv - 1) & 1, abort, status, 17)) {
      tc_fence_after();
      const float inv = 1.f / l;
      bf16* dst = out + (size_t)(row0 + r) * ld_out + h * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tO + lane_off + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(v[e]) * inv, __uint_as_float(v[e + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(v[e + 2]) * inv, __uint_as_float(v[e + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(v[e + 4]) * inv, __uint_as_float(v[e + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(v[e + 6]) * inv, __uint_as_float(v[e + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + c * 32 + e) = w;
        }
      }
      // natural-log log-sum-exp of the scaled scores
      lse[(size_t)bh * S + qt * kTile + r] = (m_ref + log2f(l)) / kLog2e;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ================================================================== backward
struct BwdCtl {
  uint64_t kv_full, qdo_full, qdo_empty, st_full, pds_full, dq_full, dq_free, kv_done, drain;
  uint32_t tmem_base;
  int abort;
  float lse[kTile];
  float dd[kTile];
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tma_qkv, const __grid_constant__ CUtensorMap tma_do,
                    const float* __restrict__ lse, const float* __restrict__ dvec, float* __restrict__ dq,
                    bf16* __restrict__ dqkv, int ld_dqkv, int B, int H, int S, float scale, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sK = smem;
  uint8_t* sV = smem + kTileBytes;
  uint8_t* sQ = smem + 2 * kTileBytes;
  uint8_t* sDO = smem + 3 * kTileBytes;
  uint8_t* sPT = smem + 4 * kTileBytes;
  uint8_t* sDST = smem + 5 * kTileBytes;
  BwdCtl* ctl = reinterpret_cast<BwdCtl*>(smem + 6 * kTileBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = S / kTile;
  const int bh = blockIdx.x % (B * H);
  const int kt = blockIdx.x / (B * H);  // key tile; tile 0 loops over every query tile
  const int b = bh / H, h = bh % H;
  const int nqi = nt - kt;               // query tiles i = kt .. nt-1
  const int krow0 = b * S + kt * kTile;

  if (threadIdx.x == 0) {
    mbar_init(&ctl->kv_full, 1);
    mbar_init(&ctl->qdo_full, 1);
    mbar_init(&ctl->qdo_empty, 1);
    mbar_init(&ctl->st_full, 1);
    mbar_init(&ctl->pds_full, 128);
    mbar_init(&ctl->dq_full, 1);
    mbar_init(&ctl->dq_free, 128);
    mbar_init(&ctl->kv_done, 1);
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_qkv);
    tma_prefetch_desc(&tma_do);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 384;
  const uint32_t tDQ = tS;  // dQ_i reuses the S^T columns once they are read
  volatile int* abort = &ctl->abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      const int qcol = h * kD, kcol = H * kD + h * kD, vcol = 2 * H * kD + h * kD;
      mbar_arrive_expect_tx(&ctl->kv_full, 2 * kTileBytes);
      tma_load_2d(sK, &tma_qkv, &ctl->kv_full, kcol, krow0);
      tma_load_2d(sK + kHalf, &tma_qkv, &ctl->kv_full, kcol + 64, krow0);
      tma_load_2d(sV, &tma_qkv, &ctl->kv_full, vcol, krow0);
      tma_load_2d(sV + kHalf, &tma_qkv, &ctl->kv_full, vcol + 64, krow0);
      int issued = -1;
      for (int it = 0; it < nqi && !*abort; ++it) {
        if (it > 0 && !mbar_wait(&ctl->qdo_empty, (it - 1) & 1, abort, status, 21)) break;
        const int qr = b * S + (kt + it) * kTile;
        issued = it;
        mbar_arrive_expect_tx(&ctl->qdo_full, 2 * kTileBytes);
        tma_load_2d(sQ, &tma_qkv, &ctl->qdo_full, qcol, qr);
        tma_load_2d(sQ + kHalf, &tma_qkv, &ctl->qdo_full, qcol + 64, qr);
        tma_load_2d(sDO, &tma_do, &ctl->qdo_full, h * kD, qr);
        tma_load_2d(sDO + kHalf, &tma_do, &ctl->qdo_full, h * kD + 64, qr);
      }
      if (*abort) {
        bounded_drain(&ctl->kv_full, 0);
        if (issued >= 0) bounded_drain(&ctl->qdo_full, issued & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t id_kk = make_idesc_bf16(kTile, kTile, 0, 0);  // A, B K-major
      const uint32_t id_kn = make_idesc_bf16(kTile, kD, 0, 1);     // A K-major, B MN-major
      const uint32_t id_mn = make_idesc_bf16(kTile, kD, 1, 1);     // A, B MN-major
      const uint32_t k = smem_u32(sK), v = smem_u32(sV), q = smem_u32(sQ), dO = smem_u32(sDO);
      const uint32_t pT = smem_u32(sPT), dsT = smem_u32(sDST);
      bool issued_any = false;
      bool ok = mbar_wait(&ctl->kv_full, 0, abort, status, 22);
      for (int it = 0; it < nqi && ok; ++it) {
        if (!mbar_wait(&ctl->qdo_full, it & 1, abort, status, 23)) break;
        // the S^T columns hold dQ of the previous tile until the compute warps read it
        if (it > 0 && !mbar_wait(&ctl->dq_free, (it - 1) & 1, abort, status, 24)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)  // S^T = K Q^T
          umma_f16(tS, desc_kmajor(k, kk), desc_kmajor(q, kk), id_kk, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)  // dP^T = V dO^T
          umma_f16(tDP, desc_kmajor(v, kk), desc_kmajor(dO, kk), id_kk, kk > 0 ? 1u : 0u);
        umma_commit(&ctl->st_full);
        issued_any = true;
        if (!mbar_wait(&ctl->pds_full, it & 1, abort, status, 25)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dV += P^T dO
          umma_f16(tDV, desc_kmajor(pT, kk), desc_mnmajor(dO, kk), id_kn, (it | kk) != 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dK += dS^T Q
          umma_f16(tDK, desc_kmajor(dsT, kk), desc_mnmajor(q, kk), id_kn, (it | kk) != 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dQ_i = dS K
          umma_f16(tDQ, desc_mnmajor(dsT, kk), desc_mnmajor(k, kk), id_mn, kk > 0 ? 1u : 0u);
        umma_commit(&ctl->dq_full);
        umma_commit(&ctl->qdo_empty);
      }
      if (!*abort) {
        umma_commit(&ctl->kv_done);
      } else if (issued_any) {
        umma_commit(&ctl->drain);
        bounded_drain(&ctl->drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ compute
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row (S^T, dP^T, dV, dK) or query row (dQ)
    const int tid = threadIdx.x - 64;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    bool ok = true;
    for (int it = 0; it < nqi; ++it) {
      const int qi = kt + it;
      // this tile's log-sum-exp (log2 units) and D, shared by all key rows
      ctl->lse[tid] = lse[(size_t)bh * S + qi * kTile + tid] * kLog2e;
      ctl->dd[tid] = dvec[(size_t)bh * S + qi * kTile + tid];
      named_sync_compute();
      if (!mbar_wait(&ctl->st_full, it & 1, abort, status, 26)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = qi == kt;
#pragma unroll 1
      for (int c = 0; c < kTile / 32; ++c) {
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + lane_off + c * 32, sv);
        tmem_ld32(tDP + lane_off + c * 32, dv);
        tmem_wait_ld();
        float p[32], ds[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int col = c * 32 + e;  // query within the tile
          float pe = exp2f(__uint_as_float(sv[e]) * sl2 - ctl->lse[col]);
          if (diag && col < r) pe = 0.f;  // query before key: masked in the forward
          p[e] = pe;
          ds[e] = pe * (__uint_as_float(dv[e]) - ctl->dd[col]) * scale;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint4 wp, wd;
          wp.x = pack_bf16x2(p[g * 8 + 0], p[g * 8 + 1]);
          wp.y = pack_bf16x2(p[g * 8 + 2], p[g * 8 + 3]);
          wp.z = pack_bf16x2(p[g * 8 + 4], p[g * 8 + 5]);
          wp.w = pack_bf16x2(p[g * 8 + 6], p[g * 8 + 7]);
          wd.x = pack_bf16x2(ds[g * 8 + 0], ds[g * 8 + 1]);
          wd.y = pack_bf16x2(ds[g * 8 + 2], ds[g * 8 + 3]);
          wd.z = pack_bf16x2(ds[g * 8 + 4], ds[g * 8 + 5]);
          wd.w = pack_bf16x2(ds[g * 8 + 6], ds[g * 8 + 7]);
          const uint32_t off = sw128_chunk(r, c * 4 + g);
          *reinterpret_cast<uint4*>(sPT + off) = wp;
          *reinterpret_cast<uint4*>(sDST + off) = wd;
        }
      }
      fence_async_shared();
      tc_fence_before();
      mbar_arrive(&ctl->pds_full);
      if (!mbar_wait(&ctl->dq_full, it & 1, abort, status, 27)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float* dqrow = dq + (size_t)(b * S + qi * kTile + r) * (H * kD) + h * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tDQ + lane_off + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          atomicAdd(reinterpret_cast<float4*>(dqrow + c * 32 + e),
                    make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]), __uint_as_float(v[e + 2]),
                                __uint_as_float(v[e + 3])));
      }
      tc_fence_before();
      mbar_arrive(&ctl->dq_free);
    }
    if (ok && mbar_wait(&ctl->kv_done, 0, abort, status, 28)) {
      tc_fence_after();
      // dK and dV rows of this key tile -> the k and v thirds of dqkv
      bf16* dk = dqkv + (size_t)(krow0 + r) * ld_dqkv + H * kD + h * kD;
      bf16* dvp = dqkv + (size_t)(krow0 + r) * ld_dqkv + 2 * H * kD + h * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t a[32], bb[32];
        tmem_ld32(tDK + lane_off + c * 32, a);
        tmem_ld32(tDV + lane_off + c * 32, bb);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(a[e]), __uint_as_float(a[e + 1]));
          w.y = pack_bf16x2(__uint_as_float(a[e + 2]), __uint_as_float(a[e + 3]));
          w.z = pack_bf16x2(__uint_as_float(a[e + 4]), __uint_as_float(a[e + 5]));
          w.w = pack_bf16x2(__uint_as_float(a[e + 6]), __uint_as_float(a[e + 7]));
          *reinterpret_cast<uint4*>(dk + c * 32 + e) = w;
          w.x = pack_bf16x2(__uint_as_float(bb[e]), __uint_as_float(bb[e + 1]));
          w.y = pack_bf16x2(__uint_as_float(bb[e + 2]), __uint_as_float(bb[e + 3]));
          w.z = pack_bf16x2(__uint_as_float(bb[e + 4]), __uint_as_float(bb[e + 5]));
          w.w = pack_bf16x2(__uint_as_float(bb[e + 6]), __uint_as_float(bb[e + 7]));
          *reinterpret_cast<uint4*>(dvp + c * 32 + e) = w;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// D[bh, s] = sum_c dO[t, h*128 + c] * O[t, h*128 + c]; one warp per (token, head).
__global__ void attn_bwd_dot_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ o, int ld,
                                    float* __restrict__ dvec, int B, int H, int S) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int total = B * S * H;
  if (w >= total) return;
  const int t = w / H, h = w % H;
  const bf16* a = dout + (size_t)t * ld + h * kD + lane * 4;
  const bf16* c = o + (size_t)t * ld + h * kD + lane * 4;
  const uint2 ua = *reinterpret_cast<const uint2*>(a), uc = *reinterpret_cast<const uint2*>(c);
  const bf162* ha = reinterpret_cast<const bf162*>(&ua);
  const bf162* hc = reinterpret_cast<const bf162*>(&uc);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float2 x = __bfloat1622float2(ha[i]), y = __bfloat1622float2(hc[i]);
    acc += x.x * y.x + x.y * y.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const int b = t / S, s = t % S;
    dvec[((size_t)b * H + h) * S + s] = acc;
  }
}

// dq (fp32 [T, H*128]) -> the q third of dqkv (bf16)
__global__ void attn_dq_cast_kernel(const float* __restrict__ dq, bf16* __restrict__ dqkv, int ld_dqkv,
                                    int T, int HD) {
  const size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= (size_t)T * HD) return;
  const size_t t = i / HD, c = i % HD;
  const float4 a = *reinterpret_cast<const float4*>(dq + i);
  const float4 b = *reinterpret_cast<const float4*>(dq + i + 4);
  uint4 w;
  w.x = pack_bf16x2(a.x, a.y);
  w.y = pack_bf16x2(a.z, a.w);
  w.z = pack_bf16x2(b.x, b.y);
  w.w = pack_bf16x2(b.z, b.w);
  *reinterpret_cast<uint4*>(dqkv + t * ld_dqkv + c) = w;
}

constexpr size_t kFwdSmem = 6 * kTileBytes + sizeof(FwdCtl) + 1024;
constexpr size_t kBwdSmem = 6 * kTileBytes + sizeof(BwdCtl) + 1024;

void check_qkv(const at::Tensor& qkv, int B, int S, int H) {
  MT_CHECK_CUDA(qkv);
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16, "attention: bf16 qkv");
  TORCH_CHECK(qkv.dim() == 2 && qkv.size(0) == (int64_t)B * S && qkv.size(1) == 3LL * H * kD,
              "attention: qkv must be [B*S, 3*H*128]");
  TORCH_CHECK(qkv.stride(1) == 1 && qkv.stride(0) % 8 == 0, "attention: qkv rows must be contiguous, 16B aligned");
  TORCH_CHECK(S % kTile == 0, "attention: sequence length must be a multiple of 128");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0, "attention: qkv must be 16-byte aligned");
}

}  // namespace

// qkv [B*S, 3*H*128] bf16 -> (out [B*S, H*128] bf16, lse [B, H, S] fp32)
std::vector<at::Tensor> attn_fwd(const at::Tensor& qkv, int64_t B, int64_t S, int64_t H) {
  check_qkv(qkv, (int)B, (int)S, (int)H);
  ensure_context();
  auto out = at::empty({B * S, H * kD}, qkv.options());
  auto lse = at::empty({B, H, S}, qkv.options().dtype(at::kFloat));
  const CUtensorMap tm = make_tma_2d(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3 * H * kD, B * S,
                                     qkv.stride(0), 64, kTile, CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kFwdSmem));
    attr = true;
  }
  const int grid = (int)(B * H * (S / kTile));
  attn_fwd_kernel<<<grid, kThreads, kFwdSmem, cur_stream()>>>(tm, (bf16*)out.data_ptr(), (int)(H * kD),
                                                              lse.data_ptr<float>(), (int)B, (int)H, (int)S,
                                                              1.0f / sqrtf((float)kD), attn_status_ptr());
  MT_LAUNCH_CHECK();
  return {out, lse};
}

// -> dqkv [B*S, 3*H*128] bf16 (dq | dk | dv)
at::Tensor attn_bwd(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& lse,
                    int64_t B, int64_t S, int64_t H) {
  check_qkv(qkv, (int)B, (int)S, (int)H);
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous() && dout.sizes() == out.sizes() &&
                  dout.size(0) == B * S && dout.size(1) == H * kD && dout.scalar_type() == at::kBFloat16,
              "attention backward: dout / out must be contiguous [B*S, H*128] bf16");
  TORCH_CHECK(lse.is_contiguous() && lse.numel() == B * H * S, "attention backward: lse [B, H, S]");
  ensure_context();
  const int64_t T = B * S, HD = H * kD;
  auto dvec = at::empty({B, H, S}, lse.options());
  auto dq = at::zeros({T, HD}, lse.options());
  auto dqkv = at::empty({T, 3 * HD}, qkv.options());
  {
    const int64_t warps = T * H;
    const int threads = 256;
    attn_bwd_dot_kernel<<<(unsigned)((warps * 32 + threads - 1) / threads), threads, 0, cur_stream()>>>(
        (const bf16*)dout.data_ptr(), (const bf16*)out.data_ptr(), (int)HD, dvec.data_ptr<float>(), (int)B,
        (int)H, (int)S);
    MT_LAUNCH_CHECK();
  }
  const CUtensorMap tq = make_tma_2d(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3 * HD, T,
                                     qkv.stride(0), 64, kTile, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap td = make_tma_2d(dout.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, T, HD, 64, kTile,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kBwdSmem));
    attr = true;
  }
  const int grid = (int)(B * H * (S / kTile));
  attn_bwd_kernel<<<grid, kThreads, kBwdSmem, cur_stream()>>>(
      tq, td, lse.data_ptr<float>(), dvec.data_ptr<float>(), dq.data_ptr<float>(), (bf16*)dqkv.data_ptr(),
      (int)(3 * HD), (int)B, (int)H, (int)S, 1.0f / sqrtf((float)kD), attn_status_ptr());
  MT_LAUNCH_CHECK();
  {
    const int64_t n8 = T * HD / 8;
    attn_dq_cast_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, cur_stream()>>>(
        dq.data_ptr<float>(), (bf16*)dqkv.data_ptr(), (int)(3 * HD), (int)T, (int)HD);
    MT_LAUNCH_CHECK();
  }
  return dqkv;
}

int64_t attn_status(bool reset) {
  int h = 0;
  C10_CUDA_CHECK(cudaMemcpy(&h, attn_status_ptr(), sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) C10_CUDA_CHECK(cudaMemset(attn_status_ptr(), 0, sizeof(int)));
  return h;
}

}  // namespace mtorus
