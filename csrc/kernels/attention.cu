// Causal multi-head attention (flash attention) on tcgen05 for the fused GPT path.
//
// Reference semantics: scores = Q K^T / sqrt(d_head) + causal mask -> softmax ->
// dropout -> P V (examples/gpt-1b/src/transformer.rs:51-85, mask :163-171).  The
// dropout variant (DROP) draws the keep mask of probability (q, k) from Philox
// (philox.cuh; element ((b*H + h) * S + q) * S + k of the site) in the forward's
// softmax warps, which scale kept probabilities by 1 / (1 - p) in the P they hand
// to the PV MMA (the row sum and the log-sum-exp stay those of the undropped
// softmax), and draws it again in the backward: dV takes the dropped P^T and
// dS = P * (mask * dP / (1 - p) - D).  In the backward a thread owns a key and 64
// queries, so each lane of a warp computes the Philox block of one (query,
// 8-key group) and the warp exchanges the bits with shuffles.
// Layout: one [T, 3*H*128] bf16 matrix holds q | k | v for T = B*S tokens (heads
// contiguous inside each third), the output is [T, H*128]; S is a multiple of 128.
//
// Forward, one CTA per (two 128-query tiles, batch, head), heaviest pairs first:
//   warp 0      TMA producer: both Q tiles once, then K_0, V_0, K_1, ... into a
//               3-slot ring
//   warp 1      MMA issuer: S = Q K^T and O += P V for the two tiles in ping-pong
//               order, so the tensor core works on one tile while the other
//               tile's softmax runs
//   warps 2..9  two softmax warpgroups (one per query tile), one query row per
//               thread, read from TMEM; running max with lazy rescaling (O is
//               rescaled only when a row max grows by more than 2^8); P is written
//               as bf16 into shared memory in the 128B-swizzled K-major layout the
//               MMA reads; the epilogue divides by the row sum and stores O and
//               the log-sum-exp.
// Backward, one CTA per (128-key tile, batch, head), looping over query tiles i >= j:
//   S^T = K Q^T and dP^T = V dO^T into TMEM; two compute warpgroups (one column
//   half each) form P^T = exp(S^T*scale - lse) and dS^T = P^T (dP^T - D) * scale
//   in one shared-memory tile (P^T for the dV MMA, then dS^T for dK and dQ);
//   dV, dK accumulate in TMEM; dQ_i = dS K lands in TMEM (reusing the S^T columns)
//   and leaves through a shared staging area as TMA reduce-adds into an fp32 dQ
//   buffer.  The next dO / Q tiles load as soon as the dV / dK MMAs release them.
// D = rowsum(dO * O) (and the zeroing of dQ) comes from a small pre-kernel; a
// post-kernel casts dQ to bf16.
//
// Every wait is bounded (2 s); on a timeout the kernel records a status code,
// lets its in-flight copies and MMAs land, frees TMEM and returns.
#include "common.cuh"
#include "mx.cuh"
#include "philox.cuh"
#include "sm100.cuh"

#include <ATen/ops/zeros.h>

#include <cstring>

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

// ================================================================== forward
//
// One CTA per (256 consecutive queries = tiles A (upper) and B (lower), batch, head).
// TMEM: S_A | O_A | S_B | O_B (128 columns each).  Shared memory: Q_A, Q_B, a ring
// of three 32 KB slots that receives K_0, V_0, K_1, V_1, ... in order, P_A, P_B.
// MMA order: S_A0 S_B0 | PV_A0 S_A1 PV_B0 S_B1 | PV_A1 S_A2 ... so the tensor core
// works on one tile while the other tile's softmax warps run.
constexpr int kRing = 3;
constexpr int kFwdThreads = 320;  // producer, MMA, 2 x 4 softmax warps

// MXFP8 copy of the attention output (the out-projection's operand both ways): row codes
// [T, H*128] and column codes [H*128, T] with their scale atoms (the mx_quantize layout),
// written by the forward's epilogue beside the bf16 output.  rc == nullptr: none.
struct AttnMxOut {
  uint8_t* rc;
  uint8_t* rsf;
  uint8_t* cc;
  uint8_t* csf;
  uint32_t fmax_bits;
  int fmt;
};

struct FwdCtl {
  uint64_t q_full, ring_full[kRing], ring_empty[kRing], s_full[2], p_full[2], o_done[2], drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two values).
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}


template <bool DROP>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tma_qkv, bf16* __restrict__ out, int ld_out,
                    float* __restrict__ lse, int B, int H, int S, float scale, int* status, DropoutArgs drop,
                    AttnMxOut mxo) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;                        // tile g at g * 32K (g = 0: A, 1: B)
  uint8_t* sRing = smem + 2 * kTileBytes;     // slot s at s * 32K
  uint8_t* sP = smem + 5 * kTileBytes;        // tile g at g * 32K
  FwdCtl* ctl = reinterpret_cast<FwdCtl*>(smem + 7 * kTileBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = S / kTile;
  const int npair = (nq + 1) / 2;
  const int bh = blockIdx.x / npair;
  const int pair = blockIdx.x % npair;        // heaviest first within a head
  const int b = bh / H, h = bh % H;
  const int qtA = nq - 1 - 2 * pair, qtB = qtA - 1;  // qtB = -1: no tile B (odd tile count)
  const int nkv = qtA + 1;                     // tile B uses tiles 0 .. nkv-2

  if (threadIdx.x == 0) {
    mbar_init(&ctl->q_full, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&ctl->ring_full[s], 1);
      mbar_init(&ctl->ring_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&ctl->s_full[g], 1);
      mbar_init(&ctl->p_full[g], 128);
      mbar_init(&ctl->o_done[g], 1);
    }
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
  volatile int* abort = &ctl->abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      const int qcol = h * kD, kcol = H * kD + h * kD, vcol = 2 * H * kD + h * kD;
      mbar_arrive_expect_tx(&ctl->q_full, 2 * kTileBytes);
      for (int g = 0; g < 2; ++g) {
        const int r0 = b * S + max(g == 0 ? qtA : qtB, 0) * kTile;  // an absent tile B loads tile 0, unused
        tma_load_2d(sQ + g * kTileBytes, &tma_qkv, &ctl->q_full, qcol, r0);
        tma_load_2d(sQ + g * kTileBytes + kHalf, &tma_qkv, &ctl->q_full, qcol + 64, r0);
      }
      uint32_t issued = 0, par = 0;
      for (int n = 0; n < 2 * nkv && !*abort; ++n) {  // n = 2j: K_j, 2j+1: V_j
        const int s = n % kRing, use = n / kRing;
        if (use > 0 && !mbar_wait(&ctl->ring_empty[s], (use - 1) & 1, abort, status, 11)) break;
        const int col = (n & 1) ? vcol : kcol;
        const int r0 = b * S + (n >> 1) * kTile;
        uint8_t* dst = sRing + s * kTileBytes;
        issued |= 1u << s;
        par = (par & ~(1u << s)) | (((uint32_t)use & 1u) << s);
        mbar_arrive_expect_tx(&ctl->ring_full[s], kTileBytes);
        tma_load_2d(dst, &tma_qkv, &ctl->ring_full[s], col, r0);
        tma_load_2d(dst + kHalf, &tma_qkv, &ctl->ring_full[s], col + 64, r0);
      }
      if (*abort) {
        bounded_drain(&ctl->q_full, 0);
        for (int s = 0; s < kRing; ++s)
          if (issued >> s & 1u) bounded_drain(&ctl->ring_full[s], (par >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t idS = make_idesc_bf16(kTile, kTile, 0, 0);
      const uint32_t idO = make_idesc_bf16(kTile, kD, 0, 1);
      bool issued_any = false;
      bool ok = mbar_wait(&ctl->q_full, 0, abort, status, 12);
      auto ring_wait = [&](int n) -> bool {
        const int s = n % kRing;
        if (!mbar_wait(&ctl->ring_full[s], (n / kRing) & 1, abort, status, 13)) return false;
        tc_fence_after();
        return true;
      };
      // S_g(j) = Q_g K_j^T; K_j's slot is released after the last tile that needs it
      auto issue_s = [&](int g, int j) {
        const uint32_t q = smem_u32(sQ + g * kTileBytes);
        const uint32_t k = smem_u32(sRing + ((2 * j) % kRing) * kTileBytes);
        const uint32_t d = tmem + g * 256;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          umma_f16(d, desc_kmajor(q, kk), desc_kmajor(k, kk), idS, kk > 0 ? 1u : 0u);
        umma_commit(&ctl->s_full[g]);
        issued_any = true;
      };
      auto issue_pv = [&](int g, int j) {
        const uint32_t p = smem_u32(sP + g * kTileBytes);
        const uint32_t v = smem_u32(sRing + ((2 * j + 1) % kRing) * kTileBytes);
        const uint32_t d = tmem + g * 256 + 128;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_f16(d, desc_kmajor(p, kk), desc_mnmajor(v, kk), idO, (j | kk) != 0 ? 1u : 0u);
        umma_commit(&ctl->o_done[g]);
      };
      // prologue: S_A(0), S_B(0)
      if (ok && (ok = ring_wait(0))) {
        issue_s(0, 0);
        if (nkv - 1 > 0) issue_s(1, 0);
        umma_commit(&ctl->ring_empty[0]);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const bool b_needs = j < nkv - 1;  // tile B uses KV tiles 0 .. nkv-2
        if (!(ok = ring_wait(2 * j + 1))) break;  // V_j
        // A: PV_A(j), then S_A(j+1)
        if (!(ok = mbar_wait(&ctl->p_full[0], j & 1, abort, status, 14))) break;
        tc_fence_after();
        issue_pv(0, j);
        const bool more = j + 1 < nkv;
        if (more) {
          if (!(ok = ring_wait(2 * j + 2))) break;  // K_{j+1}
          issue_s(0, j + 1);
        }
        // B: PV_B(j), then S_B(j+1)
        if (b_needs) {
          if (!(ok = mbar_wait(&ctl->p_full[1], j & 1, abort, status, 15))) break;
          tc_fence_after();
          issue_pv(1, j);
          if (j + 1 < nkv - 1) issue_s(1, j + 1);
        }
        umma_commit(&ctl->ring_empty[(2 * j + 1) % kRing]);  // V_j
        if (more) umma_commit(&ctl->ring_empty[(2 * j + 2) % kRing]);  // K_{j+1}
      }
      if (*abort && issued_any) {
        umma_commit(&ctl->drain);
        bounded_drain(&ctl->drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax
    const int g = (warp - 2) >> 2;            // 0: tile A (warps 2-5), 1: tile B (warps 6-9)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;        // query row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + g * 256 + lane_off, tO = tS + 128;
    const int qt = g == 0 ? qtA : qtB;
    const int n = g == 0 ? nkv : nkv - 1;
    uint8_t* myP = sP + g * kTileBytes;
    const float sl2 = scale * kLog2e;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      // dropout keep bits of this row's 128 keys of tile j (bit 8*c16 + e of word c16/4),
      // drawn before the scores arrive so the Philox rounds overlap the S MMA
      uint32_t keepw[4] = {0u, 0u, 0u, 0u};
      if constexpr (DROP) {
        const uint64_t grp0 = ((uint64_t)bh * S + qt * kTile + r) * (uint64_t)(S / 8) + j * (kTile / 8);
#pragma unroll
        for (int c16 = 0; c16 < kTile / 8; ++c16)
          keepw[c16 >> 2] |= dropout_keep8(drop.rng[0], drop.rng[1], drop.site, grp0 + c16, drop.thr16)
                             << ((c16 & 3) * 8);
      }
      if (!mbar_wait(&ctl->s_full[g], j & 1, abort, status, 16)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t t[kTile];  // raw scores, loaded straight into the row's registers
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&t[c * 32]));
      tmem_wait_ld();
      if (j == qt) {  // diagonal tile: keys after the query are masked
#pragma unroll
        for (int e = 0; e < kTile; ++e)
          if (e > r) t[e] = __float_as_uint(-INFINITY);
      }
      // row max as 8 independent chains (a single 128-long chain of dependent max
      // operations costs ~4 cycles each on the critical path)
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = __uint_as_float(t[k]);
#pragma unroll
      for (int e = 8; e < kTile; e += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmaxf(m8[k], __uint_as_float(t[e + k]));
      float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      mx *= sl2;
      float alpha = 1.f;
      if (j == 0) {
        m_ref = mx;
      } else if (mx > m_ref + kRescale) {
        alpha = ex2_approx(m_ref - mx);
        m_ref = mx;
      }
      if (j > 0) {  // O and P_g are free once PV_g(j-1) has completed
        if (!mbar_wait(&ctl->o_done[g], (j - 1) & 1, abort, status, 17)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      l *= alpha;
      // 8 independent partial row sums as 4 packed pairs; scores scaled on pairs (f32x2)
      uint64_t s8[4] = {0ull, 0ull, 0ull, 0ull};
      const float neg = -m_ref;
      const uint64_t sl2p = f2pack(sl2, sl2), negp = f2pack(neg, neg);
#pragma unroll
      for (int c16 = 0; c16 < kTile / 8; ++c16) {
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float a0, a1;
          f2unpack(fma2(f2pack(__uint_as_float(t[c16 * 8 + e]), __uint_as_float(t[c16 * 8 + e + 1])), sl2p, negp),
                   a0, a1);
          pv[e] = ex2_approx(a0);
          pv[e + 1] = ex2_approx(a1);
          s8[e / 2] = add2(s8[e / 2], f2pack(pv[e], pv[e + 1]));
        }
        if constexpr (DROP) {  // keys j*128 + 8*c16 .. +7 of query row qt*128 + r
          const uint32_t keep = keepw[c16 >> 2] >> ((c16 & 3) * 8);
#pragma unroll
          for (int e = 0; e < 8; ++e) pv[e] = (keep >> e & 1u) ? pv[e] * drop.scale : 0.f;
        }
        uint4 w;
        w.x = pack_bf16x2(pv[0], pv[1]);
        w.y = pack_bf16x2(pv[2], pv[3]);
        w.z = pack_bf16x2(pv[4], pv[5]);
        w.w = pack_bf16x2(pv[6], pv[7]);
        *reinterpret_cast<uint4*>(myP + sw128_chunk(r, c16)) = w;
      }
      float sp[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) f2unpack(s8[k], sp[2 * k], sp[2 * k + 1]);
      l += ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
      // rescale O (rows whose max grew) before PV_g(j) accumulates into it
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tO + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          tmem_st32(tO + c * 32, v);
        }
        tmem_wait_st();
      }
      fence_async_shared();
      tc_fence_before();
      mbar_arrive(&ctl->p_full[g]);
    }
    if (ok && n > 0 && mbar_wait(&ctl->o_done[g], (n - 1) & 1, abort, status, 18)) {
      tc_fence_after();
      const float inv = 1.f / l;
      const int row = b * S + qt * kTile + r;
      bf16* dst = out + (size_t)row * ld_out + h * kD;
      // MX output: this warp's 32 rows x 32 columns per chunk go through a 2 KB staging
      // area in the warpgroup's P tile (free: every PV MMA of the tile has completed)
      uint8_t* stg = myP + quarter * 2048;
      const int T = B * S, row0w = b * S + qt * kTile + quarter * 32;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tO + c * 32, v);
        tmem_wait_ld();
        uint4 wv[4];
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(v[e]) * inv, __uint_as_float(v[e + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(v[e + 2]) * inv, __uint_as_float(v[e + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(v[e + 4]) * inv, __uint_as_float(v[e + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(v[e + 6]) * inv, __uint_as_float(v[e + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + c * 32 + e) = w;
          wv[e / 8] = w;
        }
        if (mxo.rc) {
          const int ef = (int)((mxo.fmax_bits >> 23) & 0xFF);
          const uint32_t mf = mxo.fmax_bits & 0x7FFFFF;
          const int col0 = h * kD + c * 32;  // first column of the chunk in [T, H*128]
          float f[32];
#pragma unroll
          for (int q = 0; q < 4; ++q) unpack8(*reinterpret_cast<const bf16x8*>(&wv[q]), f + 8 * q);
          uint32_t cw[8];
          uint8_t sb;
          mx_block(f, ef, mf, mxo.fmt, cw, sb);  // this row's block (the bf16 values just stored)
          uint4* rdst = reinterpret_cast<uint4*>(mxo.rc + (size_t)row * ld_out + col0);
          rdst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
          rdst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
          mxo.rsf[((int64_t)(row >> 7) * H + h) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + c] = sb;
          // column block: stage the 32 x 32 bf16 chunk, then each lane quantises column col0 + lane
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(stg + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = wv[q];
          __syncwarp();
#pragma unroll
          for (int rr = 0; rr < 32; ++rr)
            f[rr] = __bfloat162float(*reinterpret_cast<const bf16*>(
                stg + rr * 64 + ((((lane >> 3) ^ ((rr >> 1) & 3))) << 4) + (lane & 7) * 2));
          __syncwarp();  // the staging area is rewritten by the next chunk
          mx_block(f, ef, mf, mxo.fmt, cw, sb);
          const int col = col0 + lane;
          uint4* cdst = reinterpret_cast<uint4*>(mxo.cc + (size_t)col * T + row0w);
          cdst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
          cdst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
          mxo.csf[((int64_t)(col >> 7) * (T >> 7) + (row0w >> 7)) * 512 + (col & 31) * 16 + ((col & 127) >> 5) * 4 +
                  ((row0w & 127) >> 5)] = sb;
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
//
// One CTA per (128-key tile j, batch, head) looping over query tiles i = j .. nt-1.
// Shared memory: K, V, Q / dO of the current query tile, one tile that first holds
// P^T (read by the dV MMA) and then dS^T (read by the dK and dQ MMAs), and a 64 KB
// fp32 staging area from which dQ_i leaves as four [128 x 32] TMA reduce-adds into
// the fp32 dQ buffer (full-line reductions in L2 instead of scattered atomics).
// TMEM: S^T | dP^T | dV | dK; dQ_i reuses S^T.
struct BwdCtl {
  uint64_t kv_full, q_full, q_empty, do_full, do_empty, st_full, p_ready, pv_done, ds_ready, dq_full, dq_free,
      kv_done, drain;
  uint32_t tmem_base;
  int abort;
  alignas(16) float lse[kTile];
  alignas(16) float dd[kTile];
};

constexpr int kBwdThreads = 320;  // producer, MMA, 2 x 4 compute warps (column halves)

template <bool DROP>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tma_qkv, const __grid_constant__ CUtensorMap tma_do,
                    const __grid_constant__ CUtensorMap tma_dq,
                    const float* __restrict__ lse, const float* __restrict__ dvec,
                    bf16* __restrict__ dqkv, int ld_dqkv, int B, int H, int S, float scale, int* status,
                    DropoutArgs drop) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sK = smem;
  uint8_t* sV = smem + kTileBytes;
  uint8_t* sQ = smem + 2 * kTileBytes;
  uint8_t* sDO = smem + 3 * kTileBytes;
  uint8_t* sPS = smem + 4 * kTileBytes;    // P^T, then dS^T
  uint8_t* sDQ = smem + 5 * kTileBytes;    // 4 x [128 rows x 128 B] fp32 boxes, SW128
  BwdCtl* ctl = reinterpret_cast<BwdCtl*>(smem + 7 * kTileBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = S / kTile;
  const int bh = blockIdx.x / nt;
  const int kt = blockIdx.x % nt;        // key tile; tile 0 loops over every query tile
  const int b = bh / H, h = bh % H;
  const int nqi = nt - kt;               // query tiles i = kt .. nt-1
  const int krow0 = b * S + kt * kTile;

  if (threadIdx.x == 0) {
    mbar_init(&ctl->kv_full, 1);
    mbar_init(&ctl->q_full, 1);
    mbar_init(&ctl->q_empty, 1);
    mbar_init(&ctl->do_full, 1);
    mbar_init(&ctl->do_empty, 1);
    mbar_init(&ctl->st_full, 1);
    mbar_init(&ctl->p_ready, 256);
    mbar_init(&ctl->pv_done, 1);
    mbar_init(&ctl->ds_ready, 256);
    mbar_init(&ctl->dq_full, 1);
    mbar_init(&ctl->dq_free, 256);
    mbar_init(&ctl->kv_done, 1);
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_qkv);
    tma_prefetch_desc(&tma_do);
    tma_prefetch_desc(&tma_dq);
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
      // dO of the next query tile loads as soon as the dV MMA has read this one, Q as
      // soon as the dK MMA has: both overlap the dS math and the dQ MMA / read-out
      int issued_q = -1, issued_do = -1;
      for (int it = 0; it < nqi && !*abort; ++it) {
        const int qr = b * S + (kt + it) * kTile;
        if (it > 0 && !mbar_wait(&ctl->do_empty, (it - 1) & 1, abort, status, 21)) break;
        issued_do = it;
        mbar_arrive_expect_tx(&ctl->do_full, kTileBytes);
        tma_load_2d(sDO, &tma_do, &ctl->do_full, h * kD, qr);
        tma_load_2d(sDO + kHalf, &tma_do, &ctl->do_full, h * kD + 64, qr);
        if (it > 0 && !mbar_wait(&ctl->q_empty, (it - 1) & 1, abort, status, 20)) break;
        issued_q = it;
        mbar_arrive_expect_tx(&ctl->q_full, kTileBytes);
        tma_load_2d(sQ, &tma_qkv, &ctl->q_full, qcol, qr);
        tma_load_2d(sQ + kHalf, &tma_qkv, &ctl->q_full, qcol + 64, qr);
      }
      if (*abort) {
        bounded_drain(&ctl->kv_full, 0);
        if (issued_q >= 0) bounded_drain(&ctl->q_full, issued_q & 1);
        if (issued_do >= 0) bounded_drain(&ctl->do_full, issued_do & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t id_kk = make_idesc_bf16(kTile, kTile, 0, 0);  // A, B K-major
      const uint32_t id_kn = make_idesc_bf16(kTile, kD, 0, 1);     // A K-major, B MN-major
      const uint32_t id_mn = make_idesc_bf16(kTile, kD, 1, 1);     // A, B MN-major
      const uint32_t k = smem_u32(sK), v = smem_u32(sV), ps = smem_u32(sPS);
      bool issued_any = false;
      bool ok = mbar_wait(&ctl->kv_full, 0, abort, status, 22);
      const uint32_t q = smem_u32(sQ), dO = smem_u32(sDO);
      for (int it = 0; it < nqi && ok; ++it) {
        if (!mbar_wait(&ctl->q_full, it & 1, abort, status, 23)) break;
        if (!mbar_wait(&ctl->do_full, it & 1, abort, status, 19)) break;
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
        if (!mbar_wait(&ctl->p_ready, it & 1, abort, status, 25)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dV += P^T dO
          umma_f16(tDV, desc_kmajor(ps, kk), desc_mnmajor(dO, kk), id_kn, (it | kk) != 0 ? 1u : 0u);
        umma_commit(&ctl->pv_done);
        umma_commit(&ctl->do_empty);  // dO is read by dP^T and dV only
        if (!mbar_wait(&ctl->ds_ready, it & 1, abort, status, 29)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dK += dS^T Q
          umma_f16(tDK, desc_kmajor(ps, kk), desc_mnmajor(q, kk), id_kn, (it | kk) != 0 ? 1u : 0u);
        umma_commit(&ctl->q_empty);  // Q is read by S^T and dK only
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)  // dQ_i = dS K
          umma_f16(tDQ, desc_mnmajor(ps, kk), desc_mnmajor(k, kk), id_mn, kk > 0 ? 1u : 0u);
        umma_commit(&ctl->dq_full);
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
    const int ch = (warp - 2) >> 2;     // column half: 0 (warps 2-5) or 1 (warps 6-9)
    const int r = quarter * 32 + lane;  // key row (S^T, dP^T, dV, dK) or query row (dQ)
    const int tid = threadIdx.x - 64;   // 0 .. 255
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = scale * kLog2e;
    bool ok = true;
    // the tile's log-sum-exp (log2 units; threads 0-127) and D (threads 128-255), fetched a tile ahead
    const float* src = tid < kTile ? lse : dvec;
    const float mul = tid < kTile ? -kLog2e : 1.f;  // smem holds -lse (log2 units) and D
    float* dst = tid < kTile ? ctl->lse : ctl->dd;
    const int ti = tid & (kTile - 1);
    float next = src[(size_t)bh * S + kt * kTile + ti] * mul;
    for (int it = 0; it < nqi; ++it) {
      const int qi = kt + it;
      // every thread read the previous tile's values before arriving on p_ready,
      // which the MMA of that tile (and so dq_full, waited below) depends on
      dst[ti] = next;
      if (it + 1 < nqi) next = src[(size_t)bh * S + (qi + 1) * kTile + ti] * mul;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const float* sl = ctl->lse;
      const float* sd = ctl->dd;
      if (!mbar_wait(&ctl->st_full, it & 1, abort, status, 26)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = qi == kt;
      uint32_t dsp[32];  // this thread's 64 dS^T values as bf16 pairs, stored after the dV MMA
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = ch * 2 + cc;
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + lane_off + c * 32, sv);
        tmem_ld32(tDP + lane_off + c * 32, dv);
        tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float p[8], ds[8];
          uint32_t kb = 0;
          if constexpr (DROP) {
            // this lane's Philox block: query c*32 + 8g + lane/4, keys of 8-group (warp's 32 keys)/8 + lane%4
            const int qq = qi * kTile + c * 32 + g * 8 + (lane >> 2);
            const uint64_t grp = ((uint64_t)bh * S + qq) * (uint64_t)(S / 8) + (kt * kTile + quarter * 32) / 8 +
                                 (lane & 3);
            kb = dropout_keep8(drop.rng[0], drop.rng[1], drop.site, grp, drop.thr16);
          }
          if constexpr (DROP) {
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              const int e = g * 8 + x, col = c * 32 + e;  // query within the tile
              float pe = ex2_approx(fmaf(__uint_as_float(sv[e]), sl2, sl[col]));
              if (diag && col < r) pe = 0.f;  // query before key: masked in the forward
              // the key bit of query e sits in the block of lane 4x + (key's 8-group within the warp)
              const bool keep = (__shfl_sync(0xffffffffu, kb, x * 4 + (lane >> 3)) >> (lane & 7)) & 1u;
              p[x] = keep ? pe * drop.scale : 0.f;
              ds[x] = pe * ((keep ? __uint_as_float(dv[e]) * drop.scale : 0.f) - sd[col]) * scale;
            }
          } else {
            // the same on value pairs: vector loads of -lse / D, packed f32x2 arithmetic
            const int col0 = c * 32 + g * 8;
            const float4 la = *reinterpret_cast<const float4*>(sl + col0);
            const float4 lb = *reinterpret_cast<const float4*>(sl + col0 + 4);
            const float4 da = *reinterpret_cast<const float4*>(sd + col0);
            const float4 db = *reinterpret_cast<const float4*>(sd + col0 + 4);
            const float lv[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
            const float dd8[8] = {da.x, da.y, da.z, da.w, db.x, db.y, db.z, db.w};
            const uint64_t s2 = f2pack(sl2, sl2), sc2 = f2pack(scale, scale);
#pragma unroll
            for (int x = 0; x < 8; x += 2) {
              const int e = g * 8 + x, col = col0 + x;
              float a0, a1;
              f2unpack(fma2(f2pack(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), s2, f2pack(lv[x], lv[x + 1])),
                       a0, a1);
              float pe0 = ex2_approx(a0), pe1 = ex2_approx(a1);
              if (diag) {  // queries before the key: masked in the forward
                if (col < r) pe0 = 0.f;
                if (col + 1 < r) pe1 = 0.f;
              }
              p[x] = pe0;
              p[x + 1] = pe1;
              const uint64_t q = sub2(f2pack(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])),
                                      f2pack(dd8[x], dd8[x + 1]));
              f2unpack(mul2(mul2(f2pack(pe0, pe1), sc2), q), ds[x], ds[x + 1]);
            }
          }
          uint4 wp;
          wp.x = pack_bf16x2(p[0], p[1]);
          wp.y = pack_bf16x2(p[2], p[3]);
          wp.z = pack_bf16x2(p[4], p[5]);
          wp.w = pack_bf16x2(p[6], p[7]);
          *reinterpret_cast<uint4*>(sPS + sw128_chunk(r, c * 4 + g)) = wp;
#pragma unroll
          for (int x = 0; x < 4; ++x) dsp[(cc * 32 + g * 8) / 2 + x] = pack_bf16x2(ds[2 * x], ds[2 * x + 1]);
        }
      }
      fence_async_shared();
      tc_fence_before();
      mbar_arrive(&ctl->p_ready);
      // dS^T replaces P^T once the dV MMA has read it
      if (!mbar_wait(&ctl->pv_done, it & 1, abort, status, 30)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c16 = 0; c16 < 8; ++c16) {
        uint4 w;
        w.x = dsp[c16 * 4 + 0];
        w.y = dsp[c16 * 4 + 1];
        w.z = dsp[c16 * 4 + 2];
        w.w = dsp[c16 * 4 + 3];
        *reinterpret_cast<uint4*>(sPS + sw128_chunk(r, ch * 8 + c16)) = w;
      }
      fence_async_shared();
      tc_fence_before();
      mbar_arrive(&ctl->ds_ready);
      if (!mbar_wait(&ctl->dq_full, it & 1, abort, status, 27)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // the previous tile's reduce-adds must have read the staging boxes of this half
      const bool leader = (quarter == 0 && lane == 0);  // one thread per column half
      if (leader) bulk_wait_group_read<0>();
      asm volatile("bar.sync %0, 128;" ::"r"(2 + ch) : "memory");
#pragma unroll 1
      for (int c = ch * 2; c < ch * 2 + 2; ++c) {
        uint32_t v[32];
        tmem_ld32(tDQ + lane_off + c * 32, v);
        tmem_wait_ld();
        uint8_t* box = sDQ + c * kHalf;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<uint4*>(box + r * 128 + ((k ^ (r & 7)) << 4)) =
              make_uint4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      }
      tc_fence_before();
      mbar_arrive(&ctl->dq_free);
      fence_async_shared();
      asm volatile("bar.sync %0, 128;" ::"r"(2 + ch) : "memory");
      if (leader) {
        const int y = b * S + qi * kTile;
        tma_reduce_add_2d(&tma_dq, sDQ + (ch * 2) * kHalf, h * kD + ch * 64, y);
        tma_reduce_add_2d(&tma_dq, sDQ + (ch * 2 + 1) * kHalf, h * kD + ch * 64 + 32, y);
        bulk_commit_group();
      }
    }
    if ((quarter == 0 && lane == 0)) bulk_wait_group<0>();  // dQ reductions complete before exit
    if (ok && mbar_wait(&ctl->kv_done, 0, abort, status, 28)) {
      tc_fence_after();
      // dK and dV rows of this key tile -> the k and v thirds of dqkv
      bf16* dk = dqkv + (size_t)(krow0 + r) * ld_dqkv + H * kD + h * kD;
      bf16* dvp = dqkv + (size_t)(krow0 + r) * ld_dqkv + 2 * H * kD + h * kD;
#pragma unroll 1
      for (int c = ch * 2; c < ch * 2 + 2; ++c) {
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

// D[bh, s] = sum_c dO[t, h*128 + c] * O[t, h*128 + c], with 16 threads per (token,
// head) row and 16-byte loads; the same threads zero that row's slice of the fp32
// dQ accumulator, which the backward kernel then reduces into.
__global__ void attn_bwd_dot_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ o, int ld,
                                    float* __restrict__ dvec, float* __restrict__ dq, int B, int H, int S) {
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long row = g >> 4;  // (token, head)
  const int sub = threadIdx.x & 15;
  const long long total = (long long)B * S * H;
  if (row >= total) return;
  const long long t = row / H;
  const int h = (int)(row % H);
  const size_t off = (size_t)t * ld + h * kD + sub * 8;
  const uint4 ua = *reinterpret_cast<const uint4*>(dout + off);
  const uint4 uc = *reinterpret_cast<const uint4*>(o + off);
  float fa[8], fc[8];
  unpack8(*reinterpret_cast<const bf16x8*>(&ua), fa);
  unpack8(*reinterpret_cast<const bf16x8*>(&uc), fc);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc += fa[i] * fc[i];
#pragma unroll
  for (int m = 8; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
  float4* z = reinterpret_cast<float4*>(dq + off);
  z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (sub == 0) {
    const long long b = t / S, s = t % S;
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

constexpr size_t kFwdSmem = 7 * kTileBytes + sizeof(FwdCtl) + 1024;
constexpr size_t kBwdSmem = 7 * kTileBytes + sizeof(BwdCtl) + 1024;

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
DropoutArgs make_dropout_args(const c10::optional<at::Tensor>& rng, int64_t site, int64_t thr16, double scale);

// mx_* (optional, all four or none): also write the output's MXFP8 row codes [B*S, H*128] /
// mx_rsf and column codes [H*128, B*S] / mx_csf in format mx_fmt (largest value mx_fmax).
std::vector<at::Tensor> attn_fwd(const at::Tensor& qkv, int64_t B, int64_t S, int64_t H,
                                 const c10::optional<at::Tensor>& drop_rng, int64_t drop_site, int64_t drop_thr16,
                                 double drop_scale, const c10::optional<at::Tensor>& mx_rc,
                                 const c10::optional<at::Tensor>& mx_rsf, const c10::optional<at::Tensor>& mx_cc,
                                 const c10::optional<at::Tensor>& mx_csf, int64_t mx_fmt, double mx_fmax) {
  check_qkv(qkv, (int)B, (int)S, (int)H);
  ensure_context();
  AttnMxOut mxo{};
  if (mx_rc.has_value()) {
    const int64_t n = B * S * H * kD, atoms = (B * S / kTile) * H * 512;
    auto chk = [](const c10::optional<at::Tensor>& t, int64_t numel, const char* what) {
      TORCH_CHECK(t.has_value() && t->is_cuda() && t->element_size() == 1 && t->is_contiguous() &&
                      t->numel() == numel && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                  what);
    };
    chk(mx_rc, n, "attention MX output: rc must be 16-byte aligned contiguous uint8 [B*S, H*128]");
    chk(mx_cc, n, "attention MX output: cc must be 16-byte aligned contiguous uint8 [H*128, B*S]");
    chk(mx_rsf, atoms, "attention MX output: rsf size");
    chk(mx_csf, atoms, "attention MX output: csf size");
    TORCH_CHECK(mx_fmt == 0 || mx_fmt == 1, "attention MX output: format 0 (E4M3) / 1 (E5M2)");
    const float fm = (float)mx_fmax;
    std::memcpy(&mxo.fmax_bits, &fm, 4);
    mxo.rc = reinterpret_cast<uint8_t*>(mx_rc->data_ptr());
    mxo.rsf = reinterpret_cast<uint8_t*>(mx_rsf->data_ptr());
    mxo.cc = reinterpret_cast<uint8_t*>(mx_cc->data_ptr());
    mxo.csf = reinterpret_cast<uint8_t*>(mx_csf->data_ptr());
    mxo.fmt = (int)mx_fmt;
  }
  auto out = at::empty({B * S, H * kD}, qkv.options());
  auto lse = at::empty({B, H, S}, qkv.options().dtype(at::kFloat));
  const CUtensorMap tm = make_tma_2d(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3 * H * kD, B * S,
                                     qkv.stride(0), 64, kTile, CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kFwdSmem));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kFwdSmem));
    attr = true;
  }
  const DropoutArgs drop = make_dropout_args(drop_rng, drop_site, drop_thr16, drop_scale);
  const int grid = (int)(B * H * ((S / kTile + 1) / 2));
  if (drop.rng)
    attn_fwd_kernel<true><<<grid, kFwdThreads, kFwdSmem, cur_stream()>>>(
        tm, (bf16*)out.data_ptr(), (int)(H * kD), lse.data_ptr<float>(), (int)B, (int)H, (int)S,
        1.0f / sqrtf((float)kD), attn_status_ptr(), drop, mxo);
  else
    attn_fwd_kernel<false><<<grid, kFwdThreads, kFwdSmem, cur_stream()>>>(
        tm, (bf16*)out.data_ptr(), (int)(H * kD), lse.data_ptr<float>(), (int)B, (int)H, (int)S,
        1.0f / sqrtf((float)kD), attn_status_ptr(), drop, mxo);
  MT_LAUNCH_CHECK();
  return {out, lse};
}

// -> dqkv [B*S, 3*H*128] bf16 (dq | dk | dv)
// dq_out (optional fp32 [B*S, H*128]): receives the fp32 dQ accumulator, and the q third
// of the returned dqkv is left unwritten (for a consumer that reads dQ in fp32, e.g. the
// MXFP8 row / column quantiser); without it dQ is cast into that third.
at::Tensor attn_bwd(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& lse,
                    int64_t B, int64_t S, int64_t H, const c10::optional<at::Tensor>& drop_rng, int64_t drop_site,
                    int64_t drop_thr16, double drop_scale, const c10::optional<at::Tensor>& dq_out) {
  check_qkv(qkv, (int)B, (int)S, (int)H);
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous() && dout.sizes() == out.sizes() &&
                  dout.size(0) == B * S && dout.size(1) == H * kD && dout.scalar_type() == at::kBFloat16,
              "attention backward: dout / out must be contiguous [B*S, H*128] bf16");
  TORCH_CHECK(lse.is_contiguous() && lse.numel() == B * H * S, "attention backward: lse [B, H, S]");
  ensure_context();
  const int64_t T = B * S, HD = H * kD;
  auto dvec = at::empty({B, H, S}, lse.options());
  if (dq_out.has_value())
    TORCH_CHECK(dq_out->scalar_type() == at::kFloat && dq_out->is_contiguous() && dq_out->numel() == T * HD &&
                    reinterpret_cast<uintptr_t>(dq_out->data_ptr()) % 16 == 0,
                "attention backward: dq_out must be contiguous fp32 [B*S, H*128]");
  auto dq = dq_out.has_value() ? *dq_out : at::empty({T, HD}, lse.options());  // zeroed by the dot kernel
  auto dqkv = at::empty({T, 3 * HD}, qkv.options());
  {
    const int64_t threads_total = T * H * 16;
    const int threads = 256;
    attn_bwd_dot_kernel<<<(unsigned)((threads_total + threads - 1) / threads), threads, 0, cur_stream()>>>(
        (const bf16*)dout.data_ptr(), (const bf16*)out.data_ptr(), (int)HD, dvec.data_ptr<float>(),
        dq.data_ptr<float>(), (int)B, (int)H, (int)S);
    MT_LAUNCH_CHECK();
  }
  const CUtensorMap tq = make_tma_2d(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3 * HD, T,
                                     qkv.stride(0), 64, kTile, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap td = make_tma_2d(dout.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, HD, T, HD, 64, kTile,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tdq = make_tma_2d(dq.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, HD, T, HD, 32, kTile,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kBwdSmem));
    C10_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kBwdSmem));
    attr = true;
  }
  const DropoutArgs drop = make_dropout_args(drop_rng, drop_site, drop_thr16, drop_scale);
  const int grid = (int)(B * H * (S / kTile));
  if (drop.rng)
    attn_bwd_kernel<true><<<grid, kBwdThreads, kBwdSmem, cur_stream()>>>(
        tq, td, tdq, lse.data_ptr<float>(), dvec.data_ptr<float>(), (bf16*)dqkv.data_ptr(),
        (int)(3 * HD), (int)B, (int)H, (int)S, 1.0f / sqrtf((float)kD), attn_status_ptr(), drop);
  else
    attn_bwd_kernel<false><<<grid, kBwdThreads, kBwdSmem, cur_stream()>>>(
        tq, td, tdq, lse.data_ptr<float>(), dvec.data_ptr<float>(), (bf16*)dqkv.data_ptr(),
        (int)(3 * HD), (int)B, (int)H, (int)S, 1.0f / sqrtf((float)kD), attn_status_ptr(), drop);
  MT_LAUNCH_CHECK();
  if (!dq_out.has_value()) {
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
