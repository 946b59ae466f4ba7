// Persistent, warp-specialised GEMMs on the 5th-generation tensor cores.
//
//   D[M,N] = epilogue( alpha * A[M,K] . B[N,K]^T )
//
// Variants: bf16 (kind::f16; a 1-SM kernel for M < 256 and the CTA-pair kernel),
// per-tensor-scaled FP8 E4M3 / E5M2 (kind::f8f6f4, CTA pair), MXFP8 with 1x32
// UE8M0 block scales (kind::mxf8f6f4.block_scale, CTA pair), and a B operand
// sharded by rows across ranks and read from its owners (gemm_fp8_gather_b).
//
// Replaces the Burn NdArray matmuls of every Linear layer of the GPT example
// (examples/gpt-1b/src/transformer.rs:34-37,54-56,84,99-100,106,109; model.rs:89,128)
// for the forward (both operands K-major), dgrad (B N-major) and wgrad (A and B
// MN-major) products.
//
// Design (sm_100a):
//   * one CTA per SM, static persistent tile loop with grouped rasterisation so
//     concurrently running tiles share A/B panels in L2;
//   * warp 0: TMA producer (128B-swizzled boxes, STAGES-deep smem ring);
//   * warp 1: allocates TMEM and issues tcgen05.mma (M=128, N=256, K=16) from
//     one thread, committing smem slots back to the producer;
//   * warps 2-5: epilogue; each warp reads its 32 TMEM lanes with tcgen05.ld and
//     applies alpha / bias / residual / GELU / dGELU / fp32 accumulate in registers;
//   * two TMEM accumulators (2 x 256 columns) so the epilogue of tile i overlaps
//     the main loop of tile i+1.
// All mbarrier waits are bounded (see sm100.cuh); a timeout raises the status word.
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "amax_publish.cuh"
#include "gelu.cuh"
#include "mx.cuh"
#include "philox.cuh"
#include "sm100.cuh"

namespace mtorus {

using namespace sm100;

struct GemmEpilogue {
  void* D;
  int64_t ldd;
  int out_f32;          // 0 = bf16 output, 1 = fp32 output
  int beta;             // fp32 output: D += result
  const float* bias;    // [N] fp32 or null
  const bf16* residual; // [M, ldr] bf16 added before the store (bf16 output) or null
  int64_t ldr;
  bf16* act;            // GELU(result) written here (D receives the pre-activation) or null
  int64_t ldact;
  const bf16* aux;      // dGELU: result *= gelu'(aux[m, n]) or null
  int64_t ldaux;
  const float* alpha;   // device scalar multiplier or null
  const float* alpha2;  // second device scalar multiplier (e.g. the other operand's 1/scale) or null
  // FP8 GELU output (2-SM kernel): act8 = fp8(GELU(result) * act8_scale), max|GELU| -> act8_amax
  uint8_t* act8;
  const float* act8_scale;
  float* act8_amax;
  int act8_fmt;         // 0 = E4M3, 1 = E5M2
};

// MXFP8 output of the 2-SM block-scaled GEMM's epilogue: the tile's values (or its
// GELU) as row-wise codes [M, N] (32-blocks along N; stored through the act tensor
// map) and column-wise codes [N, M] (32-blocks along M; its own tensor map), with the
// scale atoms of both in the mx_quantize layout, optionally summing the columns
// (the bias gradient when the tile is an output gradient).  M and N multiples of 128.
struct MxOutArgs {
  uint8_t* rsf;        // scales of the row codes: [ceil(M/128)][ceil(N/128)][512]
  uint8_t* csf;        // scales of the column codes: [ceil(N/128)][ceil(M/128)][512]
  float* colsum;       // += column sums of the quantised (bf16-rounded) values, or null
  uint32_t fmax_bits;  // largest finite value of the code format (fp32 bits)
  int fmt;             // 0 = E4M3, 1 = E5M2
  int src_act;         // 1: quantise GELU(result) (D keeps the pre-activation); 0: the result itself
  int store_d;         // 1: also store D in bf16
};

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, GROUP_M = 16;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;  // double-buffered accumulator
constexpr int kThreads = 192;

__device__ __forceinline__ float gelu_f(float x) { return gelu_fwd(x); }
__device__ __forceinline__ float gelu_grad_f(float x) { return gelu_grad(x); }

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = GROUP_M * num_n;
  const int group = tile / per_group;
  const int first_m = group * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int r = tile % per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

// Applies the epilogue to 32 consecutive accumulator columns of row m
// (columns n0..n0+31) and stores them.
__device__ __forceinline__ void epilogue_store32(const uint32_t (&r)[32], int m, int n0, int N,
                                                 float alpha, const GemmEpilogue& ep) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * alpha;
  if (ep.bias) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (n0 + i < N) v[i] += ep.bias[n0 + i];
  }
  if (ep.aux) {
    const bf16* ax = ep.aux + (size_t)m * ep.ldaux + n0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (n0 + j * 8 + 8 <= N) {
        float a8[8];
        unpack8(reinterpret_cast<const bf16x8*>(ax)[j], a8);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j * 8 + i] *= gelu_grad_f(a8[i]);
      }
    }
  }
  if (ep.out_f32) {
    float* dp = reinterpret_cast<float*>(ep.D) + (size_t)m * ep.ldd + n0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (n0 + j * 4 + 4 <= N) {
        float4 o = make_float4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]);
        if (ep.beta) {
          const float4 old = reinterpret_cast<float4*>(dp)[j];
          o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
        }
        reinterpret_cast<float4*>(dp)[j] = o;
      }
    }
  } else {
    bf16* dp = reinterpret_cast<bf16*>(ep.D) + (size_t)m * ep.ldd + n0;
    if (ep.residual) {
      const bf16* rp = ep.residual + (size_t)m * ep.ldr + n0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (n0 + j * 8 + 8 <= N) {
          float r8[8];
          unpack8(reinterpret_cast<const bf16x8*>(rp)[j], r8);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[j * 8 + i] += r8[i];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (n0 + j * 8 + 8 <= N) {
        bf16x8 pk = pack8(v + j * 8);
        reinterpret_cast<bf16x8*>(dp)[j] = pk;
        if (ep.act) {
          float p8[8], g8[8];
          unpack8(pk, p8);  // GELU of the rounded pre-activation
#pragma unroll
          for (int i = 0; i < 8; ++i) g8[i] = gelu_f(p8[i]);
          reinterpret_cast<bf16x8*>(ep.act + (size_t)m * ep.ldact + n0)[j] = pack8(g8);
        }
      }
    }
  }
}

struct Smem {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tma_a,
                        const __grid_constant__ CUtensorMap tma_b, int M, int N, int K, int a_mn,
                        int b_mn, GemmEpilogue ep, int* status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  Smem* ctl = reinterpret_cast<Smem*>(smem + STAGES * STAGE_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->tfull[b], 1);
      mbar_init(&ctl->tempty[b], 128);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort = &ctl->abort;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, parity_mask = 0;  // per stage: load in flight, its phase parity
      for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort, status, 1)) break;
          issued_mask |= 1u << stage;
          parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
          mbar_arrive_expect_tx(&ctl->full[stage], STAGE_BYTES);
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          if (!a_mn) {
            tma_load_2d(sa, &tma_a, &ctl->full[stage], kb * BK, mb * BM);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(sa + j * (BK * 128), &tma_a, &ctl->full[stage], mb * BM + j * 64, kb * BK);
          }
          if (!b_mn) {
            tma_load_2d(sb, &tma_b, &ctl->full[stage], kb * BK, nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + j * (BK * 128), &tma_b, &ctl->full[stage], nb * BN + j * 64, kb * BK);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort) {
        // drain: let every load this thread issued land before the CTA exits
        for (int s = 0; s < STAGES; ++s) {
          if (!(issued_mask >> s & 1u)) continue;
          const uint32_t par = (parity_mask >> s) & 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(smem_u32(&ctl->full[s]), par) &&
                 globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = make_idesc_bf16(BM, BN, a_mn, b_mn);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t tphase = (local >> 1) & 1;
        if (!mbar_wait(&ctl->tempty[buf], tphase ^ 1, abort, status, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&ctl->full[stage], phase, abort, status, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = a_mn ? make_sdesc(sa + k * 2048, BK * 128, 1024, kSwizzle128B)
                                     : make_sdesc(sa + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = b_mn ? make_sdesc(sb + k * 2048, BK * 128, 1024, kSwizzle128B)
                                     : make_sdesc(sb + k * 32, 16, 1024, kSwizzle128B);
            umma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&ctl->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&ctl->tfull[buf]);
      }
      if (*abort && issued_any) {
        umma_commit(&ctl->drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(smem_u32(&ctl->drain), 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int buf = local & 1;
      const uint32_t tphase = (local >> 1) & 1;
      if (!mbar_wait(&ctl->tfull[buf], tphase, abort, status, 4)) break;
      tc_fence_after();
      const int m = mb * BM + row;
      const float alpha = ep.alpha ? *ep.alpha : 1.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN + c * 32, r);
        tmem_wait_ld();
        const int n0 = nb * BN + c * 32;
        if (m >= M || n0 >= N) continue;
        epilogue_store32(r, m, n0, N, alpha, ep);
      }
      tc_fence_before();
      mbar_arrive(&ctl->tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------ 2-SM kernel
//
// The same GEMM on CTA pairs (cluster of 2, tcgen05 cta_group::2): a pair owns a
// 256 x 256 output tile, each CTA loads its own 128 rows of A and half of the B
// tile (128 rows), and the pair leader issues M=256 / N=256 MMAs that read both
// CTAs' shared memory and write each CTA's 128 accumulator rows into its own
// TMEM.  Per SM this moves 32 KB of operands per 64-deep k-block instead of
// 48 KB, which frees shared memory for a 6-stage ring.  Loads of both CTAs
// complete on the leader's "full" barrier; the leader's commits arrive on both
// CTAs' "empty" / "accumulator full" barriers; both epilogues arrive on the
// leader's "accumulator empty" barrier.
namespace {

constexpr int P_BM = 128;  // rows per CTA (pair tile M = 256)
constexpr int P_BN = 256;  // pair tile N; each CTA stages 128 rows of B
constexpr int P_STAGES = 5;       // operand ring depth
template <bool MX>
constexpr int pair_stages() { return P_STAGES; }
constexpr int P_GROUP_M = 8;  // pair tiles per raster group along M
constexpr int P_A_BYTES = P_BM * 128;        // 128 rows x 128 bytes of K
constexpr int P_B_BYTES = (P_BN / 2) * 128;  // 128 rows of B x 128 bytes of K
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
// Epilogue: eight warps, each with two 4 KB staging buffers (one in the MXFP8
// kernel, whose per-stage scales would otherwise cost it an operand stage); a
// buffer holds one 32x32 output chunk (fp32, 4 KB) or a bf16 chunk (2 KB) plus its
// GELU output (bf16 2 KB or FP8 1 KB at offset 2048), written to global memory by TMA.
constexpr int P_EPI_WARPS = 8;
constexpr int kPairThreads = 64 + 32 * P_EPI_WARPS;
constexpr int P_EPI_BUF = 4096;
template <bool MX>
constexpr int epi_nbuf() { return MX ? 1 : 2; }
template <bool MX>
constexpr int epi_bytes() { return P_EPI_WARPS * epi_nbuf<MX>() * P_EPI_BUF; }
// MXFP8 (1x32 UE8M0 block scales) per stage: this CTA's 128-row SFA atom and the
// pair tile's two 128-row SFB atoms (every CTA needs the scales of all 256 B rows,
// since its tensor core multiplies its A rows with the whole B tile).  An atom holds
// the scales of 128 rows x 4 K-blocks of 32 (one stage) in the tcgen05.cp layout:
// byte (r % 32) * 16 + (r / 32) * 4 + k.
constexpr int P_SF_ATOM = 512;
constexpr int P_SF_BYTES = 3 * P_SF_ATOM;
// TMEM in the MXFP8 kernel: the scale factors need 2 x 12 of the 512 columns (two
// sets, used by alternate stages), so the second accumulator starts one 32-column
// chunk early and overlaps the first one's last chunk; each epilogue reads the shared
// chunk first and signals "ovl" before the next tile's MMAs may start.  Scales occupy
// the last 32 columns: set s at 480 + 16 s (SFA 4 columns, SFB 8).
constexpr int MX_ACC1_COL = P_BN - 32;
constexpr int MX_SF_COL = 2 * P_BN - 32;

// Row-sharded B read straight from its owners' memory: the parameter all-gather
// fused into the GEMM that consumes the parameters.  Rank p owns rows
// [p * shard_rows, (p + 1) * shard_rows) of B's storage (N rows for a K-major B,
// K rows for an MN-major one) in its symmetric buffer, and m[p] maps that buffer
// with the local map's shape and box.  Each B tile is a plain TMA load from the
// owner (never a multicast load), so a remote tile crosses NVLink once per CTA
// that needs it and lands in this SM's shared memory.  n == 0: B is local.
struct PeerMapsB {
  CUtensorMap m[8];
  int n;
  int shard_rows;
};

struct PairSmem {
  uint64_t full[P_STAGES];   // leader: both CTAs' loads of a stage have landed
  uint64_t empty[P_STAGES];  // each CTA: the MMAs reading a stage are done
  uint64_t tfull[2];         // each CTA: accumulator buffer ready for the epilogue
  uint64_t tempty[2];        // leader: both epilogues finished with a buffer
  uint64_t ovl;              // leader (MXFP8): both epilogues read the chunk shared by the two accumulators
  long long prof[4];         // stall accounting (gemm_profile): empty, full, tempty, ovl waits
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void pair_tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = P_GROUP_M * num_n;
  const int group = tile / per_group;
  const int first_m = group * P_GROUP_M;
  const int gsize = min(num_m - first_m, P_GROUP_M);
  const int r = tile % per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

}  // namespace

// Accumulator chunk (32 columns) processed i-th by epilogue warp half h; MXFP8
// buffer 0 starts with the chunk it shares with buffer 1 (see MX_ACC1_COL).
template <bool MX>
__device__ __forceinline__ int epi_chunk(int buf, int h, int i) {
  if (MX && buf == 0 && h == 1) return i == 0 ? 7 : 3 + i;
  return h * 4 + i;
}

// The 64 bytes of row m, columns n0..n0+31 of the dGELU input (aux) or of the
// residual, whichever the epilogue reads (never both: dGELU runs in dgrad GEMMs,
// residual adds in forward GEMMs); zeros outside the matrix.
__device__ __forceinline__ void epi_prefetch(const GemmEpilogue& ep, int m, int M, int N, int n0, uint4 (&x)[4]) {
  const bf16* src = ep.aux ? ep.aux + (size_t)m * ep.ldaux + n0
                           : (ep.residual ? ep.residual + (size_t)m * ep.ldr + n0 : nullptr);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    x[j] = (src && m < M && n0 + j * 8 + 8 <= N) ? reinterpret_cast<const uint4*>(src)[j] : make_uint4(0, 0, 0, 0);
}

// One 32 x 32 output chunk of an epilogue warp: registers -> staging buffer -> TMA store.
// r: the lane's (row m) 32 accumulator values; x: its prefetched aux / residual;
// stages: the warp's two 4 KB staging buffers (D at 0, the GELU output at 2048),
// used in turn by the chunks that store (sb flips at each commit, so the buffer
// written next is never the one the most recent store still reads).
// DROP: dropout drawn in the epilogue (philox.cuh; element index m * N + n): mode 1
// drops the GEMM result before the residual add (a branch output), mode 2 drops
// GELU(result) in the act / act8 output (the FFN hidden), mode 3 applies the same
// mask to the incoming gradient before the dGELU multiply (its backward).
template <bool DROP, int NB, bool MXO>
__device__ __forceinline__ void epi_chunk_store(const uint32_t (&r)[32], const uint4 (&x)[4], int m, int M, int N,
                                                int n0, int row0, float alpha, float act_scale, float& act_amax,
                                                const GemmEpilogue& ep, bool f32out, uint8_t* stages, int& sb,
                                                const CUtensorMap* tma_d, const CUtensorMap* tma_act, int lane,
                                                const DropoutArgs& drop, int drop_mode, const MxOutArgs& mxo,
                                                const CUtensorMap* tma_cc) {
  if (n0 >= N) return;  // warp-uniform
  // A single 4 KB buffer (NB == 1) still double-buffers a plain bf16 chunk (2 KB): its halves alternate
  const bool halves = NB == 1 && !MXO && !f32out && !ep.act && !ep.act8;
  uint8_t* stage = stages + sb * (halves ? P_EPI_BUF / 2 : P_EPI_BUF);
  uint32_t keep = 0xFFFFFFFFu;
  if constexpr (DROP) {
    const uint32_t k0 = drop.rng[0], k1 = drop.rng[1];
    const uint64_t g0 = ((uint64_t)m * N + n0) >> 3;
    keep = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) keep |= dropout_keep8(k0, k1, drop.site, g0 + q, drop.thr16) << (8 * q);
  }
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * alpha;
  if (ep.bias) {
    if (n0 + 32 <= N) {
      const float4* bp = reinterpret_cast<const float4*>(ep.bias + n0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 b = bp[j];
        v[4 * j] += b.x; v[4 * j + 1] += b.y; v[4 * j + 2] += b.z; v[4 * j + 3] += b.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (n0 + i < N) v[i] += ep.bias[n0 + i];
    }
  }
  if constexpr (DROP) {
    if (drop_mode == 1 || drop_mode == 3) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = (keep >> i & 1u) ? v[i] * drop.scale : 0.f;
    }
  }
  if (ep.aux) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a8[8];
      unpack8(*reinterpret_cast<const bf16x8*>(&x[j]), a8);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[j * 8 + i] *= gelu_grad_f(a8[i]);
    }
  } else if (ep.residual) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float r8[8];
      unpack8(*reinterpret_cast<const bf16x8*>(&x[j]), r8);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[j * 8 + i] += r8[i];
    }
  }
  if (lane == 0) {  // the store that last used this buffer has read it
    if (halves)
      bulk_wait_group_read<1>();
    else
      bulk_wait_group_read<NB - 1>();
  }
  __syncwarp();
  if constexpr (MXO) {
    // The chunk is 32 rows (one per lane) x 32 columns: one row block per lane and,
    // read back through shared memory, one column block per lane.  Bytes 0..2047 of
    // the staging buffer: D (bf16, 64B swizzle); 2048..4095: first the bf16 values to
    // quantise (same swizzle), then the row codes [32 x 32 B] and the column codes.
    uint8_t* base = stage + lane * 64;
    uint8_t* sbase = stage + 2048;
    float sv[32];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bf16x8 pk = pack8(v + 8 * j);
      if (mxo.store_d) *reinterpret_cast<bf16x8*>(base + ((j ^ ((lane >> 1) & 3)) << 4)) = pk;
      bf16x8 src = pk;
      if (mxo.src_act) {
        float p8[8], g8[8];
        unpack8(pk, p8);  // GELU of the rounded pre-activation, as the bf16 path stores it
#pragma unroll
        for (int i = 0; i < 8; ++i) g8[i] = gelu_f(p8[i]);
        if constexpr (DROP) {
          if (drop_mode == 2) {
            float r8[8];
            unpack8(pack8(g8), r8);
#pragma unroll
            for (int i = 0; i < 8; ++i) g8[i] = (keep >> (8 * j + i) & 1u) ? r8[i] * drop.scale : 0.f;
          }
        }
        src = pack8(g8);
      }
      if (m >= M) {  // rows past M hold the epilogue of zero-filled A rows: they pad the column blocks as zeros
        const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        src = pack8(z);
      }
      unpack8(src, sv + 8 * j);
      *reinterpret_cast<bf16x8*>(sbase + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = src;
    }
    const int ef = (int)((mxo.fmax_bits >> 23) & 0xFF);
    const uint32_t mf = mxo.fmax_bits & 0x7FFFFF;
    uint32_t rw[8], cw[8];
    uint8_t rsb, csb;
    mx_block(sv, ef, mf, mxo.fmt, rw, rsb);  // this lane's row block (sv is dead afterwards)
    __syncwarp();
    float cv[32];  // column n0 + lane, rows row0 .. row0 + 31
#pragma unroll
    for (int rr = 0; rr < 32; ++rr)
      cv[rr] = __bfloat162float(*reinterpret_cast<const bf16*>(
          sbase + rr * 64 + ((((lane >> 3) ^ ((rr >> 1) & 3))) << 4) + (lane & 7) * 2));
    mx_block(cv, ef, mf, mxo.fmt, cw, csb);
    if (mxo.colsum) {
      float cs = 0.f;
#pragma unroll
      for (int rr = 0; rr < 32; ++rr) cs += cv[rr];
      atomicAdd(mxo.colsum + n0 + lane, cs);
    }
    __syncwarp();  // every lane has read the bf16 values
    uint4* rdst = reinterpret_cast<uint4*>(sbase + lane * 32);
    rdst[0] = make_uint4(rw[0], rw[1], rw[2], rw[3]);
    rdst[1] = make_uint4(rw[4], rw[5], rw[6], rw[7]);
    uint4* cdst = reinterpret_cast<uint4*>(sbase + 1024 + lane * 32);
    cdst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
    cdst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
    // scale bytes in the mx_quantize atom layout ((r / 128) * nkb4 + k / 4) * 512 + (r % 32) * 16 +
    // (r % 128 / 32) * 4 + k % 4, r the operand row, k the 32-block along its K
    if (m < M) {
      const int nkb = N >> 7;
      mxo.rsf[((int64_t)(m >> 7) * nkb + (n0 >> 7)) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + ((n0 & 127) >> 5)] =
          rsb;
    }
    if (row0 < M) {
      const int c = n0 + lane, mkb = M >> 7;
      mxo.csf[((int64_t)(c >> 7) * mkb + (row0 >> 7)) * 512 + (c & 31) * 16 + ((c & 127) >> 5) * 4 +
              ((row0 & 127) >> 5)] = csb;
    }
  } else if (f32out) {
    // 32 rows x 128 B, 128B swizzle: 16-byte chunk j of row r sits at j ^ (r & 7)
    uint8_t* base = stage + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(base + ((j ^ (lane & 7)) << 4)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    // 32 rows x 64 B, 64B swizzle: 16-byte chunk j of row r sits at j ^ ((r >> 1) & 3)
    uint8_t* base = stage + lane * 64;
    uint8_t* abase = stage + 2048;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bf16x8 pk = pack8(v + 8 * j);
      *reinterpret_cast<bf16x8*>(base + ((j ^ ((lane >> 1) & 3)) << 4)) = pk;
      if (ep.act) {
        float p8[8], g8[8];
        unpack8(pk, p8);  // GELU of the rounded pre-activation
#pragma unroll
        for (int i = 0; i < 8; ++i) g8[i] = gelu_f(p8[i]);
        if constexpr (DROP) {
          if (drop_mode == 2) {
            float r8[8];
            unpack8(pack8(g8), r8);  // the bf16 GELU, then the dropout (as dropout_apply does)
#pragma unroll
            for (int i = 0; i < 8; ++i) g8[i] = (keep >> (8 * j + i) & 1u) ? r8[i] * drop.scale : 0.f;
          }
        }
        *reinterpret_cast<bf16x8*>(abase + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = pack8(g8);
      } else if (ep.act8) {
        // FP8 GELU: the bf16-rounded GELU (as the bf16 path stores it) times the scale;
        // 32 rows x 32 B, unswizzled
        float p8[8], g8[8], r8[8];
        unpack8(pk, p8);
#pragma unroll
        for (int i = 0; i < 8; ++i) g8[i] = gelu_f(p8[i]);
        unpack8(pack8(g8), r8);
        if constexpr (DROP) {
          if (drop_mode == 2) {
#pragma unroll
            for (int i = 0; i < 8; ++i) g8[i] = (keep >> (8 * j + i) & 1u) ? r8[i] * drop.scale : 0.f;
            unpack8(pack8(g8), r8);
          }
        }
        uint32_t w[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (m < M) {  // rows past M hold GELU(bias) of zero-filled A rows
#pragma unroll
            for (int t = 0; t < 4; ++t) act_amax = fmaxf(act_amax, fabsf(r8[4 * k + t]));
          }
          const uint16_t lo = ep.act8_fmt == 0 ? cvt2_e4m3(r8[4 * k] * act_scale, r8[4 * k + 1] * act_scale)
                                               : cvt2_e5m2(r8[4 * k] * act_scale, r8[4 * k + 1] * act_scale);
          const uint16_t hi = ep.act8_fmt == 0 ? cvt2_e4m3(r8[4 * k + 2] * act_scale, r8[4 * k + 3] * act_scale)
                                               : cvt2_e5m2(r8[4 * k + 2] * act_scale, r8[4 * k + 3] * act_scale);
          w[k] = (uint32_t)lo | ((uint32_t)hi << 16);
        }
        *reinterpret_cast<uint2*>(abase + lane * 32 + j * 8) = make_uint2(w[0], w[1]);
      }
    }
  }
  fence_async_shared();
  __syncwarp();
  if (lane == 0) {
    if constexpr (MXO) {
      if (mxo.store_d) tma_store_2d(tma_d, stage, n0, row0);
      tma_store_2d(tma_act, stage + 2048, n0, row0);         // row codes [M, N]
      tma_store_2d(tma_cc, stage + 3072, row0, n0);          // column codes [N, M]
    } else {
      if (f32out && ep.beta)
        tma_reduce_add_2d(tma_d, stage, n0, row0);
      else
        tma_store_2d(tma_d, stage, n0, row0);
      if (ep.act || ep.act8) tma_store_2d(tma_act, stage + 2048, n0, row0);
    }
    bulk_commit_group();
  }
  if (NB == 2 || halves) sb ^= 1;
}

// EB = operand element bytes: 2 (bf16, kind::f16) or 1 (fp8 E4M3/E5M2, kind::f8f6f4).
// A k-block is always 128 bytes of K per row (64 bf16 / 128 fp8), so the stage
// layout is identical and an fp8 stage carries twice the MMA work.
// MX (EB == 1, K-major A and B only): kind::mxf8f6f4 with 1x32 UE8M0 block scales,
// loaded per stage next to the operands and copied into TMEM by the MMA thread
// (tcgen05.cp, ordered before the stage's MMAs, which read them); sf_kb = number of
// 128-wide K blocks per 128-row block of the scale tensors.
// MXFP8: the three scale atoms of a stage (A's 128 rows; B's two 128-row halves)
// from shared memory into TMEM columns sf_tmem .. sf_tmem + 11 of both CTAs.
__device__ __forceinline__ void mx_copy_scales(uint32_t sf_tmem, uint32_t ssf) {
  tmem_cp_32x128b_x4_2sm(sf_tmem, make_sdesc(ssf, 0, 128, kSwizzleNone));
  tmem_cp_32x128b_x4_2sm(sf_tmem + 4, make_sdesc(ssf + P_SF_ATOM, 0, 128, kSwizzleNone));
  tmem_cp_32x128b_x4_2sm(sf_tmem + 8, make_sdesc(ssf + 2 * P_SF_ATOM, 0, 128, kSwizzleNone));
}

template <int EB, bool MX = false, bool DROP = false, bool MXO = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_2sm_kernel(const __grid_constant__ CUtensorMap tma_a,
                    const __grid_constant__ CUtensorMap tma_b,
                    const __grid_constant__ CUtensorMap tma_d,
                    const __grid_constant__ CUtensorMap tma_act,
                    const __grid_constant__ CUtensorMap tma_sfa,
                    const __grid_constant__ CUtensorMap tma_sfb,
                    const __grid_constant__ PeerMapsB peer_b, int M, int N, int K, int a_mn,
                    int b_mn, int sf_kb, uint32_t idesc, GemmEpilogue ep, int* status,
                    unsigned long long* prof, DropoutArgs drop, int drop_mode,
                    const __grid_constant__ CUtensorMap tma_cc, MxOutArgs mxo) {
  // prof (optional, gemm_profile): stall accounting summed over CTAs: cycles the
  // producer waited for free stages [0] and ran [1], the MMA issuer waited for
  // loaded stages [2] / free accumulators [3] and ran [4], waited for the MXFP8
  // epilogue to read the chunk both accumulators share [5]; CTA pairs [7].
  static_assert(!MX || EB == 1, "block scaling is for fp8 operands");
  static_assert(!MXO || MX, "MXFP8 output is an epilogue of the block-scaled kernel");
  constexpr int BK = 128 / EB;       // K elements per stage
  constexpr int MMA_K = 32 / EB;     // K elements per tcgen05.mma
  constexpr int MN_BOX = 128 / EB;   // MN elements per 128-byte swizzle row
  constexpr int A_BOXES = P_BM * EB / 128, B_BOXES = (P_BN / 2) * EB / 128;
  constexpr int NST = pair_stages<MX>();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* epi_smem = smem + NST * P_STAGE_BYTES;
  uint8_t* sf_smem = epi_smem + epi_bytes<MX>();
  PairSmem* ctl = reinterpret_cast<PairSmem*>(sf_smem + (MX ? NST * P_SF_BYTES : 0));
  constexpr uint32_t ACC1_COL = MX ? MX_ACC1_COL : P_BN;  // TMEM column of accumulator 1

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  const int num_m = (M + 2 * P_BM - 1) / (2 * P_BM), num_n = (N + P_BN - 1) / P_BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->tfull[b], 1);
      mbar_init(&ctl->tempty[b], 2 * 32 * P_EPI_WARPS);
    }
    if constexpr (MX) mbar_init(&ctl->ovl, 2 * 128);
    for (int i = 0; i < 4; ++i) ctl->prof[i] = 0;
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc_2sm(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish_2sm();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort = &ctl->abort;
  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer (both CTAs)
      const long long prof_t0 = prof ? clock64() : 0;
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; tile < num_tiles && !*abort; tile += num_pairs) {
        int mb, nb;
        pair_tile_coords(tile, num_m, num_n, mb, nb);
        const int m0 = mb * 2 * P_BM + (int)rank * P_BM;
        const int n0 = nb * P_BN + (int)rank * (P_BN / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          const long long pw0 = prof ? clock64() : 0;
          if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort, status, 11)) break;
          if (prof) ctl->prof[0] += clock64() - pw0;
          if (leader) mbar_arrive_expect_tx(&ctl->full[stage], 2 * (P_STAGE_BYTES + (MX ? P_SF_BYTES : 0)));
          uint8_t* sa = smem + stage * P_STAGE_BYTES;
          uint8_t* sb = sa + P_A_BYTES;
          if (!a_mn) {
            tma_load_2d_pair(sa, &tma_a, &ctl->full[stage], kb * BK, m0);
          } else {
#pragma unroll
            for (int j = 0; j < A_BOXES; ++j)
              tma_load_2d_pair(sa + j * (BK * 128), &tma_a, &ctl->full[stage], m0 + j * MN_BOX, kb * BK);
          }
          const CUtensorMap* map_b = &tma_b;
          if (peer_b.n > 0)  // owner of this CTA's B rows (K-major) or of this k-block (MN-major)
            map_b = &peer_b.m[min(peer_b.n - 1, (b_mn ? kb * BK : n0) / peer_b.shard_rows)];
          if (!b_mn) {
            tma_load_2d_pair(sb, map_b, &ctl->full[stage], kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < B_BOXES; ++j)
              tma_load_2d_pair(sb + j * (BK * 128), map_b, &ctl->full[stage], n0 + j * MN_BOX, kb * BK);
          }
          if constexpr (MX) {
            // scale atoms: rows of 256 bytes, two rows per atom; boxes past the end read zeros
            uint8_t* ssf = sf_smem + stage * P_SF_BYTES;
            const int arb = m0 / 128, brb = (nb * P_BN) / 128;
            tma_load_2d_pair(ssf, &tma_sfa, &ctl->full[stage], 0, (arb * sf_kb + kb) * 2);
            tma_load_2d_pair(ssf + P_SF_ATOM, &tma_sfb, &ctl->full[stage], 0, (brb * sf_kb + kb) * 2);
            tma_load_2d_pair(ssf + 2 * P_SF_ATOM, &tma_sfb, &ctl->full[stage], 0, ((brb + 1) * sf_kb + kb) * 2);
          }
          if (++stage == NST) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (prof) {
        atomicAdd(prof + 0, (unsigned long long)ctl->prof[0]);
        atomicAdd(prof + 1, (unsigned long long)(clock64() - prof_t0));
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // ---------------------------------------------------------- MMA issuer (leader)
      const long long prof_t0 = prof ? clock64() : 0;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = pair; tile < num_tiles && !*abort; tile += num_pairs, ++local) {
        const int buf = local & 1;
        const uint32_t tphase = (local >> 1) & 1;
        const long long tw0 = prof ? clock64() : 0;
        if (!mbar_wait(&ctl->tempty[buf], tphase ^ 1, abort, status, 12)) break;
        if (prof) ctl->prof[2] += clock64() - tw0;
        if constexpr (MX) {
          // the previous tile's epilogue must have read the chunk both accumulators share
          const long long ow0 = prof ? clock64() : 0;
          if (local > 0 && !mbar_wait(&ctl->ovl, (uint32_t)(local - 1) & 1, abort, status, 15)) break;
          if (prof) ctl->prof[3] += clock64() - ow0;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * ACC1_COL;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          const long long fw0 = prof ? clock64() : 0;
          const bool got = mbar_wait(&ctl->full[stage], phase, abort, status, 13);
          if (prof) ctl->prof[1] += clock64() - fw0;
          if (!got) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES);
          const uint32_t sb = sa + P_A_BYTES;
          // MXFP8 scales of consecutive stages alternate between two TMEM column sets, so a
          // stage's copy never overwrites scales the previous stage's MMAs may still read
          const uint32_t sf_tmem = tmem_base + MX_SF_COL + (uint32_t)(stage & 1) * 16;
          if constexpr (MX) {
            // stage scales -> TMEM (in order with the MMAs of this thread, so the MMAs of
            // stage - 2, the last readers of this column set, have read them before these land)
            mx_copy_scales(sf_tmem, smem_u32(sf_smem + stage * P_SF_BYTES));
          }
#pragma unroll
          for (int k = 0; k < BK / MMA_K; ++k) {
            const uint64_t ad = a_mn ? make_sdesc(sa + k * MMA_K * 128, BK * 128, 1024, kSwizzle128B)
                                     : make_sdesc(sa + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = b_mn ? make_sdesc(sb + k * MMA_K * 128, BK * 128, 1024, kSwizzle128B)
                                     : make_sdesc(sb + k * 32, 16, 1024, kSwizzle128B);
            if constexpr (MX)
              umma_mx_2sm(d_tmem, ad, bd, idesc_mx_sf_id(idesc, (uint32_t)k),
                          sf_tmem | ((uint32_t)k << 30), (sf_tmem + 4) | ((uint32_t)k << 30), (kb | k) != 0 ? 1u : 0u);
            else if constexpr (EB == 2)
              umma_f16_2sm(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              umma_f8_2sm(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_2sm_mc(&ctl->empty[stage], 0x3);
          if (++stage == NST) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_2sm_mc(&ctl->tfull[buf], 0x3);
      }
      if (prof) {
        atomicAdd(prof + 7, 1ull);
        atomicAdd(prof + 5, (unsigned long long)ctl->prof[3]);
        atomicAdd(prof + 2, (unsigned long long)ctl->prof[1]);
        atomicAdd(prof + 3, (unsigned long long)ctl->prof[2]);
        atomicAdd(prof + 4, (unsigned long long)(clock64() - prof_t0));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // Eight warps, two per TMEM lane quarter (a warp may only read the 32 lanes of
    // quarter warp % 4): warp half h = 0 takes accumulator columns 0..127, h = 1
    // columns 128..255, as four 32-column chunks.  TMEM -> registers (alpha, bias,
    // dGELU, residual) -> swizzled smem chunk -> TMA store (or TMA reduce-add for
    // fp32 accumulation).  The TMEM load of chunk i+1 and the global loads (aux,
    // residual) it needs are issued before chunk i is processed, so their latency
    // hides behind its math; two staging buffers per warp let the math of chunk i
    // overlap the store of chunk i-1.
    const int ew = warp - 2;
    const int q = warp & 3;
    const int h = ew >> 2;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&ctl->tempty[0]), 0);
    const uint32_t tempty_leader1 = mapa_shared(smem_u32(&ctl->tempty[1]), 0);
    const uint32_t ovl_leader = mapa_shared(smem_u32(&ctl->ovl), 0);
    uint8_t* stage_base = epi_smem + ew * epi_nbuf<MX>() * P_EPI_BUF;
    const bool f32out = ep.out_f32 != 0;
    const float act_scale = ep.act8_scale ? *ep.act8_scale : 1.f;
    float act_amax = 0.f;
    int sb = 0;
    int local = 0;
    for (int tile = pair; tile < num_tiles && !*abort; tile += num_pairs, ++local) {
      int mb, nb;
      pair_tile_coords(tile, num_m, num_n, mb, nb);
      const int buf = local & 1;
      const uint32_t tphase = (local >> 1) & 1;
      if (!mbar_wait(&ctl->tfull[buf], tphase, abort, status, 14)) break;
      tc_fence_after();
      const int row0 = mb * 2 * P_BM + (int)rank * P_BM + q * 32;
      const int m = row0 + lane;
      const float alpha = (ep.alpha ? *ep.alpha : 1.f) * (ep.alpha2 ? *ep.alpha2 : 1.f);
      // MXFP8: the chunk the two accumulators share (columns 224..255 of accumulator 0
      // = columns 0..31 of accumulator 1) is read first, and its readers signal "ovl"
      const bool shared_first = MX && ((buf == 0 && h == 1) || (buf == 1 && h == 0));
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * ACC1_COL;
      uint32_t ra[32], rb[32];
      uint4 xa[4], xb[4];  // aux (dGELU input) or residual of the chunk, prefetched
      tmem_ld32(tbase + epi_chunk<MX>(buf, h, 0) * 32, ra);
      epi_prefetch(ep, m, M, N, nb * P_BN + epi_chunk<MX>(buf, h, 0) * 32, xa);
      tmem_wait_ld();
      if (shared_first) {
        tc_fence_before();
        mbar_arrive_cluster(ovl_leader);
      }
#pragma unroll 1
      for (int i = 0; i < 4; i += 2) {
        const int c0 = epi_chunk<MX>(buf, h, i), c1 = epi_chunk<MX>(buf, h, i + 1);
        tmem_ld32(tbase + c1 * 32, rb);
        epi_prefetch(ep, m, M, N, nb * P_BN + c1 * 32, xb);
        epi_chunk_store<DROP, epi_nbuf<MX>(), MXO>(ra, xa, m, M, N, nb * P_BN + c0 * 32, row0, alpha, act_scale, act_amax, ep, f32out,
                              stage_base, sb, &tma_d, &tma_act, lane, drop, drop_mode, mxo, &tma_cc);
        tmem_wait_ld();
        if (i + 1 == 3) {
          // every column of this warp's share of the buffer is in registers: release it
          tc_fence_before();
          mbar_arrive_cluster(buf ? tempty_leader1 : tempty_leader0);
        } else {
          const int c2 = epi_chunk<MX>(buf, h, i + 2);
          tmem_ld32(tbase + c2 * 32, ra);
          epi_prefetch(ep, m, M, N, nb * P_BN + c2 * 32, xa);
        }
        epi_chunk_store<DROP, epi_nbuf<MX>(), MXO>(rb, xb, m, M, N, nb * P_BN + c1 * 32, row0, alpha, act_scale, act_amax, ep, f32out,
                              stage_base, sb, &tma_d, &tma_act, lane, drop, drop_mode, mxo, &tma_cc);
        if (i + 1 != 3) tmem_wait_ld();
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
    if (ep.act8_amax) {
      const float wm = warp_max(act_amax);
      if (lane == 0) atomic_max_pos(ep.act8_amax, wm);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_2sm(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p,
                "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Driver-API calls (the tensor-map encoder) need a current context on the
// calling thread.  Runtime calls create it lazily, and a thread such as the
// autograd worker may not have made one yet (its allocations can all come from
// torch's cache), so bind the device's primary context explicitly.
void ensure_context() {
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaSetDevice(dev));
}

// 2-D row-major tensor [outer, inner] with row stride `ld` elements; 128B swizzle.
CUtensorMap make_tma_2d(const void* ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                        uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swz) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_tiled()(&m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r,
              " (inner=", inner, ", outer=", outer, ", ld=", ld, ")");
  return m;
}

static int* gemm_status_ptr() {
  static int* p = nullptr;
  if (!p) {
    C10_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  }
  return p;
}

int64_t gemm_status(bool reset) {
  int h = 0;
  int* p = gemm_status_ptr();
  C10_CUDA_CHECK(cudaMemcpy(&h, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  return h;
}

static void check_operand(const at::Tensor& t, const char* name, int elem_bytes) {
  TORCH_CHECK(t.is_cuda() && t.element_size() == elem_bytes, name, ": CUDA tensor with ", elem_bytes,
              "-byte elements expected");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, ": 2-D with unit inner stride expected");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, ": 16-byte aligned base required");
  TORCH_CHECK((t.stride(0) * elem_bytes) % 16 == 0, name, ": row stride must be a multiple of 16 bytes");
}

// SMs left free for concurrently running communication kernels (set while the
// data-parallel reducer overlaps backward): persistent GEMMs size their grid to
// the rest so a comm kernel never leaves a GEMM CTA waiting for an SM.
static int g_reserved_sms = 0;
void gemm_set_reserved_sms(int64_t n) { g_reserved_sms = (int)std::max<int64_t>(0, n); }

// Stall accounting of the CTA-pair kernels (see GemmEpilogue::prof): off unless
// gemm_profile(true) was called; gemm_profile_read() returns the eight sums.
static unsigned long long* g_gemm_prof = nullptr;
static bool g_gemm_prof_on = false;

void gemm_profile(bool on) {
  if (on && !g_gemm_prof) C10_CUDA_CHECK(cudaMalloc(&g_gemm_prof, 8 * sizeof(unsigned long long)));
  if (g_gemm_prof) C10_CUDA_CHECK(cudaMemset(g_gemm_prof, 0, 8 * sizeof(unsigned long long)));
  g_gemm_prof_on = on;
}

std::vector<int64_t> gemm_profile_read() {
  std::vector<int64_t> out(8, 0);
  if (!g_gemm_prof) return out;
  unsigned long long h[8];
  C10_CUDA_CHECK(cudaMemcpy(h, g_gemm_prof, sizeof(h), cudaMemcpyDeviceToHost));
  for (int i = 0; i < 8; ++i) out[i] = (int64_t)h[i];
  return out;
}

static GemmEpilogue build_epilogue(at::Tensor& D, int64_t M, int64_t N,
                                   const c10::optional<at::Tensor>& bias,
                                   const c10::optional<at::Tensor>& residual,
                                   const c10::optional<at::Tensor>& act,
                                   const c10::optional<at::Tensor>& aux,
                                   const c10::optional<at::Tensor>& alpha,
                                   const c10::optional<at::Tensor>& alpha2, bool beta) {
  TORCH_CHECK(D.dim() == 2 && D.size(0) == M && D.size(1) == N && D.stride(1) == 1,
              "gemm: D must be [M, N] with unit inner stride");
  TORCH_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  const bool out_f32 = D.scalar_type() == at::kFloat;
  TORCH_CHECK(out_f32 || D.scalar_type() == at::kBFloat16, "gemm: D must be bf16 or fp32");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(D.data_ptr()) % 16 == 0 && (D.stride(0) % 8) == 0,
              "gemm: D alignment");
  GemmEpilogue ep{};
  ep.D = D.data_ptr();
  ep.ldd = D.stride(0);
  ep.out_f32 = out_f32;
  ep.beta = beta ? 1 : 0;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == N, "bias must be fp32 [N]");
    ep.bias = bias->data_ptr<float>();
  }
  if (residual.has_value()) {
    TORCH_CHECK(!out_f32 && residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1,
                "residual must be bf16 with bf16 output");
    ep.residual = reinterpret_cast<const bf16*>(residual->data_ptr());
    ep.ldr = residual->stride(0);
  }
  if (act.has_value()) {
    TORCH_CHECK(!out_f32 && act->scalar_type() == at::kBFloat16 && act->stride(1) == 1, "act");
    ep.act = reinterpret_cast<bf16*>(act->data_ptr());
    ep.ldact = act->stride(0);
  }
  if (aux.has_value()) {
    TORCH_CHECK(aux->scalar_type() == at::kBFloat16 && aux->stride(1) == 1, "aux");
    ep.aux = reinterpret_cast<const bf16*>(aux->data_ptr());
    ep.ldaux = aux->stride(0);
  }
  if (alpha.has_value()) {
    TORCH_CHECK(alpha->scalar_type() == at::kFloat, "alpha must be an fp32 device scalar");
    ep.alpha = alpha->data_ptr<float>();
  }
  if (alpha2.has_value()) {
    TORCH_CHECK(alpha2->scalar_type() == at::kFloat, "alpha2 must be an fp32 device scalar");
    ep.alpha2 = alpha2->data_ptr<float>();
  }
  return ep;
}

// Dropout for the next CTA-pair GEMM launch only (gemm_set_dropout; consumed and
// cleared by that launch): the epilogue draws the mask of a site (see DROP in
// epi_chunk_store).  Setting it for one call keeps every GEMM entry point's
// signature unchanged.
static DropoutArgs g_next_drop{};
static int g_next_drop_mode = 0;

void gemm_set_dropout(const c10::optional<at::Tensor>& rng, int64_t site, int64_t thr16, double scale,
                      int64_t mode) {
  g_next_drop = DropoutArgs{};
  g_next_drop_mode = 0;
  if (!rng.has_value()) return;
  TORCH_CHECK(rng->is_cuda() && rng->scalar_type() == at::kInt && rng->numel() >= 2, "gemm dropout: int32 rng key");
  TORCH_CHECK(mode >= 1 && mode <= 3 && thr16 >= 0 && thr16 < 65536 && scale >= 1.0, "gemm dropout: mode 1..3, 0 <= p < 1");
  g_next_drop.rng = reinterpret_cast<const uint32_t*>(rng->data_ptr<int32_t>());
  g_next_drop.site = (uint32_t)site;
  g_next_drop.thr16 = (uint32_t)thr16;
  g_next_drop.scale = (float)scale;
  g_next_drop_mode = (int)mode;
}

template <int EB, bool MX = false>
static void launch_pair(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor& D,
                        const c10::optional<at::Tensor>& act, const GemmEpilogue& ep, int64_t M,
                        int64_t N, int64_t K, uint32_t idesc, const at::Tensor* sfa = nullptr,
                        const at::Tensor* sfb = nullptr, const std::vector<int64_t>* b_peers = nullptr,
                        int64_t shard_rows = 0, const MxOutArgs* mxo = nullptr, const at::Tensor* mx_rc = nullptr,
                        const at::Tensor* mx_cc = nullptr) {
  const auto dt = EB == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const auto swz = CU_TENSOR_MAP_SWIZZLE_128B;
  constexpr uint32_t BK = 128 / EB, MN_BOX = 128 / EB;
  // per-CTA boxes: 128 rows of A and 128 rows of B (the pair covers 256 x 256)
  CUtensorMap ta = a_mn ? make_tma_2d(A.data_ptr(), dt, EB, M, K, A.stride(0), MN_BOX, BK, swz)
                        : make_tma_2d(A.data_ptr(), dt, EB, K, M, A.stride(0), BK, P_BM, swz);
  auto map_b = [&](const void* ptr) {
    return b_mn ? make_tma_2d(ptr, dt, EB, N, K, B.stride(0), MN_BOX, BK, swz)
                : make_tma_2d(ptr, dt, EB, K, N, B.stride(0), BK, P_BN / 2, swz);
  };
  CUtensorMap tb = map_b(B.data_ptr());
  PeerMapsB pb;
  std::memset(&pb, 0, sizeof(pb));
  if (b_peers) {
    pb.n = (int)b_peers->size();
    pb.shard_rows = (int)shard_rows;
    for (int p = 0; p < pb.n; ++p) pb.m[p] = map_b(reinterpret_cast<const void*>((*b_peers)[p]));
  }
  const bool out_f32 = ep.out_f32 != 0;
  CUtensorMap td = out_f32
      ? make_tma_2d(D.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, D.stride(0), 32, 32,
                    CU_TENSOR_MAP_SWIZZLE_128B)
      : make_tma_2d(D.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, D.stride(0), 32, 32,
                    CU_TENSOR_MAP_SWIZZLE_64B);
  CUtensorMap tact = act.has_value()
      ? make_tma_2d(act->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, act->stride(0), 32, 32,
                    CU_TENSOR_MAP_SWIZZLE_64B)
      : ep.act8 ? make_tma_2d(ep.act8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, M, N, 32, 32,
                              CU_TENSOR_MAP_SWIZZLE_NONE)
      : mx_rc   ? make_tma_2d(mx_rc->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, M, N, 32, 32,
                              CU_TENSOR_MAP_SWIZZLE_NONE)
                : td;
  // MXFP8 output: column codes [N, M], one 32 x 32-byte box per epilogue chunk
  CUtensorMap tcc = mx_cc ? make_tma_2d(mx_cc->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, N, M, 32, 32,
                                        CU_TENSOR_MAP_SWIZZLE_NONE)
                          : td;
  const MxOutArgs mo = mxo ? *mxo : MxOutArgs{};
  // scale tensors viewed as rows of 256 bytes (an atom is two rows); x is always 0
  const int64_t sf_kb = (K + 127) / 128;
  CUtensorMap tsfa = MX ? make_tma_2d(sfa->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 256,
                                      sfa->numel() / 256, 256, 256, 2, CU_TENSOR_MAP_SWIZZLE_NONE)
                        : td;
  CUtensorMap tsfb = MX ? make_tma_2d(sfb->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 256,
                                      sfb->numel() / 256, 256, 256, 2, CU_TENSOR_MAP_SWIZZLE_NONE)
                        : td;
  const int num_tiles = (int)(((M + 2 * P_BM - 1) / (2 * P_BM)) * ((N + P_BN - 1) / P_BN));
  const int avail_pairs = std::max(1, (num_sms() - g_reserved_sms) / 2);
  const int pairs = std::min(num_tiles, avail_pairs);
  constexpr int NST = pair_stages<MX>();
  const size_t smem = NST * P_STAGE_BYTES + epi_bytes<MX>() + (MX ? NST * P_SF_BYTES : 0) + sizeof(PairSmem) + 1024;
  static_assert(NST * P_STAGE_BYTES + epi_bytes<MX>() + (MX ? NST * P_SF_BYTES : 0) + sizeof(PairSmem) + 1024 <= 232448,
                "CTA-pair GEMM: shared memory above the 227 KB per-CTA limit");
  const DropoutArgs drop = g_next_drop;
  const int drop_mode = g_next_drop_mode;
  g_next_drop = DropoutArgs{};
  g_next_drop_mode = 0;
  if (drop.rng)
    TORCH_CHECK((drop_mode != 1 || ep.residual) && (drop_mode != 2 || ep.act || ep.act8 || (mxo && mo.src_act)) &&
                    (drop_mode != 3 || ep.aux),
                "gemm dropout: mode 1 needs a residual, 2 a GELU output, 3 a dGELU input");
  // one instance per (dropout, MXFP8 output); each sets its shared-memory limit once
  auto go = [&](auto drop_c, auto mxo_c) {
    constexpr bool kDrop = decltype(drop_c)::value;
    constexpr bool kMxo = decltype(mxo_c)::value && MX;
    static bool attr_set = false;
    if (!attr_set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_2sm_kernel<EB, MX, kDrop, kMxo>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      attr_set = true;
    }
    gemm_2sm_kernel<EB, MX, kDrop, kMxo><<<2 * pairs, kPairThreads, smem, cur_stream()>>>(
        ta, tb, td, tact, tsfa, tsfb, pb, (int)M, (int)N, (int)K, a_mn ? 1 : 0, b_mn ? 1 : 0, (int)sf_kb,
        idesc, ep, gemm_status_ptr(), g_gemm_prof_on ? g_gemm_prof : nullptr, drop, kDrop ? drop_mode : 0, tcc,
        mo);
    MT_LAUNCH_CHECK();
  };
  using T = std::true_type;
  using F = std::false_type;
  if (mxo) {
    if (drop.rng) go(T{}, T{}); else go(F{}, T{});
  } else {
    if (drop.rng) go(T{}, F{}); else go(F{}, F{});
  }
}

// A: [M,K] (a_mn=false) or [K,M] (a_mn=true); B: [N,K] (b_mn=false) or [K,N] (b_mn=true).
void gemm_bf16(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor D,
               const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
               const c10::optional<at::Tensor>& act, const c10::optional<at::Tensor>& aux,
               const c10::optional<at::Tensor>& alpha, bool beta) {
  check_operand(A, "A", 2);
  check_operand(B, "B", 2);
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm_bf16: bf16 operands");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  const int64_t Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "gemm_bf16: K mismatch ", K, " vs ", Kb);
  GemmEpilogue ep = build_epilogue(D, M, N, bias, residual, act, aux, alpha, c10::nullopt, beta);
  if (M == 0 || N == 0) return;
  ensure_context();
  if (K == 0) {
    if (!beta) D.zero_();
    return;
  }
  static const bool force_1sm = std::getenv("MTORUS_GEMM_1SM") != nullptr;
  TORCH_CHECK(!g_next_drop.rng || (M >= 2 * P_BM && !force_1sm), "gemm dropout needs M >= 256 (the CTA-pair kernel)");
  if (M >= 2 * P_BM && !force_1sm) {
    launch_pair<2>(A, a_mn, B, b_mn, D, act, ep, M, N, K,
                   make_idesc_bf16(2 * P_BM, P_BN, a_mn ? 1 : 0, b_mn ? 1 : 0));
    return;
  }
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto swz = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap ta = a_mn ? make_tma_2d(A.data_ptr(), dt, 2, M, K, A.stride(0), 64, BK, swz)
                        : make_tma_2d(A.data_ptr(), dt, 2, K, M, A.stride(0), BK, BM, swz);
  CUtensorMap tb = b_mn ? make_tma_2d(B.data_ptr(), dt, 2, N, K, B.stride(0), 64, BK, swz)
                        : make_tma_2d(B.data_ptr(), dt, 2, K, N, B.stride(0), BK, BN, swz);
  const int num_tiles = (int)(((M + BM - 1) / BM) * ((N + BN - 1) / BN));
  const int grid = std::min(num_tiles, std::max(1, num_sms() - g_reserved_sms));
  const size_t smem = STAGES * STAGE_BYTES + sizeof(Smem) + 1024;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_bf16_tn_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set = true;
  }
  gemm_bf16_tn_kernel<<<grid, kThreads, smem, cur_stream()>>>(ta, tb, (int)M, (int)N, (int)K,
                                                               a_mn ? 1 : 0, b_mn ? 1 : 0, ep,
                                                               gemm_status_ptr());
  MT_LAUNCH_CHECK();
}

// FP8 GEMM (tcgen05 kind::f8f6f4, fp32 accumulate): A / B are 1-byte E4M3 (fmt 0)
// or E5M2 (fmt 1) codes; the epilogue multiplies by alpha * alpha2 (the operands'
// inverse scales) before bias / residual / GELU / dGELU / fp32 accumulate.
void gemm_fp8_act8(const at::Tensor& A, bool a_mn, int64_t a_fmt, const at::Tensor& B, bool b_mn,
                   int64_t b_fmt, at::Tensor D, const c10::optional<at::Tensor>& bias,
                   const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& act,
                   const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& alpha,
                   const c10::optional<at::Tensor>& alpha2, bool beta,
                   const c10::optional<at::Tensor>& act8, const c10::optional<at::Tensor>& act8_scale,
                   const c10::optional<at::Tensor>& act8_amax, int64_t act8_fmt);

void gemm_fp8(const at::Tensor& A, bool a_mn, int64_t a_fmt, const at::Tensor& B, bool b_mn,
              int64_t b_fmt, at::Tensor D, const c10::optional<at::Tensor>& bias,
              const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& act,
              const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& alpha,
              const c10::optional<at::Tensor>& alpha2, bool beta) {
  gemm_fp8_act8(A, a_mn, a_fmt, B, b_mn, b_fmt, D, bias, residual, act, aux, alpha, alpha2, beta, c10::nullopt,
                c10::nullopt, c10::nullopt, 0);
}

// gemm_fp8 whose epilogue may also write GELU(result) as FP8 codes (act8, uint8 [M, N]
// contiguous) with the role's scale, folding max|GELU| into act8_amax.
void gemm_fp8_act8(const at::Tensor& A, bool a_mn, int64_t a_fmt, const at::Tensor& B, bool b_mn,
                   int64_t b_fmt, at::Tensor D, const c10::optional<at::Tensor>& bias,
                   const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& act,
                   const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& alpha,
                   const c10::optional<at::Tensor>& alpha2, bool beta,
                   const c10::optional<at::Tensor>& act8, const c10::optional<at::Tensor>& act8_scale,
                   const c10::optional<at::Tensor>& act8_amax, int64_t act8_fmt) {
  check_operand(A, "A", 1);
  check_operand(B, "B", 1);
  TORCH_CHECK((a_fmt == 0 || a_fmt == 1) && (b_fmt == 0 || b_fmt == 1), "gemm_fp8: formats are 0 (E4M3) / 1 (E5M2)");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  const int64_t Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "gemm_fp8: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(K % 16 == 0, "gemm_fp8: K must be a multiple of 16");
  TORCH_CHECK(!a_mn || M % 16 == 0, "gemm_fp8: M must be a multiple of 16 for an MN-major A");
  TORCH_CHECK(!b_mn || N % 16 == 0, "gemm_fp8: N must be a multiple of 16 for an MN-major B");
  GemmEpilogue ep = build_epilogue(D, M, N, bias, residual, act, aux, alpha, alpha2, beta);
  if (act8.has_value()) {
    TORCH_CHECK(!act.has_value() && act8_scale.has_value() && act8_amax.has_value(),
                "gemm_fp8: act8 needs act8_scale and act8_amax and excludes act");
    TORCH_CHECK(act8->element_size() == 1 && act8->is_contiguous() && act8->numel() == M * N &&
                    reinterpret_cast<uintptr_t>(act8->data_ptr()) % 16 == 0 && N % 16 == 0 && M >= 2 * P_BM,
                "gemm_fp8: act8 must be a 16-byte aligned contiguous uint8 [M, N], N % 16 == 0, M >= 256");
    ep.act8 = reinterpret_cast<uint8_t*>(act8->data_ptr());
    ep.act8_scale = act8_scale->data_ptr<float>();
    ep.act8_amax = act8_amax->data_ptr<float>();
    ep.act8_fmt = (int)act8_fmt;
  }
  if (M == 0 || N == 0) return;
  ensure_context();
  launch_pair<1>(A, a_mn, B, b_mn, D, act, ep, M, N, K,
                 make_idesc_f8(2 * P_BM, P_BN, (int)a_fmt, (int)b_fmt, a_mn ? 1 : 0, b_mn ? 1 : 0));
}

// FP8 GEMM whose B operand is sharded by storage rows over the ranks of a symmetric
// buffer and read from each owner's memory inside the kernel (see PeerMapsB): the
// all-gather of B fused into the GEMM.  B is this rank's view of the full buffer
// (shape and strides of the gathered operand); b_peers[p] is rank p's address of the
// same bytes; rank p's rows are [p * shard_rows, (p + 1) * shard_rows).  The caller
// orders the owners' writes before the launch (a barrier over the ranks).
void gemm_fp8_gather_b(const at::Tensor& A, bool a_mn, int64_t a_fmt, const at::Tensor& B, bool b_mn,
                       int64_t b_fmt, const std::vector<int64_t>& b_peers, int64_t shard_rows, at::Tensor D,
                       const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
                       const c10::optional<at::Tensor>& act, const c10::optional<at::Tensor>& aux,
                       const c10::optional<at::Tensor>& alpha, const c10::optional<at::Tensor>& alpha2, bool beta) {
  check_operand(A, "A", 1);
  check_operand(B, "B", 1);
  TORCH_CHECK((a_fmt == 0 || a_fmt == 1) && (b_fmt == 0 || b_fmt == 1), "gemm_fp8_gather_b: formats 0 / 1");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  TORCH_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "gemm_fp8_gather_b: K mismatch");
  TORCH_CHECK(K % 16 == 0 && (!a_mn || M % 16 == 0) && (!b_mn || N % 16 == 0), "gemm_fp8_gather_b: alignment");
  const int64_t n = (int64_t)b_peers.size();
  TORCH_CHECK(n >= 1 && n <= 8, "gemm_fp8_gather_b: 1..8 owners");
  // a CTA's B box (128 rows of a K-major B) or k-block (128 K of an MN-major B) has one owner
  TORCH_CHECK(shard_rows > 0 && shard_rows % 128 == 0, "gemm_fp8_gather_b: shard_rows must be a multiple of 128");
  TORCH_CHECK(B.size(0) <= n * shard_rows, "gemm_fp8_gather_b: the shards do not cover B's rows");
  for (int64_t p : b_peers) TORCH_CHECK(p != 0 && p % 16 == 0, "gemm_fp8_gather_b: 16-byte aligned peer addresses");
  GemmEpilogue ep = build_epilogue(D, M, N, bias, residual, act, aux, alpha, alpha2, beta);
  if (M == 0 || N == 0) return;
  ensure_context();
  launch_pair<1>(A, a_mn, B, b_mn, D, act, ep, M, N, K,
                 make_idesc_f8(2 * P_BM, P_BN, (int)a_fmt, (int)b_fmt, a_mn ? 1 : 0, b_mn ? 1 : 0), nullptr, nullptr,
                 &b_peers, shard_rows);
}

// MXFP8 GEMM (tcgen05 kind::mxf8f6f4, 1x32 UE8M0 block scales, fp32 accumulate):
// D = epilogue(alpha * sum_k (A[m,k] 2^sa[m,k/32]) (B[n,k] 2^sb[n,k/32])).  A [M, K] and
// B [N, K] are K-major E4M3 / E5M2 codes; sfa / sfb hold one biased exponent byte
// (UE8M0, 127 = 2^0) per 32-element K block in the tcgen05 atom layout written by
// mx_quantize: [ceil(rows / 128)][ceil(K / 128)][512], byte (r % 32) * 16 + (r % 128 / 32) * 4
// + (k / 32) % 4 of atom (r / 128, k / 128).
void gemm_mxfp8(const at::Tensor& A, int64_t a_fmt, const at::Tensor& sfa, const at::Tensor& B,
                int64_t b_fmt, const at::Tensor& sfb, at::Tensor D, const c10::optional<at::Tensor>& bias,
                const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& act,
                const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& alpha, bool beta,
                const c10::optional<at::Tensor>& out_rc, const c10::optional<at::Tensor>& out_rsf,
                const c10::optional<at::Tensor>& out_cc, const c10::optional<at::Tensor>& out_csf, int64_t out_fmt,
                double out_fmax, const c10::optional<at::Tensor>& out_colsum, bool out_gelu, bool store_d) {
  check_operand(A, "A", 1);
  check_operand(B, "B", 1);
  TORCH_CHECK((a_fmt == 0 || a_fmt == 1) && (b_fmt == 0 || b_fmt == 1), "gemm_mxfp8: formats are 0 (E4M3) / 1 (E5M2)");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K, "gemm_mxfp8: K mismatch ", K, " vs ", B.size(1));
  TORCH_CHECK(K % 32 == 0, "gemm_mxfp8: K must be a multiple of 32 (one scale per 32 elements)");
  const int64_t kb = (K + 127) / 128;
  auto check_sf = [&](const at::Tensor& sf, int64_t rows, const char* name) {
    TORCH_CHECK(sf.is_cuda() && sf.element_size() == 1 && sf.is_contiguous(), name, ": contiguous uint8 on the GPU");
    TORCH_CHECK(sf.numel() == (rows + 127) / 128 * kb * P_SF_ATOM, name, ": expected ", (rows + 127) / 128 * kb * P_SF_ATOM,
                " scale bytes (the mx_quantize layout), got ", sf.numel());
    TORCH_CHECK(reinterpret_cast<uintptr_t>(sf.data_ptr()) % 16 == 0, name, ": 16-byte aligned base required");
  };
  check_sf(sfa, M, "sfa");
  check_sf(sfb, N, "sfb");
  GemmEpilogue ep = build_epilogue(D, M, N, bias, residual, act, aux, alpha, c10::nullopt, beta);
  const bool mx_out = out_rc.has_value();
  MxOutArgs mo{};
  if (mx_out) {
    // MXFP8 output (row and column codes with their scale atoms) written by the epilogue
    TORCH_CHECK(out_rsf.has_value() && out_cc.has_value() && out_csf.has_value(),
                "gemm_mxfp8: MX output needs rc, rsf, cc and csf");
    TORCH_CHECK(M % 128 == 0 && N % 128 == 0, "gemm_mxfp8: MX output needs M and N multiples of 128");
    TORCH_CHECK(D.scalar_type() == at::kBFloat16 && !beta && !act.has_value() && !residual.has_value(),
                "gemm_mxfp8: MX output with a bf16 D, no accumulate, no bf16 GELU output and no residual");
    TORCH_CHECK(out_fmt == 0 || out_fmt == 1, "gemm_mxfp8: MX output format 0 (E4M3) / 1 (E5M2)");
    auto chk = [](const at::Tensor& t, int64_t n, const char* what) {
      TORCH_CHECK(t.is_cuda() && t.element_size() == 1 && t.is_contiguous() && t.numel() == n &&
                      reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
                  what);
    };
    chk(*out_rc, M * N, "gemm_mxfp8: rc must be 16-byte aligned contiguous uint8 [M, N]");
    chk(*out_cc, M * N, "gemm_mxfp8: cc must be 16-byte aligned contiguous uint8 [N, M]");
    chk(*out_rsf, (M / 128) * (N / 128) * P_SF_ATOM, "gemm_mxfp8: rsf size");
    chk(*out_csf, (M / 128) * (N / 128) * P_SF_ATOM, "gemm_mxfp8: csf size");
    if (out_colsum.has_value())
      TORCH_CHECK(out_colsum->scalar_type() == at::kFloat && out_colsum->is_contiguous() && out_colsum->numel() == N,
                  "gemm_mxfp8: colsum must be fp32 [N]");
    const float fm = (float)out_fmax;
    std::memcpy(&mo.fmax_bits, &fm, 4);
    mo.rsf = reinterpret_cast<uint8_t*>(out_rsf->data_ptr());
    mo.csf = reinterpret_cast<uint8_t*>(out_csf->data_ptr());
    mo.colsum = out_colsum.has_value() ? out_colsum->data_ptr<float>() : nullptr;
    mo.fmt = (int)out_fmt;
    mo.src_act = out_gelu ? 1 : 0;
    mo.store_d = store_d ? 1 : 0;
  }
  if (M == 0 || N == 0) return;
  ensure_context();
  launch_pair<1, true>(A, false, B, false, D, act, ep, M, N, K, make_idesc_mx(2 * P_BM, P_BN, (int)a_fmt, (int)b_fmt),
                       &sfa, &sfb, nullptr, 0, mx_out ? &mo : nullptr, mx_out ? &*out_rc : nullptr,
                       mx_out ? &*out_cc : nullptr);
}

}  // namespace mtorus
