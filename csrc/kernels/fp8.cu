// FP8 quantisation with delayed (amax-history) scaling, on device.
//
// Reference semantics (crates/mt-core/src/precision/{quantize,scaling}.rs):
//   scale  = format_max / amax (1 when amax == 0), stored = fp8(x * scale),
//   DelayedScaling: amax ring buffer of `history` entries, current amax = max of
//   the ring, the scale used in step t comes from the history up to step t-1.
//
// Design (B200): one fused pass per tensor reads bf16, multiplies by the current
// scale (a device scalar: no host sync), converts two values at a time with the
// saturating round-to-nearest-even cvt (cvt.rn.satfinite.{e4m3,e5m2}x2), writes
// 1-byte codes with 16-byte stores and folds max|x| into the slot's running
// amax with one atomic per block.  After the step one tiny kernel rolls every
// slot's ring buffer and recomputes scale / inverse scale for all slots at once.
#include <cstring>

#include "amax_publish.cuh"
#include "gelu.cuh"
#include "mx.cuh"

namespace mtorus {



template <int FMT>  // 0 = E4M3, 1 = E5M2
__global__ void __launch_bounds__(256) fp8_quantize_kernel(const bf16* __restrict__ x,
                                                           uint8_t* __restrict__ out,
                                                           const float* __restrict__ scale,
                                                           float* __restrict__ amax, size_t n) {
  __shared__ float red[32];
  const float s = scale ? *scale : 1.f;
  float m = 0.f;
  const size_t nv = n / 16;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nv;
       i += (size_t)gridDim.x * blockDim.x) {
    float f[16];
    unpack8(reinterpret_cast<const bf16x8*>(x)[2 * i], f);
    unpack8(reinterpret_cast<const bf16x8*>(x)[2 * i + 1], f + 8);
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      m = fmaxf(m, fmaxf(fmaxf(fabsf(f[4 * k]), fabsf(f[4 * k + 1])),
                         fmaxf(fabsf(f[4 * k + 2]), fabsf(f[4 * k + 3]))));
      const uint16_t lo = FMT == 0 ? cvt2_e4m3(f[4 * k] * s, f[4 * k + 1] * s)
                                   : cvt2_e5m2(f[4 * k] * s, f[4 * k + 1] * s);
      const uint16_t hi = FMT == 0 ? cvt2_e4m3(f[4 * k + 2] * s, f[4 * k + 3] * s)
                                   : cvt2_e5m2(f[4 * k + 2] * s, f[4 * k + 3] * s);
      w[k] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (size_t i = nv * 16 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float f = __bfloat162float(x[i]);
    m = fmaxf(m, fabsf(f));
    const uint16_t c = FMT == 0 ? cvt2_e4m3(f * s, 0.f) : cvt2_e5m2(f * s, 0.f);
    out[i] = (uint8_t)(c & 0xFF);
  }
  if (amax) {
    m = block_max(m, red);
    if (threadIdx.x == 0) atomic_max_pos(amax, m);
  }
}

// ---------------------------------------------------------------- amax all-reduce (fused)
// Data parallel: every rank quantises its own activations / gradients, so the
// delayed-scaling amax of a tensor role is the max over ranks.  The quantise
// kernel below publishes its rank's running amax for the slot into every peer's
// symmetric table, from its last block (a per-slot arrival counter finds it):
//     table[parity][me][slot] = (epoch << 32) | float_bits(amax)     (one u64 store)
// At the end of the step, after a flag barrier, fp8_amax_gather takes the max
// over ranks of the entries stamped with this step's epoch.  The table is
// double-buffered by step parity, so a peer that already runs the next step
// writes the other half.
// Quantise a [rows, F] bf16 gradient and add its column sums into `colsum` (the
// bias gradient) in the same pass: blocks of 32 column groups of 8 x 8 row lanes,
// 16-byte loads, 8-byte code stores, per-block column partials in shared memory
// and one atomic per column.  Amax / all-reduce publication as above.
template <int FMT>
__global__ void __launch_bounds__(256) fp8_quantize_colsum_kernel(
    const bf16* __restrict__ x, uint8_t* __restrict__ out, const float* __restrict__ scale,
    float* __restrict__ amax, float* __restrict__ colsum, int rows, int F, int rows_per_block,
    unsigned int* __restrict__ counter, AmaxPeers table, int me, int world, int cap, int slot, int parity,
    unsigned int epoch) {
  __shared__ float red[8][257];
  __shared__ float redm[32];
  __shared__ bool last;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 256 + tx * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  const float s = *scale;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float m = 0.f;
  if (c0 < F) {
    for (int r = r0 + ty; r < r1; r += 8) {
      float f[8];
      unpack8(*reinterpret_cast<const bf16x8*>(x + (size_t)r * F + c0), f);
      uint32_t w[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[4 * k + j] += f[4 * k + j];
          m = fmaxf(m, fabsf(f[4 * k + j]));
        }
        const uint16_t lo = FMT == 0 ? cvt2_e4m3(f[4 * k] * s, f[4 * k + 1] * s)
                                     : cvt2_e5m2(f[4 * k] * s, f[4 * k + 1] * s);
        const uint16_t hi = FMT == 0 ? cvt2_e4m3(f[4 * k + 2] * s, f[4 * k + 3] * s)
                                     : cvt2_e5m2(f[4 * k + 2] * s, f[4 * k + 3] * s);
        w[k] = (uint32_t)lo | ((uint32_t)hi << 16);
      }
      *reinterpret_cast<uint2*>(out + (size_t)r * F + c0) = make_uint2(w[0], w[1]);
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
    atomicAdd(colsum + blockIdx.x * 256 + col, t);
  }
  m = block_max(m, redm);
  publish_amax(m, amax, counter, table, me, world, cap, slot, parity, epoch, &last);
}

template <int FMT>
__global__ void __launch_bounds__(256) fp8_quantize_ar_kernel(const bf16* __restrict__ x,
                                                              uint8_t* __restrict__ out,
                                                              const float* __restrict__ scale,
                                                              float* __restrict__ amax, size_t n,
                                                              unsigned int* __restrict__ counter,
                                                              AmaxPeers table, int me, int world, int cap,
                                                              int slot, int parity, unsigned int epoch) {
  __shared__ float red[32];
  __shared__ bool last;
  const float s = scale ? *scale : 1.f;
  float m = 0.f;
  const size_t nv = n / 16;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nv;
       i += (size_t)gridDim.x * blockDim.x) {
    float f[16];
    unpack8(reinterpret_cast<const bf16x8*>(x)[2 * i], f);
    unpack8(reinterpret_cast<const bf16x8*>(x)[2 * i + 1], f + 8);
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      m = fmaxf(m, fmaxf(fmaxf(fabsf(f[4 * k]), fabsf(f[4 * k + 1])),
                         fmaxf(fabsf(f[4 * k + 2]), fabsf(f[4 * k + 3]))));
      const uint16_t lo = FMT == 0 ? cvt2_e4m3(f[4 * k] * s, f[4 * k + 1] * s)
                                   : cvt2_e5m2(f[4 * k] * s, f[4 * k + 1] * s);
      const uint16_t hi = FMT == 0 ? cvt2_e4m3(f[4 * k + 2] * s, f[4 * k + 3] * s)
                                   : cvt2_e5m2(f[4 * k + 2] * s, f[4 * k + 3] * s);
      w[k] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (size_t i = nv * 16 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float f = __bfloat162float(x[i]);
    m = fmaxf(m, fabsf(f));
    const uint16_t c = FMT == 0 ? cvt2_e4m3(f * s, 0.f) : cvt2_e5m2(f * s, 0.f);
    out[i] = (uint8_t)(c & 0xFF);
  }
  m = block_max(m, red);
  publish_amax(m, amax, counter, table, me, world, cap, slot, parity, epoch, &last);
}

// amax[s] = max over ranks r of table[parity][r][s] entries stamped with `epoch`
// (plus *ep when a device step counter is given; parity is then its low bit).
__global__ void fp8_amax_gather_kernel(const unsigned long long* __restrict__ table, float* __restrict__ amax,
                                       int slots, int world, int cap, int parity, unsigned int epoch,
                                       const unsigned int* ep) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= slots) return;
  if (ep) {
    epoch += *ep;
    parity = (int)(epoch & 1u);
  }
  float m = amax[s];
  for (int r = 0; r < world; ++r) {
    const unsigned long long v =
        *reinterpret_cast<const volatile unsigned long long*>(table + ((size_t)parity * world + r) * cap + s);
    if ((unsigned int)(v >> 32) == epoch) m = fmaxf(m, __uint_as_float((unsigned int)(v & 0xffffffffu)));
  }
  amax[s] = m;
}

__global__ void __launch_bounds__(256) amax_kernel(const bf16* __restrict__ x, float* __restrict__ amax,
                                                   size_t n) {
  __shared__ float red[32];
  float m = 0.f;
  const size_t nv = n / 8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nv;
       i += (size_t)gridDim.x * blockDim.x) {
    float f[8];
    unpack8(reinterpret_cast<const bf16x8*>(x)[i], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) m = fmaxf(m, fabsf(f[k]));
  }
  for (size_t i = nv * 8 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(x[i])));
  m = block_max(m, red);
  if (threadIdx.x == 0) atomic_max_pos(amax, m);
}

// Roll the ring buffers of all slots:  hist[s][cursor] = amax[s]; amax[s] = 0;
// scale[s] = fmax[s] / max(hist[s]) (1 if 0); inv[s] = 1 / scale[s].
// When `current` is set the scale comes from the amax just measured (used for
// the very first step, whose history is still empty).
__global__ void fp8_scaling_update_kernel(float* __restrict__ hist, float* __restrict__ amax,
                                          float* __restrict__ scale, float* __restrict__ inv,
                                          const float* __restrict__ fmax_per_slot, int slots,
                                          int H, int cursor, int current, const int* cursor_dev) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= slots) return;
  if (cursor_dev) cursor = *cursor_dev;  // device-resident ring position (graph replay)
  const float a = amax[s];
  float* h = hist + (size_t)s * H;
  h[cursor] = a;
  float m = 0.f;
  for (int i = 0; i < H; ++i) m = fmaxf(m, h[i]);
  if (current) m = a;
  const float sc = m > 0.f ? fmax_per_slot[s] / m : 1.f;
  scale[s] = sc;
  inv[s] = 1.f / sc;
  amax[s] = 0.f;
}

template <int FMT>
__global__ void fp8_dequantize_kernel(const uint8_t* __restrict__ q, float* __restrict__ out,
                                      const float* __restrict__ inv_scale, size_t n) {
  const float s = *inv_scale;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    if (FMT == 0) {
      __nv_fp8_e4m3 v;
      v.__x = q[i];
      out[i] = float(v) * s;
    } else {
      __nv_fp8_e5m2 v;
      v.__x = q[i];
      out[i] = float(v) * s;
    }
  }
}

// Per-block quantisation (reference to_fp8_per_block): each block of `bs`
// consecutive values gets scale = fmax / amax(block) (1 if 0).  One warp per block.
template <int FMT>
__global__ void fp8_quantize_blocks_kernel(const float* __restrict__ x, uint8_t* __restrict__ out,
                                           float* __restrict__ scales, size_t n, int bs, float fmax,
                                           size_t nblocks) {
  const size_t b = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (b >= nblocks) return;
  const size_t s0 = b * bs, s1 = min(n, s0 + (size_t)bs);
  float m = 0.f;
  for (size_t i = s0 + lane; i < s1; i += 32) m = fmaxf(m, fabsf(x[i]));
  m = warp_max(m);
  const float sc = m > 0.f ? fmax / m : 1.f;
  if (lane == 0) scales[b] = sc;
  for (size_t i = s0 + lane; i < s1; i += 32) {
    const uint16_t c = FMT == 0 ? cvt2_e4m3(x[i] * sc, 0.f) : cvt2_e5m2(x[i] * sc, 0.f);
    out[i] = (uint8_t)(c & 0xFF);
  }
}

// MXFP8 quantisation (OCP MX: 32-element blocks along a row, one UE8M0 scale each)
// for the block-scaled GEMM.  The block's shared exponent X is the smallest integer
// with amax <= fmax * 2^X, so no element saturates; codes = fp8(x * 2^-X) and the
// scale byte is X + 127 (clamped to [0, 254]; 255 = NaN marks a block holding a
// NaN or Inf, which the GEMM turns into NaN outputs).  An all-zero block gets X = 0.
// X comes from the IEEE-754 fields: with amax = (1 + ma) 2^ea and fmax = (1 + mf) 2^ef,
// X = ea - ef + (ma > mf).  Scales go to the tcgen05 atom layout (see gemm_mxfp8);
// padding rows / K blocks of the last atoms get 127.  One thread per block of 32.
template <int FMT>
__global__ void __launch_bounds__(256) mx_quantize_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                          uint8_t* __restrict__ codes, uint8_t* __restrict__ sf,
                                                          int R, int K, int nkb4, uint32_t fmax_bits) {
  const int jper = nkb4 * 4;  // 32-blocks per padded row
  const int64_t total = (int64_t)((R + 127) / 128) * 128 * jper;
  const int kblocks = K / 32;
  const int ef = (int)((fmax_bits >> 23) & 0xFF);
  const uint32_t mf = fmax_bits & 0x7FFFFF;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(idx % jper);
    const int r = (int)(idx / jper);
    const int rr = r & 127;
    const int64_t so = ((int64_t)(r >> 7) * nkb4 + (j >> 2)) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + (j & 3);
    if (r >= R || j >= kblocks) {
      sf[so] = 127;
      continue;
    }
    const bf16x8* src = reinterpret_cast<const bf16x8*>(x + (int64_t)r * ldx + (int64_t)j * 32);
    float v[32];
#pragma unroll
    for (int q = 0; q < 4; ++q) unpack8(src[q], v + 8 * q);
    float amax = 0.f;
    bool finite = true;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      amax = fmaxf(amax, fabsf(v[i]));
      finite &= isfinite(v[i]);
    }
    int X = 0;
    if (amax > 0.f) {
      const uint32_t ua = __float_as_uint(amax);
      X = (int)((ua >> 23) & 0xFF) - ef + ((ua & 0x7FFFFF) > mf ? 1 : 0);
      X = max(-127, min(127, X));
    }
    const float inv = __uint_as_float((uint32_t)(127 - min(X, 126)) << 23);  // 2^-X (X <= 126 for finite fp32)
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float* t = v + 4 * q;
      const uint16_t lo = FMT == 0 ? cvt2_e4m3(t[0] * inv, t[1] * inv) : cvt2_e5m2(t[0] * inv, t[1] * inv);
      const uint16_t hi = FMT == 0 ? cvt2_e4m3(t[2] * inv, t[3] * inv) : cvt2_e5m2(t[2] * inv, t[3] * inv);
      w[q] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(codes + (int64_t)r * K + (int64_t)j * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    sf[so] = finite ? (uint8_t)(X + 127) : (uint8_t)255;
  }
}

// MXFP8 of a [R, C] bf16 tensor row-wise (32-blocks along C: the operand that
// contracts over C) and column-wise (its transpose, 32-blocks along R), over
// 128 x 128 tiles.  A tile is exactly one 512-byte scale atom of each output
// (128 rows x 4 K-blocks), assembled in shared memory and stored whole; padding
// rows / columns read as zero (cp.async zero fill) and get the scale byte 127, so
// no fill of the scale tensors is needed.  Persistent CTAs walk the tiles with two
// shared-memory tile buffers: the cp.async copy of the next tile is in flight
// while the current one is quantised, which hides the load latency that a
// load-then-compute CTA exposes.  Codes go from registers straight to global
// memory as whole 32-byte sectors (a row block of 32 codes, or a column block of
// 32 codes of the transpose).
// SRC picks what is quantised: 0 the tile as loaded; 1 (LN) its LayerNorm,
// bf16((x - mean[r]) * rstd[r] * gamma[c] + beta[c]) (the MXFP8 input of the QKV /
// FFN1 GEMMs straight from the residual stream); 2 (GELU) bf16(GELU(x)) (the FFN2
// GEMM's input from the FFN1 pre-activation); 3 (dGELU) bf16(x * GELU'(aux[r, c]))
// (the FFN1 GEMMs' output gradient from the FFN2 dgrad and the pre-activation).  The
// transform runs in shared memory after the tile lands.  colsum (optional):
// colsum[c] += sum over r of the tile's (transformed) values (one atomic per column
// per tile).
constexpr int kRcTileStride = 128 + 8;  // bf16 elements per staged row (16-byte rows, bank spread)
constexpr int kRcTileBytes = 128 * kRcTileStride * 2;
// dynamic shared memory: two bf16 tiles | two scale atoms | fp32 column sums [4][128]
constexpr int kRcOffSfr = 2 * kRcTileBytes;
constexpr int kRcOffSfc = kRcOffSfr + 512;
constexpr int kRcOffCsum = kRcOffSfc + 512;
constexpr int kRcSmem = kRcOffCsum + 4 * 128 * (int)sizeof(float);
constexpr int kRcCtasPerSm = 3;
static_assert(kRcTileBytes % 16 == 0 && kRcOffSfr % 16 == 0 && kRcOffSfc % 16 == 0 && kRcOffCsum % 16 == 0,
              "mx_rc_tile_kernel: 16-byte aligned shared-memory regions");
static_assert(kRcCtasPerSm * (kRcSmem + 1024) <= 233472, "mx_rc_tile_kernel: CTAs per SM must fit in shared memory");

// 16-byte cp.async global -> shared; src_bytes 0 zero-fills the destination
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, int src_bytes) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int SRC>
__global__ void __launch_bounds__(256, kRcCtasPerSm) mx_rc_tile_kernel(
    const bf16* __restrict__ x, int64_t ldx, int R, int C, int fmt, uint32_t fmax_bits,
    const float* __restrict__ mean, const float* __restrict__ rstd, const float* __restrict__ gamma,
    const float* __restrict__ beta, float* __restrict__ colsum, uint8_t* __restrict__ rc, uint8_t* __restrict__ rsf,
    uint8_t* __restrict__ cc, uint8_t* __restrict__ csf, const float* __restrict__ xq, int64_t ldq, int qcols,
    const bf16* __restrict__ aux, int64_t ldaux) {
  // xq (optional): columns [0, qcols) of the tensor come from this fp32 matrix instead of x
  // (rounded to bf16 on load; qcols a multiple of 128), e.g. the attention's dQ accumulator
  // beside the dK / dV it wrote into x
  extern __shared__ __align__(16) uint8_t rc_smem[];
  uint8_t* sfr = rc_smem + kRcOffSfr;
  uint8_t* sfc = rc_smem + kRcOffSfc;
  float* csum = reinterpret_cast<float*>(rc_smem + kRcOffCsum);  // [4][128]
  const int t = threadIdx.x;
  const int ntc = (C + 127) / 128, ntr = (R + 127) / 128;
  const int ntiles = ntc * ntr;
  const int ef = (int)((fmax_bits >> 23) & 0xFF);
  const uint32_t mf = fmax_bits & 0x7FFFFF;
  // this thread's eight 16-byte pieces of a tile: row i >> 4, columns (i & 15) * 8 .. + 8
  auto issue = [&](int tile, int buf) {
    bf16(*tl)[kRcTileStride] = reinterpret_cast<bf16(*)[kRcTileStride]>(rc_smem + buf * kRcTileBytes);
    const int r0 = (tile / ntc) * 128, c0 = (tile % ntc) * 128;
    if (xq && c0 < qcols) return;  // an fp32 tile: converted when it is processed
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = t + k * 256, rr = i >> 4, cv = (i & 15) * 8;
      const int r = r0 + rr, c = c0 + cv;
      const bool ok = r < R && c < C;
      cp_async16_zfill(&tl[rr][cv], ok ? (const void*)(x + (int64_t)r * ldx + c) : (const void*)x, ok ? 16 : 0);
    }
  };
  int tile = blockIdx.x;
  if (tile < ntiles) issue(tile, 0);
  cp_async_commit_group();
  for (int it = 0; tile < ntiles; tile += gridDim.x, ++it) {
    const int buf = it & 1;
    // prefetch the next tile into the other buffer (read by the previous iteration,
    // which every thread finished before its closing barrier)
    if (tile + (int)gridDim.x < ntiles) issue(tile + gridDim.x, buf ^ 1);
    cp_async_commit_group();
    cp_async_wait_one();
    __syncthreads();
    bf16(*tl)[kRcTileStride] = reinterpret_cast<bf16(*)[kRcTileStride]>(rc_smem + buf * kRcTileBytes);
    const int rt = tile / ntc, ct = tile % ntc;
    const int r0 = rt * 128, c0 = ct * 128;
    if (xq && c0 < qcols) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = t + k * 256, rr = i >> 4, cv = (i & 15) * 8;
        const int r = r0 + rr;
        float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (r < R) {
          const float4 a = *reinterpret_cast<const float4*>(xq + (int64_t)r * ldq + c0 + cv);
          const float4 b = *reinterpret_cast<const float4*>(xq + (int64_t)r * ldq + c0 + cv + 4);
          f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
        }
        *reinterpret_cast<bf16x8*>(&tl[rr][cv]) = pack8(f);
      }
      __syncthreads();
    }
    if constexpr (SRC == 1) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = t + k * 256, rr = i >> 4, cv = (i & 15) * 8;
        const int r = r0 + rr, c = c0 + cv;
        if (r < R && c < C) {
          float f[8];
          unpack8(*reinterpret_cast<const bf16x8*>(&tl[rr][cv]), f);
          const float mu = mean[r], rs = rstd[r];
          const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
          const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
          const float4 b0 = *reinterpret_cast<const float4*>(beta + c);
          const float4 b1 = *reinterpret_cast<const float4*>(beta + c + 4);
          const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
          const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) f[q] = (f[q] - mu) * rs * g[q] + b[q];
          *reinterpret_cast<bf16x8*>(&tl[rr][cv]) = pack8(f);
        }
      }
      __syncthreads();
    }
    if constexpr (SRC == 2 || SRC == 3) {
      // two pieces per step: their aux loads (dGELU) are in flight together, and the
      // register limit of three CTAs per SM holds no more
#pragma unroll 2
      for (int k = 0; k < 8; ++k) {
        const int i = t + k * 256, rr = i >> 4, cv = (i & 15) * 8;
        const int r = r0 + rr, c = c0 + cv;
        if (r < R && c < C) {
          float f[8];
          if constexpr (SRC == 2) {
            unpack8(*reinterpret_cast<const bf16x8*>(&tl[rr][cv]), f);
#pragma unroll
            for (int q = 0; q < 8; ++q) f[q] = gelu_fwd(f[q]);
          } else {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(aux + (int64_t)r * ldaux + c));
            float a[8];
            unpack8(*reinterpret_cast<const bf16x8*>(&u), a);
            unpack8(*reinterpret_cast<const bf16x8*>(&tl[rr][cv]), f);
#pragma unroll
            for (int q = 0; q < 8; ++q) f[q] *= gelu_grad(a[q]);
          }
          *reinterpret_cast<bf16x8*>(&tl[rr][cv]) = pack8(f);
        }
      }
      __syncthreads();
    }
    float v[32];
    uint32_t w[8];
    uint8_t sfb;
    // row-wise: row t & 127, K-blocks 2 * (t >> 7) and 2 * (t >> 7) + 1 (64 codes)
    {
      const int row = t & 127, half = t >> 7;
      const bool rok = r0 + row < R;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const int blk = 2 * half + b;
#pragma unroll
        for (int q = 0; q < 4; ++q) unpack8(*reinterpret_cast<const bf16x8*>(&tl[row][blk * 32 + 8 * q]), v + 8 * q);
        mx_block(v, ef, mf, fmt, w, sfb);
        if (rok && c0 + blk * 32 < C) {
          uint4* dst = reinterpret_cast<uint4*>(rc + (int64_t)(r0 + row) * C + c0 + blk * 32);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
        sfr[(row & 31) * 16 + (row >> 5) * 4 + blk] = sfb;
      }
    }
    // column-wise: columns 2 (t & 63), 2 (t & 63) + 1, K-block (rows) t >> 6; 32-bit loads
    {
      const int cp = t & 63, blk = t >> 6;
      float v1[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const __nv_bfloat162 pr = *reinterpret_cast<const __nv_bfloat162*>(&tl[blk * 32 + i][2 * cp]);
        v[i] = __low2float(pr);
        v1[i] = __high2float(pr);
      }
      if (colsum) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s0 += v[i];
          s1 += v1[i];
        }
        csum[blk * 128 + 2 * cp] = s0;
        csum[blk * 128 + 2 * cp + 1] = s1;
      }
      const bool kok = r0 + blk * 32 < R;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = 2 * cp + e;
        mx_block(e ? v1 : v, ef, mf, fmt, w, sfb);
        if (kok && c0 + col < C) {
          uint4* dst = reinterpret_cast<uint4*>(cc + (int64_t)(c0 + col) * R + r0 + blk * 32);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
        sfc[(col & 31) * 16 + (col >> 5) * 4 + blk] = sfb;
      }
    }
    __syncthreads();  // scale atoms and column sums complete; the tile buffer is free
    if (t < 32) {
      reinterpret_cast<uint4*>(rsf + ((int64_t)rt * ntc + ct) * 512)[t] = reinterpret_cast<const uint4*>(sfr)[t];
    } else if (t < 64) {
      reinterpret_cast<uint4*>(csf + ((int64_t)ct * ntr + rt) * 512)[t - 32] =
          reinterpret_cast<const uint4*>(sfc)[t - 32];
    }
    if (colsum && t >= 128 && c0 + (t - 128) < C) {
      const int c = t - 128;
      atomicAdd(colsum + c0 + c, (csum[c] + csum[128 + c]) + (csum[256 + c] + csum[384 + c]));
    }
    // the next iteration's first barrier orders these reads before sfr / sfc / csum are rewritten
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

static int q_grid(size_t n, int per) {
  return (int)std::max<size_t>(1, std::min<size_t>((n / per + 255) / 256, (size_t)num_sms() * 8));
}

void fp8_quantize(const at::Tensor& x, at::Tensor out, const c10::optional<at::Tensor>& scale,
                  const c10::optional<at::Tensor>& amax, int64_t fmt) {
  MT_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "fp8_quantize: contiguous bf16 input");
  MT_CHECK(out.element_size() == 1 && out.is_contiguous() && out.numel() == x.numel(), "fp8_quantize: out");
  MT_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "fp8_quantize: 16-byte aligned buffers");
  const size_t n = x.numel();
  if (n == 0) return;
  const float* sp = scale.has_value() ? scale->data_ptr<float>() : nullptr;
  float* ap = amax.has_value() ? amax->data_ptr<float>() : nullptr;
  const auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* op = reinterpret_cast<uint8_t*>(out.data_ptr());
  if (fmt == 0)
    fp8_quantize_kernel<0><<<q_grid(n, 16), 256, 0, cur_stream()>>>(xp, op, sp, ap, n);
  else
    fp8_quantize_kernel<1><<<q_grid(n, 16), 256, 0, cur_stream()>>>(xp, op, sp, ap, n);
  MT_LAUNCH_CHECK();
}

// Quantise with the fused amax all-reduce: see fp8_quantize_ar_kernel.
void fp8_quantize_ar(const at::Tensor& x, at::Tensor out, const at::Tensor& scale, at::Tensor amax,
                     at::Tensor counter, const std::vector<int64_t>& table_ptrs, int64_t me, int64_t cap,
                     int64_t slot, int64_t parity, int64_t epoch, int64_t fmt, int64_t ep_ptr) {
  MT_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "fp8_quantize_ar: contiguous bf16 input");
  MT_CHECK(out.element_size() == 1 && out.is_contiguous() && out.numel() == x.numel(), "fp8_quantize_ar: out");
  MT_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "fp8_quantize_ar: 16-byte aligned buffers");
  MT_CHECK(counter.scalar_type() == at::kInt && counter.numel() >= 1, "fp8_quantize_ar: int32 counter");
  const int world = (int)table_ptrs.size();
  MT_CHECK(world >= 1 && world <= kAmaxMaxPeers, "fp8_quantize_ar: 1..8 ranks");
  AmaxPeers t{};
  for (int i = 0; i < world; ++i) t.p[i] = (uint64_t)table_ptrs[i];
  t.ep = reinterpret_cast<const unsigned int*>(ep_ptr);
  const size_t n = x.numel();
  if (n == 0) return;
  const auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* op = reinterpret_cast<uint8_t*>(out.data_ptr());
  auto* cp = reinterpret_cast<unsigned int*>(counter.data_ptr());
  if (fmt == 0)
    fp8_quantize_ar_kernel<0><<<q_grid(n, 16), 256, 0, cur_stream()>>>(
        xp, op, scale.data_ptr<float>(), amax.data_ptr<float>(), n, cp, t, (int)me, world, (int)cap, (int)slot,
        (int)parity, (unsigned int)epoch);
  else
    fp8_quantize_ar_kernel<1><<<q_grid(n, 16), 256, 0, cur_stream()>>>(
        xp, op, scale.data_ptr<float>(), amax.data_ptr<float>(), n, cp, t, (int)me, world, (int)cap, (int)slot,
        (int)parity, (unsigned int)epoch);
  MT_LAUNCH_CHECK();
}

// Quantise a 2-D bf16 gradient and (+)= its column sums into `colsum` (fp32 [F]).
// table_ptrs empty: local amax only; otherwise the fused amax all-reduce.
void fp8_quantize_colsum(const at::Tensor& x, at::Tensor out, const at::Tensor& scale, at::Tensor amax,
                         at::Tensor colsum, bool accumulate, const c10::optional<at::Tensor>& counter,
                         const std::vector<int64_t>& table_ptrs, int64_t me, int64_t cap, int64_t slot,
                         int64_t parity, int64_t epoch, int64_t fmt, int64_t ep_ptr) {
  MT_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() >= 1, "fp8_quantize_colsum: bf16 x");
  const int F = x.size(-1);
  const int rows = x.numel() / std::max(F, 1);
  MT_CHECK(F % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "fp8_quantize_colsum: F % 8 == 0 and 16-byte aligned buffers");
  MT_CHECK(out.element_size() == 1 && out.numel() == x.numel() && out.is_contiguous(), "fp8_quantize_colsum: out");
  MT_CHECK(colsum.scalar_type() == at::kFloat && colsum.numel() == F && colsum.is_contiguous(),
           "fp8_quantize_colsum: fp32 colsum [F]");
  if (!accumulate) colsum.zero_();
  if (rows == 0) return;
  const int world = (int)table_ptrs.size();
  MT_CHECK(world <= kAmaxMaxPeers && (world == 0 || counter.has_value()), "fp8_quantize_colsum: peers");
  AmaxPeers t{};
  for (int i = 0; i < world; ++i) t.p[i] = (uint64_t)table_ptrs[i];
  t.ep = reinterpret_cast<const unsigned int*>(ep_ptr);
  unsigned int* cp = world ? reinterpret_cast<unsigned int*>(counter->data_ptr()) : nullptr;
  const int col_blocks = (F + 255) / 256;
  int row_blocks = std::max(1, std::min((rows + 63) / 64, (num_sms() * 8 + col_blocks - 1) / col_blocks));
  const int rpb = (rows + row_blocks - 1) / row_blocks;
  row_blocks = (rows + rpb - 1) / rpb;
  const dim3 grid(col_blocks, row_blocks);
  const auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* op = reinterpret_cast<uint8_t*>(out.data_ptr());
  if (fmt == 0)
    fp8_quantize_colsum_kernel<0><<<grid, 256, 0, cur_stream()>>>(
        xp, op, scale.data_ptr<float>(), amax.data_ptr<float>(), colsum.data_ptr<float>(), rows, F, rpb, cp, t,
        (int)me, world, (int)cap, (int)slot, (int)parity, (unsigned int)epoch);
  else
    fp8_quantize_colsum_kernel<1><<<grid, 256, 0, cur_stream()>>>(
        xp, op, scale.data_ptr<float>(), amax.data_ptr<float>(), colsum.data_ptr<float>(), rows, F, rpb, cp, t,
        (int)me, world, (int)cap, (int)slot, (int)parity, (unsigned int)epoch);
  MT_LAUNCH_CHECK();
}

void fp8_amax_gather(const at::Tensor& table, at::Tensor amax, int64_t world, int64_t cap, int64_t parity,
                     int64_t epoch, int64_t ep_ptr) {
  const int slots = amax.numel();
  if (slots == 0) return;
  MT_CHECK(table.element_size() == 8 && table.numel() >= 2 * world * cap, "fp8_amax_gather: table");
  fp8_amax_gather_kernel<<<(slots + 127) / 128, 128, 0, cur_stream()>>>(
      reinterpret_cast<const unsigned long long*>(table.data_ptr()), amax.data_ptr<float>(), slots, (int)world,
      (int)cap, (int)parity, (unsigned int)epoch, reinterpret_cast<const unsigned int*>(ep_ptr));
  MT_LAUNCH_CHECK();
}

// Store amax[s] (this rank's running amax of slot s, s < slots) into every peer's
// table with this step's stamp: the publication for roles whose FP8 codes come
// from a producer that does not publish itself (a GEMM epilogue writing codes).
__global__ void fp8_amax_publish_kernel(const float* __restrict__ amax, AmaxPeers table, int me, int world, int cap,
                                        int slots, int parity, unsigned int epoch) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= slots) return;
  if (table.ep) {
    epoch += *table.ep;
    parity = (int)(epoch & 1u);
  }
  const unsigned long long v = ((unsigned long long)epoch << 32) | __float_as_uint(amax[s]);
  for (int r = 0; r < world; ++r) {
    unsigned long long* t = reinterpret_cast<unsigned long long*>(table.p[r]) + ((size_t)parity * world + me) * cap + s;
    *reinterpret_cast<volatile unsigned long long*>(t) = v;
  }
  __threadfence_system();
}

void fp8_amax_publish(const at::Tensor& amax, const std::vector<int64_t>& table_ptrs, int64_t me, int64_t cap,
                      int64_t parity, int64_t epoch, int64_t ep_ptr) {
  const int slots = amax.numel();
  const int world = (int)table_ptrs.size();
  MT_CHECK(world >= 1 && world <= kAmaxMaxPeers && slots <= cap, "fp8_amax_publish: 1..8 ranks, slots <= cap");
  MT_CHECK(amax.scalar_type() == at::kFloat && amax.is_contiguous(), "fp8_amax_publish: fp32 amax");
  if (slots == 0) return;
  AmaxPeers t{};
  for (int i = 0; i < world; ++i) t.p[i] = (uint64_t)table_ptrs[i];
  t.ep = reinterpret_cast<const unsigned int*>(ep_ptr);
  fp8_amax_publish_kernel<<<(slots + 127) / 128, 128, 0, cur_stream()>>>(amax.data_ptr<float>(), t, (int)me, world,
                                                                          (int)cap, slots, (int)parity,
                                                                          (unsigned int)epoch);
  MT_LAUNCH_CHECK();
}

void fp8_amax(const at::Tensor& x, at::Tensor amax) {
  MT_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "fp8_amax: contiguous bf16");
  const size_t n = x.numel();
  if (n == 0) return;
  amax_kernel<<<q_grid(n, 8), 256, 0, cur_stream()>>>(reinterpret_cast<const bf16*>(x.data_ptr()),
                                                      amax.data_ptr<float>(), n);
  MT_LAUNCH_CHECK();
}

__global__ void fp8_cursor_advance_kernel(int* cursor, int H) { *cursor = (*cursor + 1) % H; }

// cursor_dev (int32 [1], optional): read the ring position from the device and
// advance it there, so a captured step replays correctly.
void fp8_scaling_update(at::Tensor hist, at::Tensor amax, at::Tensor scale, at::Tensor inv,
                        const at::Tensor& fmax, int64_t cursor, bool current,
                        const c10::optional<at::Tensor>& cursor_dev) {
  const int slots = amax.numel();
  const int H = hist.numel() / std::max(slots, 1);
  if (slots == 0) return;
  const int* cd = cursor_dev.has_value() ? cursor_dev->data_ptr<int>() : nullptr;
  fp8_scaling_update_kernel<<<(slots + 127) / 128, 128, 0, cur_stream()>>>(
      hist.data_ptr<float>(), amax.data_ptr<float>(), scale.data_ptr<float>(), inv.data_ptr<float>(),
      fmax.data_ptr<float>(), slots, H, (int)cursor, current ? 1 : 0, cd);
  MT_LAUNCH_CHECK();
  if (cd && !current) {
    fp8_cursor_advance_kernel<<<1, 1, 0, cur_stream()>>>(cursor_dev->data_ptr<int>(), H);
    MT_LAUNCH_CHECK();
  }
}

void fp8_dequantize(const at::Tensor& q, at::Tensor out, const at::Tensor& inv_scale, int64_t fmt) {
  const size_t n = q.numel();
  if (n == 0) return;
  if (fmt == 0)
    fp8_dequantize_kernel<0><<<q_grid(n, 1), 256, 0, cur_stream()>>>(
        reinterpret_cast<const uint8_t*>(q.data_ptr()), out.data_ptr<float>(),
        inv_scale.data_ptr<float>(), n);
  else
    fp8_dequantize_kernel<1><<<q_grid(n, 1), 256, 0, cur_stream()>>>(
        reinterpret_cast<const uint8_t*>(q.data_ptr()), out.data_ptr<float>(),
        inv_scale.data_ptr<float>(), n);
  MT_LAUNCH_CHECK();
}

// x: bf16 [R, K] (unit inner stride, 16-byte aligned rows), codes: uint8 [R, K]
// contiguous, sf: uint8 [ceil(R/128) * ceil(K/128) * 512]; fmax = the format maximum
// the block amax is scaled to.
void mx_quantize(const at::Tensor& x, at::Tensor codes, at::Tensor sf, int64_t fmt, double fmax) {
  MT_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "mx_quantize: 2-D bf16 input");
  const int64_t R = x.size(0), K = x.size(1);
  MT_CHECK(K % 32 == 0, "mx_quantize: K must be a multiple of 32");
  MT_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && (x.stride(0) * 2) % 16 == 0,
           "mx_quantize: 16-byte aligned rows");
  MT_CHECK(codes.element_size() == 1 && codes.is_contiguous() && codes.numel() == R * K &&
               reinterpret_cast<uintptr_t>(codes.data_ptr()) % 16 == 0,
           "mx_quantize: codes must be 16-byte aligned contiguous uint8 [R, K]");
  const int64_t nkb4 = (K + 127) / 128;
  MT_CHECK(sf.element_size() == 1 && sf.is_contiguous() && sf.numel() == (R + 127) / 128 * nkb4 * 512,
           "mx_quantize: sf must be contiguous uint8 of ceil(R/128) * ceil(K/128) * 512 bytes");
  MT_CHECK(fmt == 0 || fmt == 1, "mx_quantize: fmt 0 (E4M3) or 1 (E5M2)");
  MT_CHECK(fmax > 0.0, "mx_quantize: fmax > 0");
  if (R == 0 || K == 0) return;
  const float fm = (float)fmax;
  uint32_t fbits;
  std::memcpy(&fbits, &fm, 4);
  const int64_t total = (R + 127) / 128 * 128 * nkb4 * 4;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16));
  const auto* xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto* cp = reinterpret_cast<uint8_t*>(codes.data_ptr());
  auto* sp = reinterpret_cast<uint8_t*>(sf.data_ptr());
  if (fmt == 0)
    mx_quantize_kernel<0><<<grid, 256, 0, cur_stream()>>>(xp, x.stride(0), cp, sp, (int)R, (int)K, (int)nkb4, fbits);
  else
    mx_quantize_kernel<1><<<grid, 256, 0, cur_stream()>>>(xp, x.stride(0), cp, sp, (int)R, (int)K, (int)nkb4, fbits);
  MT_LAUNCH_CHECK();
}

// x: bf16 [R, C] (R, C multiples of 32, 16-byte aligned rows) -> row codes [R, C] + rsf
// (scales of [R, C]) and column codes [C, R] + csf (scales of [C, R]).
// Launches mx_rc_tile_kernel over [R, C] (see there); ln_* non-null: LayerNorm on load.
void mx_rc_tiles(const bf16* x, int64_t ldx, int64_t R, int64_t C, int64_t fmt, double fmax, const float* ln_mean,
                 const float* ln_rstd, const float* ln_gamma, const float* ln_beta, float* colsum, uint8_t* rc,
                 uint8_t* rsf, uint8_t* cc, uint8_t* csf, cudaStream_t st, const float* xq, int64_t ldq,
                 int64_t qcols, int act, const bf16* aux, int64_t ldaux) {
  const float fm = (float)fmax;
  uint32_t fbits;
  std::memcpy(&fbits, &fm, 4);
  const int64_t tiles = ((C + 127) / 128) * ((R + 127) / 128);
  const int grid = (int)std::min<int64_t>(tiles, (int64_t)num_sms() * kRcCtasPerSm);
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(mx_rc_tile_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRcSmem));
    C10_CUDA_CHECK(cudaFuncSetAttribute(mx_rc_tile_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRcSmem));
    C10_CUDA_CHECK(cudaFuncSetAttribute(mx_rc_tile_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRcSmem));
    C10_CUDA_CHECK(cudaFuncSetAttribute(mx_rc_tile_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRcSmem));
    attr = true;
  }
  if (ln_mean)
    mx_rc_tile_kernel<1><<<grid, 256, kRcSmem, st>>>(x, ldx, (int)R, (int)C, (int)fmt, fbits, ln_mean, ln_rstd,
                                                ln_gamma, ln_beta, colsum, rc, rsf, cc, csf, nullptr, 0, 0, nullptr, 0);
  else if (act == 2)
    mx_rc_tile_kernel<2><<<grid, 256, kRcSmem, st>>>(x, ldx, (int)R, (int)C, (int)fmt, fbits, nullptr, nullptr,
                                                nullptr, nullptr, colsum, rc, rsf, cc, csf, nullptr, 0, 0, nullptr, 0);
  else if (act == 3)
    mx_rc_tile_kernel<3><<<grid, 256, kRcSmem, st>>>(x, ldx, (int)R, (int)C, (int)fmt, fbits, nullptr, nullptr,
                                                nullptr, nullptr, colsum, rc, rsf, cc, csf, nullptr, 0, 0, aux, ldaux);
  else
    mx_rc_tile_kernel<0><<<grid, 256, kRcSmem, st>>>(x, ldx, (int)R, (int)C, (int)fmt, fbits, nullptr, nullptr,
                                                nullptr, nullptr, colsum, rc, rsf, cc, csf, xq, ldq, (int)qcols,
                                                nullptr, 0);
  MT_LAUNCH_CHECK();
}

// colsum (optional fp32 [C]): += the column sums of x (the bias gradient of the layer
// whose output gradient x is), in the same pass.  xq (optional fp32 [R, Q], Q a multiple
// of 128): columns [0, Q) of the tensor are taken from xq (rounded to bf16) instead of x.
void mx_quantize_rc(const at::Tensor& x, at::Tensor rc, at::Tensor rsf, at::Tensor cc, at::Tensor csf, int64_t fmt,
                    double fmax, const c10::optional<at::Tensor>& colsum, const c10::optional<at::Tensor>& xq,
                    int64_t act, const c10::optional<at::Tensor>& aux) {
  MT_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "mx_quantize_rc: 2-D bf16 input");
  const int64_t R = x.size(0), C = x.size(1);
  MT_CHECK(R % 32 == 0 && C % 32 == 0, "mx_quantize_rc: R and C must be multiples of 32");
  MT_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && (x.stride(0) * 2) % 16 == 0,
           "mx_quantize_rc: 16-byte aligned rows");
  auto chk = [](const at::Tensor& t, int64_t n, const char* what) {
    MT_CHECK(t.element_size() == 1 && t.is_contiguous() && t.numel() == n &&
                 reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
             what);
  };
  chk(rc, R * C, "mx_quantize_rc: rc must be 16-byte aligned contiguous uint8 [R, C]");
  chk(cc, R * C, "mx_quantize_rc: cc must be 16-byte aligned contiguous uint8 [C, R]");
  chk(rsf, (R + 127) / 128 * ((C + 127) / 128) * 512, "mx_quantize_rc: rsf size");
  chk(csf, (C + 127) / 128 * ((R + 127) / 128) * 512, "mx_quantize_rc: csf size");
  MT_CHECK((fmt == 0 || fmt == 1) && fmax > 0.0, "mx_quantize_rc: fmt 0 / 1, fmax > 0");
  if (colsum.has_value())
    MT_CHECK(colsum->scalar_type() == at::kFloat && colsum->is_contiguous() && colsum->numel() == C,
             "mx_quantize_rc: colsum must be fp32 [C]");
  const float* xqp = nullptr;
  int64_t ldq = 0, qcols = 0;
  if (xq.has_value()) {
    MT_CHECK(xq->scalar_type() == at::kFloat && xq->dim() == 2 && xq->size(0) == R && xq->stride(1) == 1 &&
                 xq->size(1) % 128 == 0 && xq->size(1) <= C && xq->stride(0) % 4 == 0 &&
                 reinterpret_cast<uintptr_t>(xq->data_ptr()) % 16 == 0,
             "mx_quantize_rc: xq must be fp32 [R, Q] with Q a multiple of 128, 16-byte aligned rows");
    xqp = xq->data_ptr<float>();
    ldq = xq->stride(0);
    qcols = xq->size(1);
  }
  MT_CHECK(act == 0 || act == 2 || act == 3, "mx_quantize_rc: act 0 (none), 2 (GELU) or 3 (dGELU)");
  MT_CHECK(act == 0 || !xq.has_value(), "mx_quantize_rc: xq takes no activation");
  const bf16* auxp = nullptr;
  int64_t ldaux = 0;
  if (act == 3) {
    MT_CHECK(aux.has_value() && aux->scalar_type() == at::kBFloat16 && aux->dim() == 2 && aux->size(0) == R &&
                 aux->size(1) == C && aux->stride(1) == 1 && (aux->stride(0) * 2) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(aux->data_ptr()) % 16 == 0,
             "mx_quantize_rc: dGELU needs aux bf16 [R, C] with 16-byte aligned rows");
    auxp = reinterpret_cast<const bf16*>(aux->data_ptr());
    ldaux = aux->stride(0);
  }
  if (R == 0 || C == 0) return;
  mx_rc_tiles(reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(0), R, C, fmt, fmax, nullptr, nullptr, nullptr,
              nullptr, colsum.has_value() ? colsum->data_ptr<float>() : nullptr,
              reinterpret_cast<uint8_t*>(rc.data_ptr()), reinterpret_cast<uint8_t*>(rsf.data_ptr()),
              reinterpret_cast<uint8_t*>(cc.data_ptr()), reinterpret_cast<uint8_t*>(csf.data_ptr()), cur_stream(), xqp,
              ldq, qcols, (int)act, auxp, ldaux);
}

void fp8_quantize_blocks(const at::Tensor& x, at::Tensor out, at::Tensor scales, int64_t block_size,
                         double fmax, int64_t fmt) {
  MT_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous(), "fp8_quantize_blocks: contiguous fp32");
  const size_t n = x.numel();
  const size_t nb = (n + block_size - 1) / block_size;
  if (n == 0) return;
  const int threads = 256;
  const int grid = (int)((nb * 32 + threads - 1) / threads);
  if (fmt == 0)
    fp8_quantize_blocks_kernel<0><<<grid, threads, 0, cur_stream()>>>(
        x.data_ptr<float>(), reinterpret_cast<uint8_t*>(out.data_ptr()), scales.data_ptr<float>(), n,
        (int)block_size, (float)fmax, nb);
  else
    fp8_quantize_blocks_kernel<1><<<grid, threads, 0, cur_stream()>>>(
        x.data_ptr<float>(), reinterpret_cast<uint8_t*>(out.data_ptr()), scales.data_ptr<float>(), n,
        (int)block_size, (float)fmax, nb);
  MT_LAUNCH_CHECK();
}


// ------------------------------------------------------------------ FP8 wire codec
// Compressed transfer format for pipeline-stage activations and gradients: FP8
// codes (E4M3 or E5M2) with one power-of-two scale per 32 consecutive values (the
// MX block rule of mx.cuh, so no value saturates and a NaN / Inf block carries the
// NaN scale), flat layout: codes[numel] then scales[ceil(numel / 32)].  1.03 bytes
// per value instead of 2 (bf16) or 4 (fp32).  One thread per 32-value block; the
// last block is zero-padded.
__device__ __forceinline__ void wire_dec2(uint16_t c, int fmt, float& a, float& b) {
  uint32_t h;
  if (fmt == 0)
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(c));
  else
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h) : "h"(c));
  const __half2 hh = *reinterpret_cast<__half2*>(&h);
  a = __low2float(hh);
  b = __high2float(hh);
}

template <typename T>
__global__ void __launch_bounds__(256) wire_encode_kernel(const T* __restrict__ x, uint8_t* __restrict__ codes,
                                                          uint8_t* __restrict__ sf, int64_t numel, int fmt,
                                                          uint32_t fmax_bits) {
  const int ef = (int)((fmax_bits >> 23) & 0xFF);
  const uint32_t mf = fmax_bits & 0x7FFFFF;
  const int64_t nb = (numel + 31) / 32;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
    float v[32];
    const int64_t e0 = b * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = e0 + i < numel ? to_f(x[e0 + i]) : 0.f;
    uint32_t w[8];
    uint8_t sfb;
    mx_block(v, ef, mf, fmt, w, sfb);
    if (e0 + 32 <= numel && (reinterpret_cast<uintptr_t>(codes + e0) & 15) == 0) {
      uint4* dst = reinterpret_cast<uint4*>(codes + e0);
      dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
      for (int i = 0; i < 32 && e0 + i < numel; ++i) codes[e0 + i] = (uint8_t)(w[i >> 2] >> ((i & 3) * 8));
    }
    sf[b] = sfb;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) wire_decode_kernel(const uint8_t* __restrict__ codes,
                                                          const uint8_t* __restrict__ sf, T* __restrict__ out,
                                                          int64_t numel, int fmt) {
  const int64_t nb = (numel + 31) / 32;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t s = sf[b];
    const float scale = s == 255u ? __uint_as_float(0x7FC00000u)
                                  : (s == 0u ? __uint_as_float(0x00400000u) : __uint_as_float(s << 23));
    const int64_t e0 = b * 32;
    for (int i = 0; i < 32 && e0 + i < numel; i += 2) {
      const uint16_t c = (uint16_t)codes[e0 + i] | (e0 + i + 1 < numel ? (uint16_t)codes[e0 + i + 1] << 8 : 0);
      float a, bb;
      wire_dec2(c, fmt, a, bb);
      out[e0 + i] = from_f<T>(a * scale);
      if (e0 + i + 1 < numel) out[e0 + i + 1] = from_f<T>(bb * scale);
    }
  }
}

// x: bf16 or fp32, contiguous; codes: uint8 [numel]; sf: uint8 [ceil(numel / 32)].
void fp8_wire_encode(const at::Tensor& x, at::Tensor codes, at::Tensor sf, int64_t fmt) {
  MT_CHECK(x.is_contiguous() && codes.is_contiguous() && sf.is_contiguous(), "wire_encode: contiguous tensors");
  const int64_t n = x.numel();
  MT_CHECK(codes.numel() >= n && sf.numel() >= (n + 31) / 32, "wire_encode: output sizes");
  if (n == 0) return;
  const float fmax = fmt == 0 ? 448.f : 57344.f;
  uint32_t bits;
  std::memcpy(&bits, &fmax, 4);
  const int64_t nb = (n + 31) / 32;
  const int grid = (int)std::min<int64_t>((nb + 255) / 256, 148 * 16);
  auto* c = reinterpret_cast<uint8_t*>(codes.data_ptr());
  auto* f = reinterpret_cast<uint8_t*>(sf.data_ptr());
  if (x.scalar_type() == at::kBFloat16)
    wire_encode_kernel<bf16><<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<const bf16*>(x.data_ptr()), c, f, n,
                                                           (int)fmt, bits);
  else {
    MT_CHECK(x.scalar_type() == at::kFloat, "wire_encode: bf16 or fp32 input");
    wire_encode_kernel<float><<<grid, 256, 0, cur_stream()>>>(x.data_ptr<float>(), c, f, n, (int)fmt, bits);
  }
  MT_LAUNCH_CHECK();
}

void fp8_wire_decode(const at::Tensor& codes, const at::Tensor& sf, at::Tensor out, int64_t fmt) {
  MT_CHECK(out.is_contiguous() && codes.is_contiguous() && sf.is_contiguous(), "wire_decode: contiguous tensors");
  const int64_t n = out.numel();
  if (n == 0) return;
  const int64_t nb = (n + 31) / 32;
  const int grid = (int)std::min<int64_t>((nb + 255) / 256, 148 * 16);
  const auto* c = reinterpret_cast<const uint8_t*>(codes.data_ptr());
  const auto* f = reinterpret_cast<const uint8_t*>(sf.data_ptr());
  if (out.scalar_type() == at::kBFloat16)
    wire_decode_kernel<bf16><<<grid, 256, 0, cur_stream()>>>(c, f, reinterpret_cast<bf16*>(out.data_ptr()), n,
                                                           (int)fmt);
  else {
    MT_CHECK(out.scalar_type() == at::kFloat, "wire_decode: bf16 or fp32 output");
    wire_decode_kernel<float><<<grid, 256, 0, cur_stream()>>>(c, f, out.data_ptr<float>(), n, (int)fmt);
  }
  MT_LAUNCH_CHECK();
}

}  // namespace mtorus
