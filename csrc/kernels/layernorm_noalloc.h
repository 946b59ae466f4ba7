// Allocation-free LayerNorm backward: a C entry point for callers that cannot
// allocate device memory.
//
// This entry point has no counterpart in the reference implementation; it is an
// addition of this library.
//
// Who needs it: code that runs where cudaMalloc is not allowed or not safe --
// for example an inference-engine plugin whose enqueue callback must not
// allocate, or a serving process that reserved all of HBM into fixed pools at
// start-up under its own memory planner.  Such a caller passes only its inputs
// and outputs; the kernel's scratch (per-block dgamma/dbeta partial sums) lives
// in a fixed-size array that is part of the loaded library.
//
// Limits and behaviour:
//   * d must be a multiple of 8 and at most MTORUS_LN_NOALLOC_MAX_D (4096);
//     rows must be > 0.  Pointers must be 16-byte aligned.  Other sizes are
//     rejected with MTORUS_NOALLOC_ESIZE / MTORUS_NOALLOC_EARG and nothing runs.
//   * The scratch array holds MTORUS_LN_NOALLOC_MAX_BLOCKS x 2 x 4096 floats
//     (5 MiB).  Every GPU that loads the library keeps it until the process exits.
//   * The first call on a device does the set-up for that device (it looks up
//     the array's device address).  Make that first call before any stream
//     capture.  Every call also raises the shared-memory limit of the kernel it
//     launches (a function attribute, which other code may lower in between).
//   * An error already pending on the calling thread (from earlier, unrelated
//     work) is left in place and reported as MTORUS_NOALLOC_EPENDING; nothing
//     is launched.
//   * All calls share the one array, and it keeps the last call's contents
//     (every call overwrites what it reads).  Calls that overlap on the GPU --
//     on two streams, or from two threads -- race on it; serialise them.
//   * Nothing is allocated or freed: no cudaMalloc / cudaFree, no library
//     allocator.  The work is enqueued on `stream`; the call does not synchronise.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define MTORUS_LN_NOALLOC_MAX_D 4096
#define MTORUS_LN_NOALLOC_MAX_BLOCKS 160

#define MTORUS_NOALLOC_OK 0
#define MTORUS_NOALLOC_EARG -1    // null or misaligned pointer, d % 8 != 0, rows <= 0
#define MTORUS_NOALLOC_ESIZE -2   // d above MTORUS_LN_NOALLOC_MAX_D
#define MTORUS_NOALLOC_ESETUP -3  // device set-up failed (symbol lookup / attribute)
#define MTORUS_NOALLOC_ELAUNCH -4 // kernel launch failed
#define MTORUS_NOALLOC_EPENDING -5 // a CUDA error from earlier work was already pending

#ifdef __cplusplus
extern "C" {
#endif

// dx[rows, d] = LayerNorm backward of dy given x, gamma and the forward's
// per-row mean / rstd.  dgamma[d] / dbeta[d] are overwritten (accumulate == 0)
// or added to (accumulate != 0).  dy, x, dx are bf16 (passed as uint16_t);
// gamma, mean, rstd, dgamma, dbeta are fp32.  Returns MTORUS_NOALLOC_OK or a
// negative code above.
__attribute__((visibility("default"))) int mtorus_layernorm_bwd_noalloc(
    const uint16_t* dy, const uint16_t* x, const float* gamma, const float* mean,
    const float* rstd, uint16_t* dx, float* dgamma, float* dbeta, int rows, int d,
    int accumulate, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
