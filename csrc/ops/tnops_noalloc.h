// tnops_noalloc.h - LayerNorm backward that allocates no device memory.
//
// This entry point has no counterpart in the tiny-nccl reference; it is an
// addition of this library for callers that cannot allocate device memory
// while they run, for example:
//   * a serving or training engine that plans all device memory once at
//     start-up and forbids any allocation afterwards (a fixed arena),
//   * C or C++ code that does not link PyTorch and therefore has no caching
//     allocator to borrow a temporary buffer from,
//   * code called back from inside another runtime, where a cudaMalloc would
//     implicitly synchronize the device or fail.
// For those callers the scratch buffer that tnops_ln_bwd takes as an argument
// (`partial`, the per-CTA column sums of dweight/dbias) is replaced by a
// buffer compiled into libtnccl_ops.so.
#pragma once

#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest row width (C) this entry point accepts. The built-in scratch holds
// 2 * tnops_ln_partial_rows() * TNOPS_NOALLOC_MAX_C floats (about 2.3 MiB);
// every GPU that loads the library keeps that much memory until the process
// exits.
#define TNOPS_NOALLOC_MAX_C 1024

// Same contract and results as tnops_ln_bwd (tnccl_ops.h) without the
// `partial` argument; allocates no device or host memory.
//  * C must be a multiple of 4 and at most TNOPS_NOALLOC_MAX_C; a larger C
//    returns cudaErrorInvalidValue and prints the limit to stderr, without
//    launching anything.
//  * The first call on a device looks up the device address of the built-in
//    scratch for that device (the device must be current). Make that first
//    call before any CUDA stream capture starts. The address is kept for the
//    life of the process's context on that device: after cudaDeviceReset (or
//    anything else that destroys the primary context) do not call this
//    entry point again in the same process.
//  * All calls share one scratch buffer per device, which keeps what the
//    last call wrote. Every element a call reads is written earlier in the
//    same call, so nothing has to be cleared between calls. Calls whose
//    kernels overlap on the GPU (different streams without ordering between
//    them) race on that buffer and give wrong results: order them.
int tnops_ln_bwd_noalloc(const uint16_t* gy, const float* g_res, const float* x_out,
                         const float* w, const float* mean, const float* rstd, float* dx,
                         uint16_t* dx_bf16, float* dw, float* db, int rows, int C,
                         cudaStream_t stream);

#ifdef __cplusplus
}
#endif
