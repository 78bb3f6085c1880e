// launch.h - host entry points into the kernel translation unit.
#pragma once

#include <cuda_runtime_api.h>
#include <stdint.h>

#include "devcomm.h"

namespace tnccl {

// Launches the all-reduce kernel of `algo` (tncclAlgo_t) on stream.
cudaError_t launchAllReduceKernel(const DevComm& comm, const AllReduceArgs& args, int algo,
                                  int threads, cudaStream_t stream);

// Single-rank path: y = alpha * x.
cudaError_t launchScale(const void* x, void* y, uint64_t n, int dtype, float alpha,
                        int vectorized, cudaStream_t stream);

// Cooperative launch of the emulated ranks (grid = channels x nranks).
cudaError_t launchEmulated(const EmulatedLaunch& e, int channels, int threads,
                           cudaStream_t stream);
// CTAs of the emulation kernel that fit on the device at once.
int emulatedMaxCtas(int threads);

}  // namespace tnccl
