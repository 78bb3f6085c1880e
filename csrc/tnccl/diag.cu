// diag.cu - diagnostics of the collective library: the bounded-wait self
// test (a kernel that waits on a word nothing writes), mailbox canary
// corruption for the validation test, and the read-out of the device phase
// trace (TNCCL_TRACE=1).
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "comm.h"
#include "device.cuh"
#include "diag.h"

// ---------------------------------------------------------------------------
// Bounded-wait self test: one CTA waits (through the same waitFlag used by
// the collectives) on a device word that nothing ever writes, with the
// caller's bound. The wait must give up, record TNCCL_TIMEOUT in the
// communicator's status block and let the kernel return.
// ---------------------------------------------------------------------------
namespace tnccl {
namespace {

__global__ void diagWaitKernel(const __grid_constant__ DevComm comm, const uint64_t* word) {
  if (threadIdx.x == 0) (void)dev::waitFlag(comm, word, 1, dev::whereCode(15, 0, 9));
}

}  // namespace
}  // namespace tnccl

using namespace tnccl;

extern "C" tncclResult tncclDiagWaitTimeout(tncclComm_t comm, int timeoutMs, cudaStream_t stream) {
  if (comm == nullptr || timeoutMs < 1 || comm->diagWord == nullptr) return TNCCL_INVALID_ARGUMENT;
  DevComm d = comm->dev;
  d.timeoutNs = (uint64_t)timeoutMs * 1000000ull;
  diagWaitKernel<<<1, 32, 0, stream>>>(d, comm->diagWord);
  gLaunchCount.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError() == cudaSuccess ? TNCCL_SUCCESS : TNCCL_CUDA_ERROR;
}

extern "C" int tncclDiagDeviceChecks(void) { return TNCCL_DEVICE_CHECKS ? 1 : 0; }

extern "C" tncclResult tncclDiagCorruptCanary(tncclComm_t comm, int which) {
  if (comm == nullptr || which < 0 || which >= kNumCanaries || comm->local.base == nullptr)
    return TNCCL_INVALID_ARGUMENT;
  if (cudaMemset(comm->local.base + comm->layout.canaryOff[which], 0, 8) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess)
    return TNCCL_CUDA_ERROR;
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclCommTraceRead(tncclComm_t comm, int channel, unsigned long long* out,
                                          size_t maxRecords, size_t* n) {
  if (comm == nullptr || n == nullptr || channel < 0 || channel >= kMaxChannels)
    return TNCCL_INVALID_ARGUMENT;
  *n = 0;
  if (comm->trace == nullptr) return TNCCL_SUCCESS;
  if (cudaDeviceSynchronize() != cudaSuccess) return TNCCL_CUDA_ERROR;
  uint32_t count = 0;
  if (cudaMemcpy(&count, comm->traceCount + channel, sizeof(count), cudaMemcpyDeviceToHost) !=
      cudaSuccess)
    return TNCCL_CUDA_ERROR;
  const uint32_t E = (uint32_t)comm->cfg.traceEvents;
  const uint32_t have = count < E ? count : E;
  std::vector<unsigned long long> ring((size_t)E * 2);
  if (cudaMemcpy(ring.data(), comm->trace + (size_t)channel * E * 2, ring.size() * 8,
                 cudaMemcpyDeviceToHost) != cudaSuccess)
    return TNCCL_CUDA_ERROR;
  const uint32_t first = count < E ? 0 : count % E;
  size_t k = 0;
  for (uint32_t i = 0; i < have && k < maxRecords; ++i, ++k) {
    const uint32_t j = (first + i) % E;
    out[2 * k] = ring[2 * (size_t)j];
    out[2 * k + 1] = ring[2 * (size_t)j + 1];
  }
  *n = k;
  return TNCCL_SUCCESS;
}
