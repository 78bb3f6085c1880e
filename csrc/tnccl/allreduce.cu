// allreduce.cu - sm_100a all-reduce kernels and their launcher. The device
// bodies live in kernel_common.cuh (shared loops and helpers), ring.cuh,
// oneshot.cuh, twoshot.cuh and nvls.cuh; this file holds the kernels, the
// single-GPU emulation kernel and the host launchers.
//
// One CTA is one channel; channel c walks tiles c, c + C, ... of the message
// (protocol.h) and keeps its FIFO sequence number in device memory, so every
// launch continues where the previous one on the same communicator stopped.
//
//   ring     tiny-nccl's reduce-scatter + all-gather rotation
//            (src/ring_allreduce.cu:12-54) per channel, with 16-byte vector
//            peer stores, pre-scale, fp32 math and a fused final
//            reduce+store+forward step. Summation order of chunk s:
//            ((a*x[s+1] + a*x[s+2]) + ...) + a*x[s], rounded to the wire
//            type at every hop.
//   one-shot every rank pushes its whole tile into every peer's mailbox and
//            reduces all P contributions locally in rank order 0..P-1.
//   two-shot reduce-scatter by pushing chunk j to rank j, which reduces in
//            rank order 0..P-1, then all-gather by pushing the reduced chunk
//            to every peer; three warp-specialised teams (push, reduce,
//            gather) per CTA run the phases of successive tiles
//            concurrently. Each rank both sends to and receives from every
//            peer in both phases, which doubles as flow control: no credit
//            words are needed (slot-reuse argument in twoshot.cuh).
//   NVLS     teams copy the tile into the multicast-bound buffer, reduce this
//            rank's share in the NVSwitch (multimem.ld_reduce) and broadcast
//            it with multimem.st, and copy the result out; the barriers
//            between them are per-slot counters that every rank increments
//            on every GPU with one multimem.red. For buffers registered with
//            tncclCommRegister a zero-copy variant reduces and broadcasts
//            straight from and into the user's buffers.
//
// Every wait is bounded (device.cuh); a CTA whose wait fails stops, leaves
// its sequence number untouched and the host sees the recorded error.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <utility>

#include <atomic>

#include "device.cuh"
#include "launch.h"
#include "protocol.h"
#include "tnccl.h"
// the device bodies, in dependency order
#include "kernel_common.cuh"
#include "twoshot.cuh"
#include "oneshot.cuh"
#include "ring.cuh"
#include "nvls.cuh"

namespace tnccl {
namespace {

using namespace dev;

// ---------------------------------------------------------------------------
// Single rank: y = alpha * x (identity copy when alpha == 1 is done with
// cudaMemcpyAsync by the host).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kMaxThreads)
    scaleKernel(const T* __restrict__ x, T* y, uint64_t n, float alpha, int vectorized) {
  using Pk = Pack<T>;
  constexpr int V = Pk::V;
  const uint64_t nvec = vectorized ? n / V : 0;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    float f[V];
    Pk::unpack(ldInput(reinterpret_cast<const uint4*>(x) + i), f);
#pragma unroll
    for (int e = 0; e < V; ++e) f[e] = scaled(alpha, f[e]);
    st16(reinterpret_cast<uint4*>(y) + i, Pk::pack(f));
  }
  for (uint64_t e = nvec * V + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += stride)
    stElem(y + e, scaled(alpha, ldElem<T, kLdInput>(x + e)));
}

// ---------------------------------------------------------------------------
// Kernels: one CTA per channel (blockIdx.x).
// ---------------------------------------------------------------------------
template <typename T, int MAXP>
__global__ void __launch_bounds__(kMaxThreads)
    twoShotKernel(const __grid_constant__ DevComm comm, const __grid_constant__ AllReduceArgs a) {
  twoShotBody<T, MAXP>(comm, a, blockIdx.x);
}

template <typename T, int MAXP>
__global__ void __launch_bounds__(kMaxThreads)
    oneShotKernel(const __grid_constant__ DevComm comm, const __grid_constant__ AllReduceArgs a) {
  oneShotBody<T, MAXP>(comm, a, blockIdx.x);
}

// NET: the communicator has socket ring edges (TNCCL_NET), so either edge of
// this rank may be a host-mapped FIFO; the NVLink-only ring is compiled
// without those branches.
template <typename T, bool NET>
__global__ void __launch_bounds__(kMaxThreads)
    ringKernel(const __grid_constant__ DevComm comm, const __grid_constant__ AllReduceArgs a) {
  ringBody<T, NET>(comm, a, blockIdx.x);
}

// Single-GPU emulation of `nranks` ranks: blockIdx.y selects the emulated
// rank, blockIdx.x its channel. All ranks' mailboxes live in this GPU's
// memory. The launch is cooperative, so every CTA is resident and CTAs of
// different emulated ranks can wait on one another.
template <typename T, int MAXP>
__global__ void __launch_bounds__(kMaxThreads)
    emulatedKernel(const __grid_constant__ EmulatedLaunch e) {
  const int r = blockIdx.y;
  switch (e.algo) {
    case TNCCL_ALGO_TWOSHOT:
      twoShotBody<T, MAXP>(e.comm[r], e.args[r], blockIdx.x);
      break;
    case TNCCL_ALGO_ONESHOT:
      oneShotBody<T, MAXP>(e.comm[r], e.args[r], blockIdx.x);
      break;
    default:
      ringBody<T, false>(e.comm[r], e.args[r], blockIdx.x);
      break;
  }
}

// Emulated ranks joined by socket edges (the emulator with TNCCL_NET=force):
// the ring over host-mapped FIFOs that in-process proxy threads move over
// loopback TCP. Also cooperative: rank k's CTAs wait for data that rank k-1's
// CTAs produce.
template <typename T>
__global__ void __launch_bounds__(kMaxThreads)
    emulatedNetRingKernel(const __grid_constant__ EmulatedLaunch e) {
  ringBody<T, true>(e.comm[blockIdx.y], e.args[blockIdx.y], blockIdx.x);
}

template <typename T>
cudaError_t launchEmulatedTyped(const EmulatedLaunch& e, int channels, int threads,
                                cudaStream_t stream) {
  const dim3 grid((unsigned)channels, (unsigned)e.nranks);
  const dim3 block((unsigned)threads);
  void* args[] = {const_cast<EmulatedLaunch*>(&e)};
  bool socketEdges = false;
  for (int k = 0; k < e.nranks; ++k)
    socketEdges = socketEdges || e.comm[k].netSend != nullptr || e.comm[k].netRecv != nullptr;
  if (e.algo == TNCCL_ALGO_RING && socketEdges)
    return cudaLaunchCooperativeKernel((const void*)emulatedNetRingKernel<T>, grid, block, args,
                                       0, stream);
  const void* fn = e.nranks <= 2   ? (const void*)emulatedKernel<T, 2>
                   : e.nranks <= 4 ? (const void*)emulatedKernel<T, 4>
                                   : (const void*)emulatedKernel<T, 8>;
  // Dynamic shared memory of the two-shot body for this kernel's MAXP.
  const uint32_t smem = twoShotSmemBytes(e.comm[0], e.nranks <= 2 ? 2 : e.nranks <= 4 ? 4 : 8);
  cudaError_t err = e.nranks <= 2   ? allowSmem<emulatedKernel<T, 2>>(smem)
                    : e.nranks <= 4 ? allowSmem<emulatedKernel<T, 4>>(smem)
                                    : allowSmem<emulatedKernel<T, 8>>(smem);
  if (err != cudaSuccess) return err;
  return cudaLaunchCooperativeKernel(fn, grid, block, args, smem, stream);
}

template <typename T>
int emulatedMaxCtasTyped(int threads) {
  int perSm = 0, sms = 0, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  DevComm d{};
  d.tsStages = 2;
  d.tsPushStage = 32768;
  d.tsRedStage = 65536;
  const uint32_t smem = twoShotSmemBytes(d, 2);  // the largest layout
  if (allowSmem<emulatedKernel<T, 8>>(smem) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&perSm, emulatedKernel<T, 8>, threads, smem) !=
          cudaSuccess)
    return 0;
  return perSm * sms;
}

// Launches `kernel` and returns that launch's own error. A triple-chevron
// launch followed by cudaGetLastError would also report (and clear) an
// unrelated error that an earlier call of the caller left behind.
template <typename... Params, typename... Args>
cudaError_t launchOwn(void (*kernel)(Params...), unsigned grid, dim3 block, uint32_t smem,
                      cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename T, int MAXP>
cudaError_t launchTwoShot(const DevComm& comm, const AllReduceArgs& a, dim3 block,
                          cudaStream_t stream) {
  const uint32_t smem = twoShotSmemBytes(comm, MAXP);
  cudaError_t err = allowSmem<twoShotKernel<T, MAXP>>(smem);
  if (err != cudaSuccess) return err;
  return launchOwn(twoShotKernel<T, MAXP>, a.chunk.channels, block, smem, stream, comm, a);
}

template <typename T>
cudaError_t launchTyped(const DevComm& comm, const AllReduceArgs& a, int algo, int threads,
                        cudaStream_t stream) {
  const dim3 block((unsigned)threads);
  switch (algo) {
    case TNCCL_ALGO_RING:
      if (comm.netSend || comm.netRecv)
        return launchOwn(ringKernel<T, true>, a.chunk.channels, block, 0, stream, comm, a);
      return launchOwn(ringKernel<T, false>, a.chunk.channels, block, 0, stream, comm, a);
    case TNCCL_ALGO_TWOSHOT:
      if (comm.nranks <= 2)
        return launchTwoShot<T, 2>(comm, a, block, stream);
      else if (comm.nranks <= 4)
        return launchTwoShot<T, 4>(comm, a, block, stream);
      else if (comm.nranks <= 8)
        return launchTwoShot<T, 8>(comm, a, block, stream);
      return launchTwoShot<T, 16>(comm, a, block, stream);
    case TNCCL_ALGO_ONESHOT:
      if (comm.nranks <= 2)
        return launchOwn(oneShotKernel<T, 2>, a.block.channels, block, 0, stream, comm, a);
      if (comm.nranks <= 4)
        return launchOwn(oneShotKernel<T, 4>, a.block.channels, block, 0, stream, comm, a);
      if (comm.nranks <= 8)
        return launchOwn(oneShotKernel<T, 8>, a.block.channels, block, 0, stream, comm, a);
      return launchOwn(oneShotKernel<T, 16>, a.block.channels, block, 0, stream, comm, a);
    case TNCCL_ALGO_NVLS: {
      if (a.mcSend != nullptr)
        return launchOwn(nvlsZeroCopyKernel<T>, a.zcChannels, block, 0, stream, comm, a);
      const uint32_t smem = nvlsSmemBytes(comm);
      cudaError_t err = allowSmem<nvlsKernel<T>>(smem);
      if (err != cudaSuccess) return err;
      return launchOwn(nvlsKernel<T>, a.block.channels, block, smem, stream, comm, a);
    }
    default:
      return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launchScaleTyped(const void* x, void* y, uint64_t n, float alpha, int vectorized,
                             cudaStream_t stream) {
  const uint64_t work = vectorized ? n / Pack<T>::V + 1 : n;
  unsigned blocks = (unsigned)minU64(divUp(work, 256), 148ull * 8);
  if (blocks == 0) blocks = 1;
  return launchOwn(scaleKernel<T>, blocks, dim3(256), 0, stream, static_cast<const T*>(x),
                   static_cast<T*>(y), n, alpha, vectorized);
}

}  // namespace

cudaError_t launchAllReduceKernel(const DevComm& comm, const AllReduceArgs& a, int algo,
                                  int threads, cudaStream_t stream) {
  if (threads > kMaxThreads) threads = kMaxThreads;
  switch (a.dtype) {
    case kF32:
      return launchTyped<float>(comm, a, algo, threads, stream);
    case kBF16:
      return launchTyped<__nv_bfloat16>(comm, a, algo, threads, stream);
    case kF16:
      return launchTyped<__half>(comm, a, algo, threads, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launchScale(const void* x, void* y, uint64_t n, int dtype, float alpha,
                        int vectorized, cudaStream_t stream) {
  switch (dtype) {
    case kF32:
      return launchScaleTyped<float>(x, y, n, alpha, vectorized, stream);
    case kBF16:
      return launchScaleTyped<__nv_bfloat16>(x, y, n, alpha, vectorized, stream);
    case kF16:
      return launchScaleTyped<__half>(x, y, n, alpha, vectorized, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace tnccl

namespace tnccl {

cudaError_t launchEmulated(const EmulatedLaunch& e, int channels, int threads,
                           cudaStream_t stream) {
  if (threads > kMaxThreads) threads = kMaxThreads;
  switch (e.dtype) {
    case kF32:
      return launchEmulatedTyped<float>(e, channels, threads, stream);
    case kBF16:
      return launchEmulatedTyped<__nv_bfloat16>(e, channels, threads, stream);
    case kF16:
      return launchEmulatedTyped<__half>(e, channels, threads, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

int emulatedMaxCtas(int threads) {
  return emulatedMaxCtasTyped<float>(threads > kMaxThreads ? kMaxThreads : threads);
}

}  // namespace tnccl
