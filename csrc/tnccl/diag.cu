// diag.cu - NVLink / HBM primitive micro-benchmarks used to size the
// collective kernels (tncclDiagBench in diag.h). Each mode moves `bytes`
// between this rank's mailbox and the next rank's mailbox with `ctas` CTAs of
// `threads` threads and `unroll` 16-byte accesses in flight per thread:
//   0 push   : weak 16-byte stores into the peer's mailbox
//   1 pull   : 16-byte loads from the peer's mailbox (summed so they count)
//   2 push+flag: push in `chunk`-byte pieces, each followed by bar.sync and a
//              st.release.sys flag to the peer (the cost of publishing)
//   3 local  : copy within this rank's mailbox
//   4 local->peer copy, 5 two local loads -> one local + one peer store
//   6 push while warp 0 keeps issuing one ordering operation (chunk picks it)
//   7 / 8 TMA-staged copy local->peer / local->local (unroll = stages,
//         chunk = stage bytes); 9 = 7 with every stage split into 8 copies
//   10 / 11 / 12 NVLS: multimem.ld_reduce of this rank's share / multimem.st
//         of the whole block / both (bytes <= the NVLS region)
// The caller runs the same mode on every rank at the same time; no kernel
// waits on another rank, so there is nothing to time out.
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "comm.h"
#include "device.cuh"
#include "diag.h"

namespace tnccl {
namespace {

using namespace dev;

template <int U>
__global__ void diagKernel(char* local, char* peer, uint64_t bytes, int mode, uint64_t chunk,
                           uint64_t* peerFlag, unsigned* sink) {
  const uint64_t per = bytes / gridDim.x / 16 * 16;
  const uint64_t base = per * blockIdx.x;
  const uint64_t nvec = per / 16;
  const uint64_t NT = blockDim.x;
  uint32_t acc = 0;
  if (mode == 6) {
    // Warps 1.. push like mode 0 while warp 0 (lane 0) keeps issuing one
    // ordering operation every ~500 ns: chunk 0 none, 1 fence.acq_rel.sys,
    // 2 ld.acquire.sys of a local word, 3 st.release.sys to the peer.
    __shared__ volatile int sDone;
    if (threadIdx.x == 0) sDone = 0;
    __syncthreads();
    const uint64_t NT2 = NT - 32;
    if (threadIdx.x >= 32) {
      for (uint64_t b = threadIdx.x - 32; b < nvec; b += NT2 * U) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint64_t i = b + u * NT2;
          if (i < nvec) st16(peer + base + i * 16, make_uint4((uint32_t)i, 1, 2, 3));
        }
      }
      asm volatile("bar.sync 1, %0;" ::"r"((int)NT2) : "memory");
      if (threadIdx.x == 32) sDone = 1;
    } else if (threadIdx.x == 0) {
      uint64_t n = 0;
      while (!sDone && n < (1u << 24)) {
        if (chunk == 1) fenceAcqRelSys();
        if (chunk == 2) acc += (uint32_t)ldAcquireSys(reinterpret_cast<uint64_t*>(local));
        if (chunk == 3) stReleaseSys(peerFlag + blockIdx.x, ++n);
        ++n;
        __nanosleep(500);
      }
    }
  } else if (mode == 2) {
    const uint64_t cvec = chunk / 16;
    uint64_t seq = 0;
    for (uint64_t c0 = 0; c0 < nvec; c0 += cvec) {
      const uint64_t c1 = c0 + cvec < nvec ? c0 + cvec : nvec;
      for (uint64_t i = c0 + threadIdx.x; i < c1; i += NT) {
        uint4 v = make_uint4((uint32_t)i, 1, 2, 3);
        st16(peer + base + i * 16, v);
      }
      __syncthreads();
      if (threadIdx.x == 0) stReleaseSys(peerFlag + blockIdx.x, ++seq);
    }
  } else {
    for (uint64_t b = threadIdx.x; b < nvec; b += NT * U) {
      uint4 v[U];
      if (mode == 0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint64_t i = b + u * NT;
          if (i < nvec) st16(peer + base + i * 16, make_uint4((uint32_t)i, 1, 2, 3));
        }
        continue;
      }
      if (mode == 4 || mode == 5) {
        // 4: local -> peer copy; 5: two local sources summed into one local
        // and one peer store (the two-shot reduce mix).
        uint4 w[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint64_t i = b + u * NT;
          if (i < nvec) {
            v[u] = ldMailbox(local + base + i * 16);
            if (mode == 5) w[u] = ldMailbox(local + bytes + base + i * 16);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint64_t i = b + u * NT;
          if (i < nvec) {
            uint4 o = v[u];
            if (mode == 5) {
              o.x = __float_as_uint(__uint_as_float(o.x) + __uint_as_float(w[u].x));
              o.y = __float_as_uint(__uint_as_float(o.y) + __uint_as_float(w[u].y));
              o.z = __float_as_uint(__uint_as_float(o.z) + __uint_as_float(w[u].z));
              o.w = __float_as_uint(__uint_as_float(o.w) + __uint_as_float(w[u].w));
              st16(local + 2 * bytes + base + i * 16, o);
            }
            st16(peer + base + i * 16, o);
          }
        }
        continue;
      }
      char* src = mode == 1 ? peer : local;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint64_t i = b + u * NT;
        if (i < nvec) v[u] = ldMailbox(src + base + i * 16);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint64_t i = b + u * NT;
        if (i < nvec) {
          if (mode == 1)
            acc += v[u].x ^ v[u].w;
          else
            st16(local + bytes + base + i * 16, v[u]);
        }
      }
    }
  }
  if (acc == 0x12345678u) *sink = acc;
}

// Modes 7 / 8: the TMA-staged stream of the collectives (stageStream) with
// one team of the whole CTA: local -> peer (7) or local -> local (8), with
// `nb` stages of `stageBytes` in flight.
__global__ void diagStageKernel(const __grid_constant__ DevComm comm, char* local, char* peer,
                                uint64_t bytes, int mode, uint32_t stageBytes, int nb,
                                int pieces) {
  extern __shared__ __align__(128) char dsmem[];
  __shared__ int sFlag;
  uint64_t* bars = reinterpret_cast<uint64_t*>(dsmem);
  if (threadIdx.x == 0) {
    for (int i = 0; i < nb; ++i) mbarInit(bars + i, 1);
    fenceMbarInit();
  }
  __syncthreads();
  StageRing ring{dsmem + 128, bars, stageBytes, nb, 0, pieces};
  const Team tm = wholeCta();
  const uint64_t per = bytes / gridDim.x / 16 * 16;
  const char* src = local + per * blockIdx.x;
  char* dst = (mode == 8 ? local + bytes : peer) + per * blockIdx.x;
  (void)stageStream<1>(
      comm, tm, ring, 1, per / 16, [&](int) -> const void* { return src; },
      [&](uint64_t i, const uint4* v) { st16(reinterpret_cast<uint4*>(dst) + i, v[0]); },
      whereCode(15, blockIdx.x, 10), &sFlag);
}

// Modes 10-12: NVLS throughput over the multicast region: 10 streams
// multimem.ld_reduce (fp32 add), 11 streams multimem.st, 12 does both (the
// switch step of the NVLS all-reduce) on this rank's 1/P share. U operations
// in flight per thread.
template <int U>
__global__ void diagNvlsKernel(char* mc, uint64_t bytes, int mode, int nranks, int rank,
                               unsigned* sink) {
  uint64_t per = bytes / gridDim.x / 16 * 16;
  uint64_t base = per * blockIdx.x;
  if (mode != 11) {  // this rank's share of the CTA's block
    const uint64_t share = per / (uint64_t)nranks / 16 * 16;
    base += share * (uint64_t)rank;
    per = share;
  }
  const uint64_t nvec = per / 16, NT = blockDim.x;
  uint32_t acc = 0;
  for (uint64_t b = threadIdx.x; b < nvec; b += NT * U) {
    uint4 v[U];
    if (mode != 11) {
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (b + u * NT < nvec) v[u] = Multimem<float>::ldReduce(mc + base + (b + u * NT) * 16);
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = make_uint4((uint32_t)(b + u), 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (b + u * NT >= nvec) continue;
      if (mode == 10)
        acc += v[u].x ^ v[u].w;
      else
        Multimem<float>::st(mc + base + (b + u * NT) * 16, v[u]);
    }
  }
  if (acc == 0x12345678u) *sink = acc;
}

}  // namespace
}  // namespace tnccl

using namespace tnccl;

extern "C" tncclResult tncclDiagBench(tncclComm_t comm, int mode, size_t bytes, int ctas,
                                      int threads, int unroll, size_t chunk, int iters,
                                      cudaStream_t stream, float* msPerIter) {
  if (comm == nullptr || msPerIter == nullptr || comm->nranks < 2 || ctas < 1 || threads < 32 ||
      threads > 1024 || iters < 1)
    return TNCCL_INVALID_ARGUMENT;
  const int next = (comm->rank + 1) % comm->nranks;
  // Use the ring data area (and, for mode 3, its second half as destination).
  const size_t area = (size_t)comm->layout.channels *
                                                     comm->layout.ringSlots *
                                                     comm->layout.ringChunkBytes;
  const size_t span = bytes * (mode == 5 ? 3 : (mode == 3 || mode == 8) ? 2 : 1);
  if (bytes == 0 || span > area) return TNCCL_INVALID_ARGUMENT;
  char* local = comm->local.base + comm->layout.ringDataOff;
  char* peer = comm->dev.peers[next] + comm->layout.ringDataOff;
  // Flag words and the sink live in the scratch area after the payload, so
  // no FIFO sequence word is touched.
  const size_t tail = (span + 255) / 256 * 256;
  if (tail + 8 * (size_t)ctas + 256 > area) return TNCCL_INVALID_ARGUMENT;
  uint64_t* flag = reinterpret_cast<uint64_t*>(peer + tail);
  unsigned* sink = reinterpret_cast<unsigned*>(local + tail + 8 * (size_t)ctas);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  // Modes 7 / 8: `unroll` is the number of stages, `chunk` the stage bytes.
  const uint32_t smem = 128 + (uint32_t)unroll * (uint32_t)chunk;
  const bool staged = mode == 7 || mode == 8 || mode == 9;
  const bool nvls = mode >= 10 && mode <= 12;
  if (nvls && (!comm->nvls.enabled || bytes > comm->nvls.bytes)) return TNCCL_INVALID_ARGUMENT;
  char* mc = reinterpret_cast<char*>(comm->nvls.mcVa);
  if (staged) {
    if (unroll < 1 || unroll > 8 || chunk < 16 || chunk % 16 || smem > 220 * 1024)
      return TNCCL_INVALID_ARGUMENT;
    if (cudaFuncSetAttribute(diagStageKernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return TNCCL_CUDA_ERROR;
  }
  auto launch = [&]() {
    if (nvls) {
      switch (unroll) {
        case 2: diagNvlsKernel<2><<<ctas, threads, 0, stream>>>(mc, bytes, mode, comm->nranks, comm->rank, sink); break;
        case 8: diagNvlsKernel<8><<<ctas, threads, 0, stream>>>(mc, bytes, mode, comm->nranks, comm->rank, sink); break;
        case 16: diagNvlsKernel<16><<<ctas, threads, 0, stream>>>(mc, bytes, mode, comm->nranks, comm->rank, sink); break;
        default: diagNvlsKernel<4><<<ctas, threads, 0, stream>>>(mc, bytes, mode, comm->nranks, comm->rank, sink); break;
      }
      return;
    }
    if (staged) {
      diagStageKernel<<<ctas, threads, smem, stream>>>(comm->dev, local, peer, bytes, mode,
                                                       (uint32_t)chunk, unroll,
                                                       mode == 9 ? 8 : 1);
      return;
    }
    switch (unroll) {
      case 1: diagKernel<1><<<ctas, threads, 0, stream>>>(local, peer, bytes, mode, chunk, flag, sink); break;
      case 2: diagKernel<2><<<ctas, threads, 0, stream>>>(local, peer, bytes, mode, chunk, flag, sink); break;
      case 8: diagKernel<8><<<ctas, threads, 0, stream>>>(local, peer, bytes, mode, chunk, flag, sink); break;
      case 16: diagKernel<16><<<ctas, threads, 0, stream>>>(local, peer, bytes, mode, chunk, flag, sink); break;
      default: diagKernel<4><<<ctas, threads, 0, stream>>>(local, peer, bytes, mode, chunk, flag, sink); break;
    }
  };
  launch();
  cudaError_t err = cudaGetLastError();
  cudaEventRecord(e0, stream);
  for (int i = 0; i < iters; ++i) launch();
  cudaEventRecord(e1, stream);
  if (err == cudaSuccess) err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaEventSynchronize(e1);
  float ms = 0.f;
  if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  gLaunchCount.fetch_add((unsigned long long)iters + 1, std::memory_order_relaxed);
  if (err != cudaSuccess) return TNCCL_CUDA_ERROR;
  *msPerIter = ms / (float)iters;
  return TNCCL_SUCCESS;
}

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

extern "C" tncclResult tncclDiagWaitTimeout(tncclComm_t comm, int timeoutMs, cudaStream_t stream) {
  if (comm == nullptr || timeoutMs < 1 || comm->diagWord == nullptr) return TNCCL_INVALID_ARGUMENT;
  DevComm d = comm->dev;
  d.timeoutNs = (uint64_t)timeoutMs * 1000000ull;
  diagWaitKernel<<<1, 32, 0, stream>>>(d, comm->diagWord);
  gLaunchCount.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError() == cudaSuccess ? TNCCL_SUCCESS : TNCCL_CUDA_ERROR;
}

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
