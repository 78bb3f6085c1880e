// enqueue.cc - collective entry points: validation, algorithm selection,
// partition planning and the asynchronous launch on the bound stream.
//
// Validation follows tiny-nccl src/api.cc:29-96 (null pointers, byte-count
// overflow, partial overlap, current device, stream binding, single-rank
// identity). There is no host ticket reservation: FIFO sequence numbers live
// in device memory and advance inside the kernels (devcomm.h), which is what
// lets a captured CUDA graph replay a collective.
#include <stdint.h>

#include <atomic>
#include <limits>

#include "comm.h"
#include "launch.h"
#include "nvtx.h"

namespace tnccl {

std::atomic<unsigned long long> gLaunchCount{0};

namespace {

size_t elemSize(tncclDataType_t t) {
  switch (t) {
    case tncclFloat32:
      return 4;
    case tncclBfloat16:
    case tncclFloat16:
      return 2;
    default:
      return 0;
  }
}

bool partialOverlap(const void* send, const void* recv, size_t bytes) {
  if (send == recv || bytes == 0) return false;
  const uintptr_t s = reinterpret_cast<uintptr_t>(send);
  const uintptr_t r = reinterpret_cast<uintptr_t>(recv);
  const uintptr_t maxp = std::numeric_limits<uintptr_t>::max();
  if (s > maxp - bytes || r > maxp - bytes) return true;
  return s < r + bytes && r < s + bytes;
}

void bindStream(tncclComm* comm, cudaStream_t stream) {
  if (!comm->streamBound) {
    comm->boundStream = stream;
    comm->streamBound = true;
  }
}

}  // namespace

tncclAlgo_t selectAlgo(const tncclComm* comm, uint64_t bytes) {
  // With socket edges only the ring carries data between every neighbour;
  // on one host (TNCCL_NET=force) a forced algorithm still runs over NVLink.
  if (comm->net.any && (!comm->allPeersMapped || comm->cfg.forcedAlgo == TNCCL_ALGO_AUTO))
    return TNCCL_ALGO_RING;
  if (comm->cfg.forcedAlgo != TNCCL_ALGO_AUTO) {
    if (comm->cfg.forcedAlgo == TNCCL_ALGO_NVLS && !comm->nvls.enabled) return TNCCL_ALGO_TWOSHOT;
    return (tncclAlgo_t)comm->cfg.forcedAlgo;
  }
  const int tuned = tunedAlgo(comm->cfg.tuning, comm->nranks, bytes);
  if (tuned > 0 && (tuned != TNCCL_ALGO_NVLS || comm->nvls.enabled)) return (tncclAlgo_t)tuned;
  if (bytes <= comm->oneShotMaxBytes) return TNCCL_ALGO_ONESHOT;
  if (comm->nvls.enabled && bytes >= comm->nvlsMinBytes) return TNCCL_ALGO_NVLS;
  return TNCCL_ALGO_TWOSHOT;
}

}  // namespace tnccl

using namespace tnccl;

extern "C" tncclResult tncclAllReduceEx(const void* send, void* recv, size_t count,
                                        tncclDataType_t dtype, tncclRedOp_t op, float preScale,
                                        tncclAlgo_t algo, tncclComm_t comm,
                                        cudaStream_t stream) {
  const size_t es = elemSize(dtype);
  if (comm == nullptr || es == 0 || op < tncclSum || op >= tncclNumOps || algo < 0 ||
      algo >= TNCCL_NUM_ALGOS || (count != 0 && (send == nullptr || recv == nullptr)) ||
      count > std::numeric_limits<size_t>::max() / es) {
    return TNCCL_INVALID_ARGUMENT;
  }
  const size_t bytes = count * es;
  if (partialOverlap(send, recv, bytes)) return TNCCL_INVALID_ARGUMENT;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return TNCCL_CUDA_ERROR;
  if (device != comm->device) return TNCCL_INVALID_ARGUMENT;
  if (comm->streamBound && comm->boundStream != stream) return TNCCL_UNSUPPORTED;
  if (comm->aborted) return TNCCL_ABORTED;
  if (comm->hostStatus && comm->hostStatus->error != 0) {
    const int e = comm->hostStatus->error;
    const tncclResult r = e > 0 && e < TNCCL_NUM_RESULTS ? (tncclResult)e : TNCCL_SYSTEM_ERROR;
    if (!comm->deviceErrorReported) {
      comm->deviceErrorReported = true;
      // where = (counter family << 24) | (channel << 8) | phase (device.cuh).
      const int where = comm->hostStatus->where;
      const int family = (where >> 24) & 0x7f, channel = (where >> 8) & 0xffff;
      const int phase = where & 0xff;
      // The zero-copy kernel's entry barrier waits for every rank to reach
      // the same launch: ranks that chose differently (a buffer registered on
      // one rank only, different offsets or sizes, different channel caps)
      // launch different kernels and meet it only at the wait bound.
      const bool zcEntry = family == kCounterNvlsZc && phase == 1;
      TN_WARN("rank %d: a device wait gave up (result %d) in counter family %d, channel %d, "
              "phase %d; expected %llu, observed %llu%s",
              comm->rank, (int)r, family, channel, phase,
              (unsigned long long)comm->hostStatus->expectedSeq,
              (unsigned long long)comm->hostStatus->observedSeq,
              zcEntry ? ": the zero-copy NVLS entry barrier; every rank must pass registered "
                        "buffers at the same offsets, with the same size and the same "
                        "tncclCommSetMaxChannels value"
                      : "");
    }
    return r;
  }
  float scale = preScale;
  if (op == tncclAvg) scale = preScale / (float)comm->nranks;
  const int vectorized =
      (reinterpret_cast<uintptr_t>(send) % kVectorBytes == 0 &&
       reinterpret_cast<uintptr_t>(recv) % kVectorBytes == 0)
          ? 1
          : 0;

  if (comm->nranks == 1) {
    if (count != 0) {
      if (scale == 1.0f) {
        if (send != recv &&
            cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
          return TNCCL_CUDA_ERROR;
      } else {
        if (launchScale(send, recv, count, (int)dtype, scale, vectorized, stream) != cudaSuccess)
          return TNCCL_CUDA_ERROR;
        gLaunchCount.fetch_add(1, std::memory_order_relaxed);
      }
    }
    bindStream(comm, stream);
    return TNCCL_SUCCESS;
  }
  if (count == 0) {
    // Every rank derives zero tiles, so no FIFO state changes and no kernel
    // is needed to keep the ranks in step.
    bindStream(comm, stream);
    return TNCCL_SUCCESS;
  }

  // Zero-copy NVLS: both buffers registered (every rank registered the same
  // buffers, so every rank makes the same choice), whole 16-byte vectors, and
  // no socket edges (with them AUTO keeps every message on the ring).
  const Registration* regSend = nullptr;
  const Registration* regRecv = nullptr;
  if (comm->cfg.nvlsZeroCopy && comm->nvls.enabled && !comm->net.any && vectorized &&
      bytes % kVectorBytes == 0 &&
      (algo == TNCCL_ALGO_NVLS ||
       (algo == TNCCL_ALGO_AUTO &&
        (comm->cfg.forcedAlgo == TNCCL_ALGO_NVLS ||
         (comm->cfg.forcedAlgo == TNCCL_ALGO_AUTO &&
          bytes >= (uint64_t)comm->cfg.nvlsZcMinBytes))))) {
    regSend = findRegistration(comm, send, bytes);
    regRecv = regSend ? findRegistration(comm, recv, bytes) : nullptr;
  }
  const bool zeroCopy = regSend != nullptr && regRecv != nullptr;
  tncclAlgo_t chosen =
      zeroCopy ? TNCCL_ALGO_NVLS : algo == TNCCL_ALGO_AUTO ? selectAlgo(comm, bytes) : algo;
  if (chosen == TNCCL_ALGO_NVLS && !comm->nvls.enabled) return TNCCL_UNSUPPORTED;
  // The all-peer algorithms need every peer mapped.
  if (chosen != TNCCL_ALGO_RING && !comm->allPeersMapped) return TNCCL_UNSUPPORTED;

  AllReduceArgs a{};
  a.send = send;
  a.recv = recv;
  a.count = count;
  a.scale = scale;
  a.dtype = (int)dtype;
  a.vectorized = vectorized;
  const uint64_t V = kVectorBytes / es;
  const Config& cfg = comm->cfg;
  auto cap = [comm](int channels) {
    return comm->maxChannels > 0 && comm->maxChannels < channels ? comm->maxChannels : channels;
  };
  switch (chosen) {
    case TNCCL_ALGO_RING: {
      // Socket edges carry the first net.layout.channels channels only.
      int ch = cap(cfg.channels);
      if (comm->net.any && ch > comm->net.layout.channels) ch = comm->net.layout.channels;
      a.chunk = makeChunkPlan(count, comm->nranks, ch, (uint64_t)cfg.ringChunkBytes / es,
                              kRingMinChunkBytes / es, V);
      break;
    }
    case TNCCL_ALGO_TWOSHOT:
      a.chunk = makeChunkPlan(count, comm->nranks, cap(cfg.channels),
                              (uint64_t)cfg.tsChunkBytes / es, kTwoShotMinChunkBytes / es, V);
      break;
    case TNCCL_ALGO_ONESHOT:
      a.block = makeBlockPlan(count, cap(cfg.osChannels), (uint64_t)cfg.osTileBytes / es,
                              kOneShotMinTileBytes / es, V);
      break;
    case TNCCL_ALGO_NVLS:
      if (zeroCopy) {
        a.mcSend = reinterpret_cast<const char*>(regSend->mcVa) +
                   (static_cast<const char*>(send) - regSend->base);
        a.mcRecv = reinterpret_cast<char*>(regRecv->mcVa) +
                   (static_cast<char*>(recv) - regRecv->base);
        a.zcVecs = bytes / kVectorBytes;
        // From the message size and the configuration only: equal on every rank.
        a.zcChannels = nvlsZcChannels(a.zcVecs, comm->nranks, cap(cfg.nvlsZcChannels),
                                      kNvlsMinTileBytes / kVectorBytes);
        break;
      }
      a.block = makeBlockPlan(count, cap(comm->nvls.channels), comm->nvls.tileBytes / es,
                              kNvlsMinTileBytes / es, V);
      break;
    default:
      return TNCCL_INVALID_ARGUMENT;
  }
  TN_TRACE("rank %d: allreduce %zu x %zu B algo %s%s", comm->rank, count, es,
           tncclAlgoName(chosen), zeroCopy ? " (zero-copy)" : "");
  NvtxRange range("tncclAllReduce %s %zu B rank %d", tncclAlgoName(chosen), bytes, comm->rank);
  if (launchAllReduceKernel(comm->dev, a, (int)chosen, cfg.threads, stream) != cudaSuccess)
    return TNCCL_CUDA_ERROR;
  gLaunchCount.fetch_add(1, std::memory_order_relaxed);
  if (zeroCopy) ++comm->zeroCopyLaunches;
  bindStream(comm, stream);
  return TNCCL_SUCCESS;
}

extern "C" tncclResult tncclAllReduce(const void* send, void* recv, size_t count,
                                      tncclDataType_t dtype, tncclRedOp_t op, tncclComm_t comm,
                                      cudaStream_t stream) {
  return tncclAllReduceEx(send, recv, count, dtype, op, 1.0f, TNCCL_ALGO_AUTO, comm, stream);
}

extern "C" tncclResult tncclAllReduceSumF32(const float* send, float* recv, size_t count,
                                            tncclComm_t comm, cudaStream_t stream) {
  return tncclAllReduceEx(send, recv, count, tncclFloat32, tncclSum, 1.0f, TNCCL_ALGO_AUTO, comm,
                          stream);
}

extern "C" tncclResult tncclCommSelectAlgo(tncclComm_t comm, size_t count,
                                           tncclDataType_t dtype, tncclAlgo_t* algo) {
  const size_t es = elemSize(dtype);
  if (comm == nullptr || algo == nullptr || es == 0) return TNCCL_INVALID_ARGUMENT;
  *algo = comm->nranks == 1 ? TNCCL_ALGO_AUTO : selectAlgo(comm, (uint64_t)count * es);
  return TNCCL_SUCCESS;
}
