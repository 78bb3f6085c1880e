// ring.cuh - the multi-channel ring all-reduce body (included by
// allreduce.cu).
#pragma once

#include "kernel_common.cuh"

namespace tnccl {
namespace {

using namespace dev;

// ---------------------------------------------------------------------------
// Ring (per-channel FIFO with ready words in the consumer and credit words in
// the producer, both polled locally). Each edge is a RingFifo: over NVLink
// it is made of the two mailboxes; a socket edge (TNCCL_NET) is a host-mapped
// FIFO that the rank's proxy thread moves over TCP, where the producer also
// writes each slot's payload size.
// ---------------------------------------------------------------------------
template <typename T, bool NET>
struct RingChannel {
  const DevComm* comm;
  int c, next, prev;
  char* me;
  uint64_t sendT, recvT;

  // The two edges, rebuilt from the launch parameters at each use (cheaper in
  // registers than keeping them). NET = false compiles the NVLink-only ring.
  __device__ RingFifo out() const {
    return NET && comm->netSend ? netRingFifo(comm->netSend, comm->netLayout)
                                : nvlinkRingFifo(comm->peers[next], me, comm->layout);
  }
  __device__ RingFifo in() const {
    return NET && comm->netRecv ? netRingFifo(comm->netRecv, comm->netLayout)
                                : nvlinkRingFifo(me, comm->peers[prev], comm->layout);
  }
  __device__ char* outSlot(uint64_t t) const { return ringFifoData(out(), c, t); }
  __device__ const T* inSlot(uint64_t t) const {
    return reinterpret_cast<const T*>(ringFifoData(in(), c, t));
  }
  // Thread 0 waits; the caller passes bar.sync before using the slots.
  __device__ bool waitSend(int phase) const {
    const RingFifo f = out();
    return waitExact(f.credit + ringFifoIndex(f, c, sendT), sendT, phase);
  }
  __device__ bool waitRecv(int phase) const {
    const RingFifo f = in();
    return waitExact(f.ready + ringFifoIndex(f, c, recvT), recvT + 1, phase);
  }
  // A ring FIFO word never runs ahead of its waiter: a credit cannot pass
  // ticket t before t was sent, a ready word cannot pass t + 1 before t was
  // credited back. Debug builds check the word equals the target exactly.
  __device__ bool waitExact(const uint64_t* w, uint64_t target, int phase) const {
    if (!waitFlag(*comm, w, target, whereCode(kCounterRing, c, phase))) return false;
#if TNCCL_DEVICE_CHECKS
    const uint64_t v = ldAcquireSys(w);
    if (v != target) {
      recordFailure(*comm, 3, whereCode(kCounterRing, c, phase | kCheckPhase), target, v);
      return false;
    }
#endif
    return true;
  }
  // Called by thread 0 after bar.sync.
  __device__ void publishSend(uint64_t bytes) {
    const RingFifo f = out();
    const uint64_t i = ringFifoIndex(f, c, sendT);
    if (NET && f.bytes) f.bytes[i] = bytes;  // ordered by the release below
    stReleaseSys(f.ready + i, sendT + 1);
    ++sendT;
  }
  __device__ void releaseRecv() {
    const RingFifo f = in();
    stReleaseSys(f.credit + ringFifoIndex(f, c, recvT), recvT + (uint64_t)f.slots);
    ++recvT;
  }
};

template <typename T, bool NET>
__device__ __forceinline__ void ringBody(const DevComm& comm, const AllReduceArgs& a,
                                         const int c) {
  using Pk = Pack<T>;
  constexpr int V = Pk::V;
  const int tid = threadIdx.x, P = comm.nranks, r = comm.rank;
  const Team cta = wholeCta();
  const T* x = static_cast<const T*>(a.send);
  T* y = static_cast<T*>(a.recv);
  const ChunkPlan& pl = a.chunk;
  const bool vec = a.vectorized != 0;
  const float alpha = a.scale;
  const bool scale = alpha != 1.0f;
  __shared__ int sFail;
  if (tid == 0) sFail = 0;
  RingChannel<T, NET> ch;
  ch.comm = &comm;
  ch.c = c;
  ch.next = (r + 1) % P;
  ch.prev = (r + P - 1) % P;
  ch.me = comm.peers[r];
  ch.sendT = ch.recvT = comm.counters[kCounterRing * kMaxChannels + c];
  // A socket edge provisions netLayout.channels channels (the host caps the
  // plan to them); a launch beyond them would write outside its FIFO.
  if (NET && tid == 0 && (comm.netSend || comm.netRecv) && c >= comm.netLayout.channels) {
    recordFailure(comm, 1 /* TNCCL_INVALID_ARGUMENT */, whereCode(kCounterRing, c, 0), 0, 0);
    sFail = 1;
  }
  {
    const uint64_t cap = minU64(ch.out().chunkBytes, ch.in().chunkBytes);
    if (!planFits(comm, pl.chunkElems * sizeof(T), cap, c, comm.layout.channels, kCounterRing) &&
        tid == 0)
      sFail = 1;
  }
  __syncthreads();

  // Wait helpers: `needRecv` / `needSend` select which FIFO ends to acquire.
  auto acquire = [&](bool needRecv, bool needSend, int phase) -> bool {
    if (tid == 0) {
      bool ok = true;
      if (needRecv) ok = ch.waitRecv(phase);
      if (ok && needSend) ok = ch.waitSend(phase);
      if (!ok) sFail = 1;
    }
    __syncthreads();
    return sFail == 0;
  };
  // sendElems: elements of T in the slot just written (socket edges carry
  // exactly those bytes).
  auto finish = [&](bool recvDone, bool sendDone, uint64_t sendElems) {
    __syncthreads();
    if (tid == 0) {
      if (recvDone) ch.releaseRecv();
      if (sendDone) ch.publishSend(sendElems * sizeof(T));
    } else {
      if (recvDone) ++ch.recvT;
      if (sendDone) ++ch.sendT;
    }
  };

  const uint64_t ntiles = channelTiles(pl.numTiles, pl.channels, c);
  for (uint64_t t = 0; t < ntiles && !sFail; ++t) {
    const uint64_t tile = (uint64_t)c + t * (uint64_t)pl.channels;
    // Reduce-scatter: send chunk r-1.
    {
      const Span sp = chunkSpan(pl, tile, ringChunkBehind(r, 1, P), V);
      if (!acquire(false, true, 1)) break;
      char* out = ch.outSlot(ch.sendT);
      copyOut<T, kLdInput, 8>(cta, x + sp.offset, sp.count, vec, scale, alpha, 1,
                              [out](int) { return out; });
      finish(false, true, sp.count);
    }
    // recv + reduce + send for distances 2..P-1.
    bool ok = true;
    for (int d = 2; d < P && ok; ++d) {
      const Span sp = chunkSpan(pl, tile, ringChunkBehind(r, d, P), V);
      if (!(ok = acquire(true, true, 2))) break;
      const T* in = ch.inSlot(ch.recvT);
      char* out = ch.outSlot(ch.sendT);
      ringHop<T, 2>(
          cta, sp.count, vec, in, x + sp.offset, alpha,
          [&](uint64_t i, uint4 v) { st16(reinterpret_cast<uint4*>(out) + i, v); },
          [&](uint64_t e, float f) { stElem(reinterpret_cast<T*>(out) + e, f); });
      finish(true, true, sp.count);
    }
    if (!ok) break;
    // Final reduce-scatter step: y[chunk r] = in + a*x, stored and forwarded.
    {
      const Span sp = chunkSpan(pl, tile, r, V);
      if (!acquire(true, true, 3)) break;
      const T* in = ch.inSlot(ch.recvT);
      char* out = ch.outSlot(ch.sendT);
      T* yo = y + sp.offset;
      ringHop<T, 2>(
          cta, sp.count, vec, in, x + sp.offset, alpha,
          [&](uint64_t i, uint4 v) {
            st16(reinterpret_cast<uint4*>(yo) + i, v);
            st16(reinterpret_cast<uint4*>(out) + i, v);
          },
          [&](uint64_t e, float f) {
            stElem(yo + e, f);
            stElem(reinterpret_cast<T*>(out) + e, f);
          });
      finish(true, true, sp.count);
    }
    // All-gather: recv + store + forward for distances 1..P-2, then store.
    for (int d = 1; d < P - 1 && ok; ++d) {
      const Span sp = chunkSpan(pl, tile, ringChunkBehind(r, d, P), V);
      if (!(ok = acquire(true, true, 4))) break;
      const T* in = ch.inSlot(ch.recvT);
      char* out = ch.outSlot(ch.sendT);
      T* yo = y + sp.offset;
      copyOut<T, kLdMailbox, 8>(cta, in, sp.count, vec, false, 1.f, 2, [&](int k) {
        return k == 0 ? reinterpret_cast<char*>(yo) : out;
      });
      finish(true, true, sp.count);
    }
    if (!ok) break;
    {
      const Span sp = chunkSpan(pl, tile, ringChunkBehind(r, P - 1, P), V);
      if (!acquire(true, false, 5)) break;
      T* yo = y + sp.offset;
      copyOut<T, kLdMailbox, 8>(cta, ch.inSlot(ch.recvT), sp.count, vec, false, 1.f, 1,
                                [yo](int) { return reinterpret_cast<char*>(yo); });
      finish(true, false, 0);
    }
  }
  if (tid == 0 && !sFail) comm.counters[kCounterRing * kMaxChannels + c] = ch.sendT;
}

}  // namespace
}  // namespace tnccl
