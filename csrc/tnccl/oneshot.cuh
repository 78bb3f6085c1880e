// oneshot.cuh - the one-shot all-reduce body (included by allreduce.cu).
#pragma once

#include "kernel_common.cuh"

namespace tnccl {
namespace {

using namespace dev;

// ---------------------------------------------------------------------------
// One-shot: osSlots slots per channel; consumers acknowledge each slot so the
// producer never overwrites a block that a peer has not reduced yet.
// ---------------------------------------------------------------------------
template <typename T, int MAXP>
__device__ __forceinline__ void oneShotBody(const DevComm& comm, const AllReduceArgs& a,
                                            const int c) {
  constexpr int U = MAXP <= 2 ? 4 : MAXP <= 4 ? 2 : 1;
  const int tid = threadIdx.x, P = comm.nranks, r = comm.rank;
  const Team cta = wholeCta();
  const MailboxLayout& L = comm.layout;
  const int S = L.osSlots;
  char* const me = comm.peers[r];
  const T* x = static_cast<const T*>(a.send);
  T* y = static_cast<T*>(a.recv);
  const BlockPlan& pl = a.block;
  const bool vec = a.vectorized != 0;
  if (!planFits(comm, pl.tileElems * sizeof(T), L.osTileBytes, c, L.osChannels,
                kCounterOneShot))
    return;
  __shared__ int sFail;
  if (tid == 0) sFail = 0;
  uint64_t seq = comm.counters[kCounterOneShot * kMaxChannels + c];
  __syncthreads();
  const uint64_t ntiles = channelTiles(pl.numTiles, pl.channels, c);
  for (uint64_t t = 0; t < ntiles; ++t) {
    const uint64_t tile = (uint64_t)c + t * (uint64_t)pl.channels;
    const Span sp = blockTileSpan(pl, tile);
    const int s = (int)(seq % (uint64_t)S);
    const uint64_t want = seq + 1;
    traceMark(comm, c, kCounterOneShot, 0, t);
    // The slot is free once every consumer acknowledged its previous use.
    if (seq >= (uint64_t)S && tid < P && tid != r &&
        !waitFlag(comm, flagPtr(me, osAckAt(L, c, s, tid)), seq - (uint64_t)S + 1,
                  whereCode(kCounterOneShot, c, 0)))
      sFail = 1;
    __syncthreads();
    if (sFail) break;
    traceMark(comm, c, kCounterOneShot, 1, t);
    const uint64_t dataOff = osDataAt(L, c, s, r);
    copyOut<T, kLdInput, 8>(cta, x + sp.offset, sp.count, vec, false, 1.f, P - 1, [&](int d) {
      return comm.peers[(r + 1 + d) % P] + dataOff;
    });
    __syncthreads();
    if (tid < P && tid != r) stReleaseSys(flagPtr(comm.peers[tid], osFlagAt(L, c, s, r)), want);
    traceMark(comm, c, kCounterOneShot, 2, t);
    if (tid < P && tid != r &&
        !waitFlag(comm, flagPtr(me, osFlagAt(L, c, s, tid)), want,
                  whereCode(kCounterOneShot, c, 1)))
      sFail = 1;
    __syncthreads();
    if (sFail) break;
    traceMark(comm, c, kCounterOneShot, 3, t);
    reduceRanks<T, MAXP, U>(
        cta, sp.count, vec, P, r, x + sp.offset, a.scale,
        [&](int k) { return me + osDataAt(L, c, s, k); },
        [&](uint64_t i, uint4 v) { st16(reinterpret_cast<uint4*>(y + sp.offset) + i, v); },
        [&](uint64_t e, float f) { stElem(y + sp.offset + e, f); });
    __syncthreads();  // every read of slot s is done
    if (tid < P && tid != r) stReleaseSys(flagPtr(comm.peers[tid], osAckAt(L, c, s, r)), want);
    traceMark(comm, c, kCounterOneShot, 4, t);
    ++seq;
  }
  if (tid == 0 && !sFail) comm.counters[kCounterOneShot * kMaxChannels + c] = seq;
}

}  // namespace
}  // namespace tnccl
