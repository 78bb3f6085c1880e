// twoshot.cuh - the warp-specialised two-shot all-reduce body (included by
// allreduce.cu).
#pragma once

#include "kernel_common.cuh"

namespace tnccl {
namespace {

using namespace dev;

// ---------------------------------------------------------------------------
// Two-shot with three warp-specialised teams per channel CTA, each running
// its own loop over the channel's tiles:
//
//   push    RS(t): chunk j of my input -> rank j's reduce-scatter slot
//   reduce  wait RS(t) from every peer; y[own chunk] = sum in rank order,
//           pushed to every peer's all-gather slot
//   gather  wait AG(t) from every peer; copy the chunks out into y
//
// so NVLink stores (push, reduce), local copies (gather) and flag drains of
// one channel overlap instead of taking turns. S = kTwoShotSlots slots per
// channel and direction. Slot reuse needs no credit words:
//  * push writes RS(t) into slot t%S of rank j only after this CTA's gather
//    team copied AG(t-S) out (shared counter); j published AG(t-S) after it
//    finished reading RS(t-S) from that slot.
//  * reduce writes AG(t) into slot t%S of rank j only after j's RS(t)
//    arrived, which j's push team sent after j's gather team copied AG(t-S)
//    out of that slot.
// In-place calls are safe: gather overwrites chunk j of tile t only after
// AG(t) from j arrived, which needs this rank's RS(t) push, whose loads of
// that chunk completed before its release.
// ---------------------------------------------------------------------------
template <typename T, int MAXP>
__device__ __forceinline__ void twoShotBody(const DevComm& comm, const AllReduceArgs& a,
                                            const int c) {
  constexpr int V = Pack<T>::V;
  constexpr int U = MAXP <= 2 ? 4 : MAXP <= 4 ? 2 : 1;
  constexpr int S = kTwoShotSlots;
  const int P = comm.nranks, r = comm.rank;
  const MailboxLayout& L = comm.layout;
  char* const me = comm.peers[r];
  const T* x = static_cast<const T*>(a.send);
  T* y = static_cast<T*>(a.recv);
  const ChunkPlan& pl = a.chunk;
  const bool vec = a.vectorized != 0;
  using Pk = Pack<T>;
  const float alpha = a.scale;
  if (!haveSmem(comm, twoShotSmemBytes(comm, MAXP), kCounterTwoShot, c)) return;
  if (!planFits(comm, pl.chunkElems * sizeof(T), L.tsChunkBytes, c, L.channels, kCounterTwoShot))
    return;
  __shared__ int sFail;
  __shared__ int sTeamFlag[3];
  __shared__ unsigned long long sGathered;  // tiles the gather team copied out
  // Dynamic shared memory: the mbarriers of the two staged teams, then the
  // push and the reduce stage rings.
  constexpr int NP = MAXP > 1 ? MAXP - 1 : 1;  // peers' chunks per tile
  extern __shared__ __align__(128) char dsmem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(dsmem);
  const int nst = comm.tsStages;
  const uint32_t pushSrc = perSource(comm.tsPushStage, NP);
  const uint32_t redSrc = perSource(comm.tsRedStage, MAXP);
  char* ring0 = dsmem + kBarBytes;
  char* ring1 = ring0 + (size_t)nst * NP * pushSrc;
  StageRing pushRing{ring0, bars, pushSrc, nst, 0};
  StageRing redRing{ring1, bars + kMaxStages, redSrc, nst, 0};
  if (threadIdx.x == 0) {
    sFail = 0;
    sGathered = 0;
    for (int i = 0; i < nst; ++i) {
      mbarInit(bars + i, 1);
      mbarInit(bars + kMaxStages + i, 1);
    }
    fenceMbarInit();
  }
  const uint64_t seq0 = comm.counters[kCounterTwoShot * kMaxChannels + c];
  __syncthreads();
  const uint64_t ntiles = channelTiles(pl.numTiles, pl.channels, c);
  auto tileOf = [&](uint64_t t) { return (uint64_t)c + t * (uint64_t)pl.channels; };
  auto slotOf = [&](uint64_t t) { return (int)((seq0 + t) % S); };
  int role;
  const Team tm = splitTeams(comm.tsSplit, &role);
  // Thread k < P of a team waits for / publishes to peer k.
  const bool peerThread = tm.tid < P && tm.tid != r;
  const int k = tm.tid;

  if (role == kTsPush) {
    for (uint64_t t = 0; t < ntiles; ++t) {
      if (t >= (uint64_t)S) {
        if (tm.lead() && !waitLocal(comm, &sGathered, t - S + 1, &sFail,
                                    whereCode(kCounterTwoShot, c, 3)))
          sFail = 1;
        tm.sync();
        if (sFail) break;
      }
      const uint64_t tile = tileOf(t);
      const int slot = slotOf(t);
      // Chunk j of my input -> rank j's slot, every peer in one staged pass
      // (source k is peer (r + 1 + k) % P).
      auto peerOf = [&](int q) { return (r + 1 + q) % P; };
      const bool ok = stagedCopy<T, NP, kLdInput>(
          comm, tm, pushRing, P - 1, vec,
          [&](int q) { return x + chunkSpan(pl, tile, peerOf(q), V).offset; },
          [&](int q) { return chunkSpan(pl, tile, peerOf(q), V).count; },
          [&](int q) { return comm.peers[peerOf(q)] + tsRsDataAt(L, c, slot, r); },
          whereCode(kCounterTwoShot, c, 6), sTeamFlag + 0);
      if (!ok) {
        sFail = 1;
        break;
      }
      tm.sync();
      if (peerThread) stReleaseSys(flagPtr(comm.peers[k], tsRsFlagAt(L, c, slot, r)), seq0 + t + 1);
      traceMark(comm, c, kCounterTwoShot, 0, t, tm.lead());
    }
  } else if (role == kTsReduce) {
    for (uint64_t t = 0; t < ntiles; ++t) {
      const int slot = slotOf(t);
      if (peerThread && !waitFlag(comm, flagPtr(me, tsRsFlagAt(L, c, slot, k)), seq0 + t + 1,
                                  whereCode(kCounterTwoShot, c, 1)))
        sFail = 1;
      tm.sync();
      if (sFail) break;
      traceMark(comm, c, kCounterTwoShot, 1, t, tm.lead());
      const Span own = chunkSpan(pl, tileOf(t), r, V);
      const uint64_t agOff = tsAgDataAt(L, c, slot, r);
      // Vector part: every rank's contribution staged through shared memory
      // by TMA (own input from x, the others from the reduce-scatter slots),
      // summed in rank order in fp32, stored to y and pushed to every peer.
      // Short chunks skip the staging (one TMA round trip and two team
      // barriers per stage cost more than they hide) and reduce through
      // registers below.
      const uint64_t nv =
          vec && own.count * sizeof(T) >= comm.stageMinBytes ? own.count / V : 0;
      if (nv > 0 &&
          !stageStream<MAXP>(
              comm, tm, redRing, P, nv,
              [&](int q) -> const void* {
                return q == r ? static_cast<const void*>(x + own.offset)
                              : static_cast<const void*>(me + tsRsDataAt(L, c, slot, q));
              },
              [&](uint64_t i, const uint4* v) {
                float acc[V], f[V];
                Pk::unpack(v[0], acc);
#pragma unroll
                for (int e = 0; e < V; ++e) acc[e] = scaled(alpha, acc[e]);
#pragma unroll
                for (int q = 1; q < MAXP; ++q) {
                  if (q < P) {
                    Pk::unpack(v[q], f);
#pragma unroll
                    for (int e = 0; e < V; ++e) acc[e] = addRn(acc[e], scaled(alpha, f[e]));
                  }
                }
                const uint4 o = Pk::pack(acc);
                st16(reinterpret_cast<uint4*>(y + own.offset) + i, o);
                for (int d = 1; d < P; ++d) {
                  const int j = (r + d) % P;
                  st16(reinterpret_cast<uint4*>(comm.peers[j] + agOff) + i, o);
                }
              },
              whereCode(kCounterTwoShot, c, 7), sTeamFlag + 1)) {
        sFail = 1;
        break;
      }
      // The rest: scalar tail, or the whole chunk when it is short (vectors)
      // or the buffers are unaligned (scalars).
      const uint64_t e0 = nv * V;
      reduceRanks<T, MAXP, U>(
          tm, own.count - e0, vec && nv == 0, P, r, x + own.offset + e0, alpha,
          [&](int q) { return me + tsRsDataAt(L, c, slot, q) + e0 * sizeof(T); },
          [&](uint64_t i, uint4 v) {
            st16(reinterpret_cast<uint4*>(y + own.offset + e0) + i, v);
            for (int d = 1; d < P; ++d) {
              const int j = (r + d) % P;
              st16(reinterpret_cast<uint4*>(comm.peers[j] + agOff + e0 * sizeof(T)) + i, v);
            }
          },
          [&](uint64_t e, float f) {
            stElem(y + own.offset + e0 + e, f);
            for (int d = 1; d < P; ++d) {
              const int j = (r + d) % P;
              stElem(reinterpret_cast<T*>(comm.peers[j] + agOff) + e0 + e, f);
            }
          });
      tm.sync();
      if (peerThread) stReleaseSys(flagPtr(comm.peers[k], tsAgFlagAt(L, c, slot, r)), seq0 + t + 1);
      traceMark(comm, c, kCounterTwoShot, 2, t, tm.lead());
    }
  } else {
    for (uint64_t t = 0; t < ntiles; ++t) {
      const int slot = slotOf(t);
      if (peerThread && !waitFlag(comm, flagPtr(me, tsAgFlagAt(L, c, slot, k)), seq0 + t + 1,
                                  whereCode(kCounterTwoShot, c, 2)))
        sFail = 1;
      tm.sync();
      if (sFail) break;
      traceMark(comm, c, kCounterTwoShot, 4, t, tm.lead());
      const uint64_t tile = tileOf(t);
      // Every peer's reduced chunk: all-gather slot -> y (register path).
      for (int d = 1; d < P; ++d) {
        const int j = (r + P - d) % P;
        const Span sp = chunkSpan(pl, tile, j, V);
        T* dst = y + sp.offset;
        copyOut<T, kLdMailbox, 8>(tm, reinterpret_cast<const T*>(me + tsAgDataAt(L, c, slot, j)),
                                  sp.count, vec, false, 1.f, 1, [dst](int) { return dst; });
      }
      tm.sync();
      if (tm.lead()) stReleaseCta(&sGathered, t + 1);
      traceMark(comm, c, kCounterTwoShot, 5, t, tm.lead());
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && !sFail) comm.counters[kCounterTwoShot * kMaxChannels + c] = seq0 + ntiles;
}

}  // namespace
}  // namespace tnccl
