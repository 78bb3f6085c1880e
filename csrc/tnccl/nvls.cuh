// nvls.cuh - the warp-specialised NVLS all-reduce kernel (included by
// allreduce.cu).
#pragma once

#include "kernel_common.cuh"

namespace tnccl {
namespace {

using namespace dev;

// ---------------------------------------------------------------------------
// NVLS with three warp-specialised teams per channel CTA:
//
//   copy-in   x tile t -> this rank's input block (slot t%S, TMA-staged);
//             count "copied in" on every rank
//   switch    wait until all P ranks copied tile t in; multimem.ld_reduce
//             this rank's share of the tile in the NVSwitch and multimem.st
//             it to every rank's output block; count "stored"
//   copy-out  wait until all P ranks stored their share; copy the output
//             block to y
//
// The barriers are 64-bit counters per phase ("copied in", "stored"),
// channel and slot in the multicast region: a team leader adds 1 to every
// rank's copy with one multimem.red.release, and a wait polls the local copy
// until it reaches P x (uses of the slot so far). Block reuse (S = kNvlsSlots): copy-in overwrites input
// block t%S with tile t only after this CTA's copy-out finished tile t-S,
// which waited until every rank stored t-S, so every switch read of that
// block is done; a peer's multimem store of tile t into output block t%S
// follows its wait for this rank's "copied in t", counted after the same
// copy-out.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kMaxThreads)
    nvlsKernel(const __grid_constant__ DevComm comm, const __grid_constant__ AllReduceArgs a) {
  using Pk = Pack<T>;
  constexpr int V = Pk::V;
  constexpr int S = kNvlsSlots;
  const int c = blockIdx.x, P = comm.nranks, r = comm.rank;
  const T* x = static_cast<const T*>(a.send);
  T* y = static_cast<T*>(a.recv);
  const BlockPlan& pl = a.block;
  const bool vec = a.vectorized != 0;
  const float alpha = a.scale;
  const bool scale = alpha != 1.0f;
  const uint64_t tb = comm.nvlsTileBytes;
  if (!haveSmem(comm, nvlsSmemBytes(comm), kCounterNvls, c)) return;
  if (!planFits(comm, pl.tileElems * sizeof(T), tb, c, comm.nvlsChannels, kCounterNvls)) return;
  __shared__ int sFail;
  __shared__ int sTeamFlag[3];
  __shared__ unsigned long long sOut;  // tiles this CTA copied out
  // Dynamic shared memory: mbarriers, then the copy-in ring.
  extern __shared__ __align__(128) char dsmem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(dsmem);
  const int nst = comm.nvlsStages;
  const uint32_t stB = perSource(comm.nvlsStage, 1);
  StageRing inRing{dsmem + kBarBytes, bars, stB, nst, 0};
  if (threadIdx.x == 0) {
    sFail = 0;
    sOut = 0;
    for (int i = 0; i < nst; ++i) mbarInit(bars + i, 1);
    fenceMbarInit();
  }
  const uint64_t seq0 = comm.counters[kCounterNvls * kMaxChannels + c];
  __syncthreads();
  const uint64_t ntiles = channelTiles(pl.numTiles, pl.channels, c);
  auto slotOf = [&](uint64_t t) { return (int)((seq0 + t) % S); };
  auto spanOf = [&](uint64_t t) {
    return blockTileSpan(pl, (uint64_t)c + t * (uint64_t)pl.channels);
  };
  int role;
  const Team tm = splitTeams(comm.nvlsSplit, &role);  // copy-in / switch / copy-out
  auto counter = [&](char* base, int phase, uint64_t t) {
    return reinterpret_cast<uint64_t*>(
        base + nvlsCounterAt(tb, comm.nvlsChannels, phase, c, slotOf(t)));
  };
  // Counts phase `phase` of tile t on every rank.
  auto publish = [&](int phase, uint64_t t) {
    fenceProxyAlias();
    tm.sync();
    if (tm.lead()) multimemAddRelease(counter(comm.nvlsMc, phase, t), 1);
  };
  // Waits until every rank counted phase `phase` of tile t: its slot's
  // counter reaches P x (uses of the slot up to tile t).
  auto waitAll = [&](int phase, uint64_t t) -> bool {
    const uint64_t uses = (seq0 + t) / S + 1;
    if (tm.lead() && !waitFlag(comm, counter(comm.nvlsUc, phase, t), (uint64_t)P * uses,
                               whereCode(kCounterNvls, c, phase + 1)))
      sFail = 1;
    tm.sync();
    fenceProxyAlias();
    return sFail == 0;
  };

  if (role == 0) {
    for (uint64_t t = 0; t < ntiles; ++t) {
      if (t >= (uint64_t)S) {
        if (tm.lead() &&
            !waitLocal(comm, &sOut, t - S + 1, &sFail, whereCode(kCounterNvls, c, 3)))
          sFail = 1;
        tm.sync();
        if (sFail) break;
      }
      const Span sp = spanOf(t);
      char* dst = comm.nvlsUc + nvlsInAt(tb, c, slotOf(t));
      if (!stagedCopy<T, 1, kLdInput>(
              comm, tm, inRing, 1, vec, [&](int) { return x + sp.offset; },
              [&](int) { return sp.count; }, [&](int) { return dst; },
              whereCode(kCounterNvls, c, 7), sTeamFlag + 0)) {
        sFail = 1;
        break;
      }
      publish(0, t);
      traceMark(comm, c, kCounterNvls, 1, t, tm.lead());
    }
  } else if (role == 1) {
    for (uint64_t t = 0; t < ntiles; ++t) {
      if (!waitAll(0, t)) break;
      traceMark(comm, c, kCounterNvls, 2, t, tm.lead());
      // This rank's share of the tile, in whole vectors (padding past the
      // tile end is reduced but never copied out).
      const Span sp = spanOf(t);
      const int slot = slotOf(t);
      char* const mcIn = comm.nvlsMc + nvlsInAt(tb, c, slot);
      char* const mcOut = comm.nvlsMc + nvlsOutAt(tb, c, slot);
      const Span share = blockShare(divUp(sp.count, V), P, r, 1);
      const uint64_t NT = tm.nt;
      constexpr int UN = 8;  // switch reductions in flight per thread
      for (uint64_t base = tm.tid; base < share.count; base += NT * UN) {
        uint4 v[UN];
#pragma unroll
        for (int u = 0; u < UN; ++u) {
          const uint64_t i = share.offset + base + u * NT;
          if (base + u * NT < share.count) v[u] = Multimem<T>::ldReduce(mcIn + i * 16);
        }
#pragma unroll
        for (int u = 0; u < UN; ++u) {
          const uint64_t i = share.offset + base + u * NT;
          if (base + u * NT < share.count) {
            uint4 w = v[u];
            if (scale) {
              float f[V];
              Pk::unpack(w, f);
#pragma unroll
              for (int e = 0; e < V; ++e) f[e] = scaled(alpha, f[e]);
              w = Pk::pack(f);
            }
            Multimem<T>::st(mcOut + i * 16, w);
          }
        }
      }
      publish(1, t);
      traceMark(comm, c, kCounterNvls, 3, t, tm.lead());
    }
  } else {
    for (uint64_t t = 0; t < ntiles; ++t) {
      if (!waitAll(1, t)) break;
      traceMark(comm, c, kCounterNvls, 4, t, tm.lead());
      const Span sp = spanOf(t);
      const T* src = reinterpret_cast<const T*>(comm.nvlsUc + nvlsOutAt(tb, c, slotOf(t)));
      T* yo = y + sp.offset;
      copyOut<T, kLdMailbox, 8>(tm, src, sp.count, vec, false, 1.f, 1,
                                [yo](int) { return reinterpret_cast<char*>(yo); });
      tm.sync();
      if (tm.lead()) stReleaseCta(&sOut, t + 1);
      traceMark(comm, c, kCounterNvls, 5, t, tm.lead());
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && !sFail) comm.counters[kCounterNvls * kMaxChannels + c] = seq0 + ntiles;
}

// ---------------------------------------------------------------------------
// Zero-copy NVLS over buffers registered with tncclCommRegister. send and
// recv are bound to multicast objects of their own, so the switch reads every
// rank's send directly (multimem.ld_reduce) and multimem.st writes every
// rank's recv: nothing is copied in or out, and each GPU moves about
// (1 + 1/P) x the message per NVLink direction.
//
// Channel c of every rank counts two phases on every GPU with one
// multimem.red each: "entered" (this rank's stream reached the kernel, so its
// send is final and its recv no longer in use) and "stored" (its stores into
// everyone's recv are issued). A CTA reduces only after all P ranks entered
// and leaves only after all P stored, so recv is complete when the kernel
// ends on any rank, and no rank's buffers are touched after its kernel ended.
// The counters are monotone: launch k of channel c waits for P x (k + 1).
// Every rank must pass buffers at the same offsets inside their registrations
// (the multicast address names the same offset on every GPU).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kMaxThreads)
    nvlsZeroCopyKernel(const __grid_constant__ DevComm comm,
                       const __grid_constant__ AllReduceArgs a) {
  using Pk = Pack<T>;
  constexpr int V = Pk::V;
  const int c = blockIdx.x, P = comm.nranks, r = comm.rank;
  const float alpha = a.scale;
  const bool scale = alpha != 1.0f;
  __shared__ int sFail;
  if (threadIdx.x == 0) sFail = 0;
#if TNCCL_DEVICE_CHECKS
  // The grid is the plan's channel count and both multicast views are
  // 16-byte aligned (the host guarantees both; a debug build verifies).
  if (threadIdx.x == 0 &&
      ((int)gridDim.x != a.zcChannels ||
       ((reinterpret_cast<uintptr_t>(a.mcSend) | reinterpret_cast<uintptr_t>(a.mcRecv)) & 15))) {
    recordFailure(comm, 3, whereCode(kCounterNvlsZc, c, kCheckPhase), (uint64_t)a.zcChannels,
                  (uint64_t)gridDim.x);
    sFail = 1;
  }
  __syncthreads();
  if (sFail) return;
#endif
  const uint64_t seq0 = comm.counters[kCounterNvlsZc * kMaxChannels + c];
  const uint64_t target = (uint64_t)P * (seq0 + 1);
  auto counterOff = [&](int phase) {
    return nvlsZcCounterAt(comm.nvlsTileBytes, comm.nvlsChannels, phase, c);
  };
  // Counts `phase` on every rank, then waits until all P ranks counted it.
  auto barrier = [&](int phase) -> bool {
    fenceProxyAlias();
    __syncthreads();
    if (threadIdx.x == 0) {
      multimemAddRelease(reinterpret_cast<uint64_t*>(comm.nvlsMc + counterOff(phase)), 1);
      if (!waitFlag(comm, reinterpret_cast<const uint64_t*>(comm.nvlsUc + counterOff(phase)),
                    target, whereCode(kCounterNvlsZc, c, phase + 1)))
        sFail = 1;
    }
    __syncthreads();
    fenceProxyAlias();
    return sFail == 0;
  };
  if (!barrier(0)) return;
  traceMark(comm, c, kCounterNvlsZc, 1, seq0);
  const Span sp = nvlsZcSpan(a.zcVecs, P, r, a.zcChannels, c);
  const char* const in = a.mcSend + sp.offset * 16;
  char* const out = a.mcRecv + sp.offset * 16;
  const uint64_t NT = blockDim.x;
  constexpr int UN = 8;  // switch reductions in flight per thread
  for (uint64_t base = threadIdx.x; base < sp.count; base += NT * UN) {
    uint4 v[UN];
#pragma unroll
    for (int u = 0; u < UN; ++u) {
      const uint64_t i = base + u * NT;
      if (i < sp.count) v[u] = Multimem<T>::ldReduce(in + i * 16);
    }
#pragma unroll
    for (int u = 0; u < UN; ++u) {
      const uint64_t i = base + u * NT;
      if (i < sp.count) {
        uint4 w = v[u];
        if (scale) {
          float f[V];
          Pk::unpack(w, f);
#pragma unroll
          for (int e = 0; e < V; ++e) f[e] = scaled(alpha, f[e]);
          w = Pk::pack(f);
        }
        Multimem<T>::st(out + i * 16, w);
      }
    }
  }
  traceMark(comm, c, kCounterNvlsZc, 2, seq0);
  // The stores went to the recv buffers' multicast object, the barrier
  // counters live in the communicator's: a release on the counter does not
  // order stores to another multicast object, so every thread waits for its
  // own stores to be performed at system scope before the CTA counts
  // "stored".
  __threadfence_system();
  if (!barrier(1)) return;
  traceMark(comm, c, kCounterNvlsZc, 3, seq0);
  if (threadIdx.x == 0) comm.counters[kCounterNvlsZc * kMaxChannels + c] = seq0 + 1;
}

}  // namespace
}  // namespace tnccl
