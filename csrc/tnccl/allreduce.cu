// allreduce.cu - sm_100a all-reduce kernels and their launcher.
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
//            words are needed (see the slot-reuse argument below).
//   NVLS     teams copy the tile into the multicast-bound buffer, reduce this
//            rank's share in the NVSwitch (multimem.ld_reduce) and broadcast
//            it with multimem.st, and copy the result out; the barriers
//            between them are per-slot counters that every rank increments
//            on every GPU with one multimem.red.
//
// Every wait is bounded (device.cuh); a CTA whose wait fails stops, leaves
// its sequence number untouched and the host sees the recorded error.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "device.cuh"
#include "launch.h"
#include "protocol.h"
#include "tnccl.h"

namespace tnccl {
namespace {

using namespace dev;

constexpr int kLdInput = 0;
constexpr int kLdMailbox = 1;
constexpr int kMaxThreads = 512;

// Shared-memory staging (TMA bulk copies into a ring of stages per team).
// Two-shot: DevComm::tsStages stages for the push and the reduce team; a
// stage of tsPushStage / tsRedStage bytes is split evenly among the team's
// sources (MAXP - 1 peers' chunks for push, MAXP contributions for reduce).
// NVLS: nvlsStages stages of nvlsStage bytes for the copy-in team. The
// gather / copy-out teams load through registers: a CTA's TMA unit is shared
// by its teams, and on 2 x B200 moving the gather onto it as well cost 15-25%
// at 4-64 MiB. The first kBarBytes bytes hold the mbarriers, kMaxStages per
// team.
constexpr int kMaxStages = 8;
constexpr uint32_t kBarBytes = 256;
__host__ __device__ constexpr uint32_t perSource(uint32_t stage, int nsrc) {
  return stage / (uint32_t)nsrc / 16 * 16;
}
// The rings are reserved only when staging can happen: a staged copy moves at
// least stageMinBytes per source, and no source of a tile exceeds the two-shot
// chunk / the NVLS tile. With staging off (the default) a launch asks for the
// mbarrier bytes only, so it does not change the SM's shared-memory carve-out
// under the compute kernels it overlaps with.
__host__ __device__ uint32_t twoShotSmemBytes(const DevComm& d, int maxp) {
  if (d.stageMinBytes > d.layout.tsChunkBytes) return kBarBytes;
  const int np = maxp > 1 ? maxp - 1 : 1;
  return kBarBytes + (uint32_t)d.tsStages * (perSource(d.tsPushStage, np) * np +
                                             perSource(d.tsRedStage, maxp) * maxp);
}
__host__ __device__ uint32_t nvlsSmemBytes(const DevComm& d) {
  if (d.stageMinBytes > d.nvlsTileBytes) return kBarBytes;
  return kBarBytes + (uint32_t)d.nvlsStages * perSource(d.nvlsStage, 1);
}

// Opts `Kernel` into `bytes` of dynamic shared memory, once per device.
template <auto Kernel>
cudaError_t allowSmem(uint32_t bytes) {
  static std::atomic<uint32_t> done[64];
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 64 && done[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  err = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (err == cudaSuccess && dev < 64) done[dev].store(bytes, std::memory_order_release);
  return err;
}


template <int LD>
__device__ __forceinline__ uint4 ld16(const void* p) {
  return LD == kLdInput ? ldInput(p) : ldMailbox(p);
}

// Scalar element access (message tails and unaligned buffers).
template <typename T, int LD>
__device__ __forceinline__ float ldElem(const T* p) {
  if constexpr (sizeof(T) == 4) {
    uint32_t v;
    if (LD == kLdMailbox)
      asm volatile("ld.global.cg.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    else
      asm volatile("ld.global.cs.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return __uint_as_float(v);
  } else {
    unsigned short v;
    if (LD == kLdMailbox)
      asm volatile("ld.global.cg.b16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
    else
      asm volatile("ld.global.cs.b16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
    T t = *reinterpret_cast<T*>(&v);
    return Pack<T>::toF(t);
  }
}

template <typename T>
__device__ __forceinline__ void stElem(T* p, float x) {
  *p = Pack<T>::fromF(x);
}

// dst[i] = (scale ? alpha*src[i] : src[i]) for every destination returned by
// dstPtr(d), d < ndst. Loads are issued U at a time before any store.
template <typename T, int LD, int U, bool SCALE, typename DstF>
__device__ __forceinline__ void copyOutImpl(const Team& tm, const T* src, uint64_t n, bool vec,
                                            float alpha, int ndst, DstF dstPtr) {
  constexpr bool scale = SCALE;
  using Pk = Pack<T>;
  constexpr int V = Pk::V;
  const uint64_t NT = tm.nt;
  const uint64_t nvec = vec ? n / V : 0;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  for (uint64_t base = tm.tid; base < nvec; base += NT * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = base + u * NT;
      if (i < nvec) v[u] = ld16<LD>(s4 + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = base + u * NT;
      if (i < nvec) {
        uint4 w = v[u];
        if (scale) {
          float f[V];
          Pk::unpack(w, f);
#pragma unroll
          for (int e = 0; e < V; ++e) f[e] = scaled(alpha, f[e]);
          w = Pk::pack(f);
        }
        for (int d = 0; d < ndst; ++d) st16(reinterpret_cast<uint4*>(dstPtr(d)) + i, w);
      }
    }
  }
  for (uint64_t e = nvec * V + tm.tid; e < n; e += NT) {
    float f = ldElem<T, LD>(src + e);
    if (scale) f = scaled(alpha, f);
    for (int d = 0; d < ndst; ++d) stElem(reinterpret_cast<T*>(dstPtr(d)) + e, f);
  }
}

// Pure copies keep 8 loads in flight per thread; scaled copies convert
// through fp32 and keep 4 (register budget of a 512-thread CTA).
template <typename T, int LD, int U, typename DstF>
__device__ __forceinline__ void copyOut(const Team& tm, const T* src, uint64_t n, bool vec,
                                        bool scale, float alpha, int ndst, DstF dstPtr) {
  if (scale)
    copyOutImpl<T, LD, (U > 4 ? 4 : U), true>(tm, src, n, vec, alpha, ndst, dstPtr);
  else
    copyOutImpl<T, LD, U, false>(tm, src, n, vec, alpha, ndst, dstPtr);
}

// out[i] = sum_{k<P} alpha * src_k[i] in rank order, fp32 accumulation.
// Source localIdx is read from `local` (user input), every other source from
// srcPtr(k) (mailbox). out(i, pack) stores a 16-byte result; outElem(e, f)
// stores a scalar result.
template <typename T, int MAXP, int U, typename SrcF, typename OutF, typename OutElemF>
__device__ __forceinline__ void reduceRanks(const Team& tm, uint64_t n, bool vec, int P,
                                            int localIdx,
                                            const T* local, float alpha, SrcF srcPtr, OutF out,
                                            OutElemF outElem) {
  using Pk = Pack<T>;
  constexpr int V = Pk::V;
  const uint64_t NT = tm.nt;
  const uint64_t nvec = vec ? n / V : 0;
  for (uint64_t base = tm.tid; base < nvec; base += NT * U) {
    uint4 raw[U][MAXP];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = base + u * NT;
      if (i < nvec) {
#pragma unroll
        for (int k = 0; k < MAXP; ++k) {
          if (k < P) {
            raw[u][k] = k == localIdx
                            ? ldInput(reinterpret_cast<const uint4*>(local) + i)
                            : ldMailbox(reinterpret_cast<const uint4*>(srcPtr(k)) + i);
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = base + u * NT;
      if (i < nvec) {
        float acc[V], f[V];
        Pk::unpack(raw[u][0], acc);
#pragma unroll
        for (int e = 0; e < V; ++e) acc[e] = scaled(alpha, acc[e]);
#pragma unroll
        for (int k = 1; k < MAXP; ++k) {
          if (k < P) {
            Pk::unpack(raw[u][k], f);
#pragma unroll
            for (int e = 0; e < V; ++e) acc[e] = addRn(acc[e], scaled(alpha, f[e]));
          }
        }
        out(i, Pk::pack(acc));
      }
    }
  }
  for (uint64_t e = nvec * V + tm.tid; e < n; e += NT) {
    float acc = 0.f;
    for (int k = 0; k < P; ++k) {
      const float v = k == localIdx ? ldElem<T, kLdInput>(local + e)
                                    : ldElem<T, kLdMailbox>(reinterpret_cast<const T*>(srcPtr(k)) + e);
      acc = k == 0 ? scaled(alpha, v) : addRn(acc, scaled(alpha, v));
    }
    outElem(e, acc);
  }
}

// One ring hop: out = in + alpha * x with fp32 math and one rounding to T
// (tiny-nccl src/device.cuh:187 adds `received + local` the same way).
template <typename T, int U, typename OutF, typename OutElemF>
__device__ __forceinline__ void ringHop(const Team& tm, uint64_t n, bool vec, const T* in,
                                        const T* x,
                                        float alpha, OutF out, OutElemF outElem) {
  using Pk = Pack<T>;
  constexpr int V = Pk::V;
  const uint64_t NT = tm.nt;
  const uint64_t nvec = vec ? n / V : 0;
  for (uint64_t base = tm.tid; base < nvec; base += NT * U) {
    uint4 a[U], b[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = base + u * NT;
      if (i < nvec) {
        a[u] = ldMailbox(reinterpret_cast<const uint4*>(in) + i);
        b[u] = ldInput(reinterpret_cast<const uint4*>(x) + i);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t i = base + u * NT;
      if (i < nvec) {
        float fa[V], fb[V];
        Pk::unpack(a[u], fa);
        Pk::unpack(b[u], fb);
#pragma unroll
        for (int e = 0; e < V; ++e) fa[e] = addRn(fa[e], scaled(alpha, fb[e]));
        out(i, Pk::pack(fa));
      }
    }
  }
  for (uint64_t e = nvec * V + tm.tid; e < n; e += NT)
    outElem(e, addRn(ldElem<T, kLdMailbox>(in + e), scaled(alpha, ldElem<T, kLdInput>(x + e))));
}

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
enum TwoShotRole { kTsPush = 0, kTsReduce = 1, kTsGather = 2 };

// True when the launch provided at least `need` bytes of dynamic shared
// memory. Otherwise thread 0 records TNCCL_CUDA_ERROR (where-code phase 15)
// and every thread of the CTA must return before touching the rings.
__device__ __forceinline__ bool haveSmem(const DevComm& comm, uint32_t need, int family, int c) {
  uint32_t dyn;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
  if (need <= dyn) return true;
  if (threadIdx.x == 0) recordFailure(comm, 4, whereCode(family, c, 15), need, dyn);
  return false;
}

// Copies n (<= MAXSRC) local sources to their destinations: source k holds
// count(k) elements at src(k) (local memory), destination k is dst(k) (local
// or a peer's mailbox). The vectors that every source has are streamed
// through the team's TMA stage ring, all sources in one pass; what is left
// of each source (other chunk lengths, scalar tails, unaligned buffers) goes
// through registers; so does everything when the shortest source is below
// DevComm::stageMinBytes. Returns false if a stage never landed.
template <typename T, int MAXSRC, int LD, typename SrcF, typename CountF, typename DstF>
__device__ __forceinline__ bool stagedCopy(const DevComm& comm, const Team& tm, StageRing& R,
                                           int n, bool vec, SrcF src, CountF count, DstF dst,
                                           int where, volatile int* teamFlag) {
  constexpr int V = Pack<T>::V;
  uint64_t nv = ~0ull;
  for (int k = 0; k < n; ++k) {
    const uint64_t c = count(k) / V;
    nv = c < nv ? c : nv;
  }
  if (!vec || n == 0 || nv * 16 < comm.stageMinBytes) nv = 0;
  if (nv > 0 && !stageStream<MAXSRC>(
                    comm, tm, R, n, nv, [&](int k) -> const void* { return src(k); },
                    [&](uint64_t i, const uint4* v) {
#pragma unroll
                      for (int k = 0; k < MAXSRC; ++k)
                        if (k < n) st16(reinterpret_cast<uint4*>(dst(k)) + i, v[k]);
                    },
                    where, teamFlag))
    return false;
  for (int k = 0; k < n; ++k) {
    const uint64_t e0 = nv * V;
    char* d = dst(k) + e0 * sizeof(T);
    copyOut<T, LD, 8>(tm, src(k) + e0, count(k) - e0, vec, false, 1.f, 1,
                      [d](int) { return d; });
  }
  return true;
}

// Warp split of a CTA into three teams: split = a | b << 4 gives the first
// two teams a/8 and b/8 of the warps (at least one each), the third the rest
// (at least one; the launch has >= 4 warps).
__device__ __forceinline__ Team splitTeams(int split, int* role) {
  const int nw = blockDim.x / 32, w = threadIdx.x / 32;
  const TeamWarps tw = teamWarps(nw, split);
  const int nPush = tw.first, nRed = tw.second;
  if (w < nPush) {
    *role = kTsPush;
    return Team{(int)threadIdx.x, nPush * 32, 1};
  }
  if (w < nPush + nRed) {
    *role = kTsReduce;
    return Team{(int)threadIdx.x - nPush * 32, nRed * 32, 2};
  }
  *role = kTsGather;
  return Team{(int)threadIdx.x - (nPush + nRed) * 32, (nw - nPush - nRed) * 32, 3};
}

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

// ---------------------------------------------------------------------------
// One-shot: osSlots slots per channel; consumers acknowledge each slot so the
// producer never overwrites a block that a peer has not reduced yet.
// ---------------------------------------------------------------------------
template <typename T, int MAXP>
__device__ __forceinline__ void oneShotBody(const DevComm& comm, const AllReduceArgs& a,
                                            const int c) {
  constexpr int V = Pack<T>::V;
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

// ---------------------------------------------------------------------------
// Ring (per-channel FIFO with ready words in the consumer and credit words in
// the producer, both polled locally).
// ---------------------------------------------------------------------------
template <typename T>
struct RingChannel {
  const DevComm* comm;
  int c, S, next, prev;
  char* me;
  uint64_t sendT, recvT;

  __device__ char* outSlot(uint64_t t) const {
    return comm->peers[next] + ringDataAt(comm->layout, c, (int)(t % (uint64_t)S));
  }
  __device__ const T* inSlot(uint64_t t) const {
    return reinterpret_cast<const T*>(me + ringDataAt(comm->layout, c, (int)(t % (uint64_t)S)));
  }
  // Thread 0 waits; the caller passes bar.sync before using the slots.
  __device__ bool waitSend(int phase) const {
    return waitFlag(*comm, flagPtr(me, ringCreditAt(comm->layout, c, (int)(sendT % (uint64_t)S))),
                    sendT, whereCode(kCounterRing, c, phase));
  }
  __device__ bool waitRecv(int phase) const {
    return waitFlag(*comm, flagPtr(me, ringReadyAt(comm->layout, c, (int)(recvT % (uint64_t)S))),
                    recvT + 1, whereCode(kCounterRing, c, phase));
  }
  // Called by thread 0 after bar.sync.
  __device__ void publishSend() {
    stReleaseSys(flagPtr(comm->peers[next], ringReadyAt(comm->layout, c, (int)(sendT % (uint64_t)S))),
                 sendT + 1);
    ++sendT;
  }
  __device__ void releaseRecv() {
    stReleaseSys(flagPtr(comm->peers[prev], ringCreditAt(comm->layout, c, (int)(recvT % (uint64_t)S))),
                 recvT + (uint64_t)S);
    ++recvT;
  }
};

template <typename T>
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
  RingChannel<T> ch;
  ch.comm = &comm;
  ch.c = c;
  ch.S = comm.layout.ringSlots;
  ch.next = (r + 1) % P;
  ch.prev = (r + P - 1) % P;
  ch.me = comm.peers[r];
  ch.sendT = ch.recvT = comm.counters[kCounterRing * kMaxChannels + c];
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
  auto finish = [&](bool recvDone, bool sendDone) {
    __syncthreads();
    if (tid == 0) {
      if (recvDone) ch.releaseRecv();
      if (sendDone) ch.publishSend();
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
      finish(false, true);
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
      finish(true, true);
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
      finish(true, true);
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
      finish(true, true);
    }
    if (!ok) break;
    {
      const Span sp = chunkSpan(pl, tile, ringChunkBehind(r, P - 1, P), V);
      if (!acquire(true, false, 5)) break;
      T* yo = y + sp.offset;
      copyOut<T, kLdMailbox, 8>(cta, ch.inSlot(ch.recvT), sp.count, vec, false, 1.f, 1,
                                [yo](int) { return reinterpret_cast<char*>(yo); });
      finish(true, false);
    }
  }
  if (tid == 0 && !sFail) comm.counters[kCounterRing * kMaxChannels + c] = ch.sendT;
}

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

template <typename T>
__global__ void __launch_bounds__(kMaxThreads)
    ringKernel(const __grid_constant__ DevComm comm, const __grid_constant__ AllReduceArgs a) {
  ringBody<T>(comm, a, blockIdx.x);
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
      ringBody<T>(e.comm[r], e.args[r], blockIdx.x);
      break;
  }
}

template <typename T>
cudaError_t launchEmulatedTyped(const EmulatedLaunch& e, int channels, int threads,
                                cudaStream_t stream) {
  const dim3 grid((unsigned)channels, (unsigned)e.nranks);
  const dim3 block((unsigned)threads);
  void* args[] = {const_cast<EmulatedLaunch*>(&e)};
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

template <typename T, int MAXP>
cudaError_t launchTwoShot(const DevComm& comm, const AllReduceArgs& a, dim3 block,
                          cudaStream_t stream) {
  const uint32_t smem = twoShotSmemBytes(comm, MAXP);
  cudaError_t err = allowSmem<twoShotKernel<T, MAXP>>(smem);
  if (err != cudaSuccess) return err;
  twoShotKernel<T, MAXP><<<a.chunk.channels, block, smem, stream>>>(comm, a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launchTyped(const DevComm& comm, const AllReduceArgs& a, int algo, int threads,
                        cudaStream_t stream) {
  const dim3 block((unsigned)threads);
  switch (algo) {
    case TNCCL_ALGO_RING:
      ringKernel<T><<<a.chunk.channels, block, 0, stream>>>(comm, a);
      break;
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
        oneShotKernel<T, 2><<<a.block.channels, block, 0, stream>>>(comm, a);
      else if (comm.nranks <= 4)
        oneShotKernel<T, 4><<<a.block.channels, block, 0, stream>>>(comm, a);
      else if (comm.nranks <= 8)
        oneShotKernel<T, 8><<<a.block.channels, block, 0, stream>>>(comm, a);
      else
        oneShotKernel<T, 16><<<a.block.channels, block, 0, stream>>>(comm, a);
      break;
    case TNCCL_ALGO_NVLS: {
      const uint32_t smem = nvlsSmemBytes(comm);
      cudaError_t err = allowSmem<nvlsKernel<T>>(smem);
      if (err != cudaSuccess) return err;
      nvlsKernel<T><<<a.block.channels, block, smem, stream>>>(comm, a);
      break;
    }
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launchScaleTyped(const void* x, void* y, uint64_t n, float alpha, int vectorized,
                             cudaStream_t stream) {
  const uint64_t work = vectorized ? n / Pack<T>::V + 1 : n;
  unsigned blocks = (unsigned)minU64(divUp(work, 256), 148ull * 8);
  if (blocks == 0) blocks = 1;
  scaleKernel<T><<<blocks, 256, 0, stream>>>(static_cast<const T*>(x), static_cast<T*>(y), n,
                                             alpha, vectorized);
  return cudaGetLastError();
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
