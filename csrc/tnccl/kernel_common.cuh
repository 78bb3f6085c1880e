// kernel_common.cuh - building blocks of the all-reduce kernels (included
// once, by allreduce.cu): launch constants, shared-memory sizes of the staged
// teams, 16-byte and scalar element access, the fused copy / P-way reduce /
// ring-hop loops over a team's threads, the multi-source TMA-staged copy and
// the warp split of warp-specialised CTAs.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "device.cuh"
#include "protocol.h"

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

// Debug builds (-DTNCCL_DEVICE_CHECKS=1) check every launch's plan against the
// mailbox capacities at kernel entry: a chunk or tile must fit its slot and
// the channel must be provisioned. On failure thread 0 records
// TNCCL_SYSTEM_ERROR with the check bit in the where-code phase
// (kCheckPhase; expected = capacity, observed = need) and every thread of the
// CTA returns; the other CTAs' waits see the error. Release builds compile
// the check away.
__device__ __forceinline__ bool planFits(const DevComm& comm, uint64_t needBytes,
                                         uint64_t slotBytes, int channel, int channels,
                                         int family) {
#if TNCCL_DEVICE_CHECKS
  if (needBytes <= slotBytes && channel < channels) return true;
  if (threadIdx.x == 0)
    recordFailure(comm, 3, whereCode(family, channel, kCheckPhase), slotBytes, needBytes);
  return false;
#else
  return true;
#endif
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

}  // namespace
}  // namespace tnccl
