// device.cuh - sm_100a device primitives: flag protocol with bounded waits,
// 16-byte vector loads/stores with explicit cache behaviour, element packing
// for fp32/bf16/fp16 with fp32 accumulation, and NVLS multimem operations.
//
// Memory-ordering protocol (tiny-nccl src/device.cuh:77-162 uses the same
// release/acquire idea with a fence in every thread): producers store
// payload with weak 16-byte stores, the CTA passes bar.sync, and then one
// thread per destination publishes a 64-bit sequence word with
// st.release.sys. bar.sync orders every thread's stores before that release
// at CTA scope and release is cumulative, so one system fence per
// destination suffices. Consumers poll their own (local) sequence word with
// ld.relaxed.sys, issue fence.acq_rel.sys once it matches, and pass
// bar.sync before any thread reads the payload. Payload reads of mailbox
// memory use ld.global.cg (L2, never a possibly stale L1 line).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "devcomm.h"

namespace tnccl {
namespace dev {

// ---------------------------------------------------------------------------
// Flags and waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t ldRelaxedSys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ldAcquireSys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void stReleaseSys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void fenceAcqRelSys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}
__device__ __forceinline__ void fenceProxyAlias() {
  asm volatile("fence.proxy.alias;" ::: "memory");
}
__device__ __forceinline__ uint64_t globalTimerNs() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Where-codes recorded on a failed wait: family, channel, phase.
__device__ __forceinline__ int whereCode(int family, int channel, int phase) {
  return (family << 24) | (channel << 8) | phase;
}

// Acquire side of a flag that was seen at or past its target: re-read it
// with ld.acquire.sys (it is monotone, so the value still satisfies the
// wait and synchronises with the release that wrote it), or, with
// acquireMode 0, a fence.acq_rel.sys after the relaxed poll.
__device__ __forceinline__ void acquireFlag(const DevComm& comm, const uint64_t* flag) {
  if (comm.acquireMode)
    (void)ldAcquireSys(flag);
  else
    fenceAcqRelSys();
}

// Debug protocol checks (-DTNCCL_DEVICE_CHECKS=1; off by default): plan
// capacities at kernel entry and exact sequence numbers on the ring's FIFO
// words. A failed check records TNCCL_SYSTEM_ERROR with this bit set in the
// where-code phase.
#ifndef TNCCL_DEVICE_CHECKS
#define TNCCL_DEVICE_CHECKS 0
#endif
constexpr int kCheckPhase = 0x80;

static __device__ __noinline__ void recordFailure(const DevComm& comm, int code, int where,
                                           uint64_t expected, uint64_t observed) {
  DevStatus* s = comm.status;
  if (s->error == 0) {
    s->where = where;
    s->expectedSeq = expected;
    s->observedSeq = observed;
    __threadfence_system();
    s->error = code;
  }
}

// Spins until *flag >= target. Every 256 polls it checks the abort word,
// an error raised elsewhere, the wall-clock bound (globaltimer) and an
// iteration bound; any of them ends the wait with false. The code TNCCL_TIMEOUT
// (5) or TNCCL_ABORTED (6) is recorded in the host-mapped status block.
static __device__ __noinline__ bool waitSlow(const DevComm& comm, const uint64_t* flag,
                                      uint64_t target, int where) {
  const uint64_t start = globalTimerNs();
  const uint64_t maxPolls = comm.timeoutNs / 16 + 4096;  // polls take >= 16 ns
  uint64_t polls = 0;
  uint64_t v = 0;
  for (;;) {
    v = ldRelaxedSys(flag);
    if (v >= target) {
      acquireFlag(comm, flag);
      return true;
    }
    ++polls;
    if ((polls & 255) == 0) {
      if (comm.status->abort) {
        recordFailure(comm, 6, where, target, v);
        return false;
      }
      if (comm.status->error) return false;
      if (globalTimerNs() - start > comm.timeoutNs || polls > maxPolls) {
        recordFailure(comm, 5, where, target, v);
        return false;
      }
    }
    if (polls > 64) __nanosleep(64);
  }
}

__device__ __forceinline__ bool waitFlag(const DevComm& comm, const uint64_t* flag,
                                         uint64_t target, int where) {
  if (ldRelaxedSys(flag) >= target) {
    acquireFlag(comm, flag);
    return true;
  }
  return waitSlow(comm, flag, target, where);
}

// Records a phase boundary of channel c (by one thread: thread 0, or the
// caller's `lead`; no-op when tracing is off). Several teams of one CTA may
// record concurrently, so the slot index is taken atomically.
__device__ __forceinline__ void traceMark(const DevComm& comm, int c, int family, int phase,
                                          uint64_t tile, bool lead) {
  if (comm.trace == nullptr || !lead) return;
  const uint32_t i = atomicAdd(comm.traceCount + c, 1u);
  uint64_t* rec = comm.trace + ((uint64_t)c * comm.traceEvents + i % comm.traceEvents) * 2;
  rec[0] = globalTimerNs();
  rec[1] = traceTag(family, phase, tile);
}

__device__ __forceinline__ void traceMark(const DevComm& comm, int c, int family, int phase,
                                          uint64_t tile) {
  traceMark(comm, c, family, phase, tile, threadIdx.x == 0);
}

// ---------------------------------------------------------------------------
// Teams: warp-aligned groups of a CTA that run different roles of one
// channel concurrently. A team synchronises on its own named barrier
// (bar.sync id, count); id 0 with the whole CTA is __syncthreads.
// ---------------------------------------------------------------------------
struct Team {
  int tid;  // thread index within the team
  int nt;   // threads in the team (multiple of 32)
  int bar;  // named barrier id
  __device__ __forceinline__ void sync() const {
    if (bar == 0)
      __syncthreads();
    else
      asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nt) : "memory");
  }
  __device__ __forceinline__ bool lead() const { return tid == 0; }
};

__device__ __forceinline__ Team wholeCta() {
  return Team{(int)threadIdx.x, (int)blockDim.x, 0};
}

// Progress counters between teams of one CTA live in shared memory: the
// producer team passes its barrier, then its leader publishes with a
// CTA-scope release; the consumer's leader polls with a CTA-scope acquire
// and then passes its own team barrier.
__device__ __forceinline__ void stReleaseCta(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.cta.shared.u64 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(p)),
               "l"(v)
               : "memory");
}
__device__ __forceinline__ unsigned long long ldAcquireCta(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.cta.shared.u64 %0, [%1];"
               : "=l"(v)
               : "r"((uint32_t)__cvta_generic_to_shared(p))
               : "memory");
  return v;
}

// Bounded wait on a shared-memory progress counter written by another team.
// Ends early (false) when `fail` (shared) is raised by any team, when an
// error or abort is recorded in the status block, or on the time/iteration
// bound (records TNCCL_TIMEOUT).
static __device__ __noinline__ bool waitLocal(const DevComm& comm, const unsigned long long* ctr,
                                              uint64_t target, const volatile int* fail,
                                              int where) {
  if (ldAcquireCta(ctr) >= target) return true;
  const uint64_t start = globalTimerNs();
  const uint64_t maxPolls = comm.timeoutNs / 16 + 4096;
  uint64_t polls = 0;
  for (;;) {
    const unsigned long long v = ldAcquireCta(ctr);
    if (v >= target) return true;
    if (*fail) return false;
    ++polls;
    if ((polls & 255) == 0) {
      if (comm.status->abort) {
        recordFailure(comm, 6, where, target, v);
        return false;
      }
      if (comm.status->error) return false;
      if (globalTimerNs() - start > comm.timeoutNs || polls > maxPolls) {
        recordFailure(comm, 5, where, target, v);
        return false;
      }
    }
    if (polls > 64) __nanosleep(32);
  }
}

// ---------------------------------------------------------------------------
// TMA bulk copies into shared memory (cp.async.bulk, completion counted in
// bytes on an mbarrier). Only this GPU's own memory is ever a source.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smemAddr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbarInit(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smemAddr(bar)), "r"(count)
               : "memory");
}
// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fenceMbarInit() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbarArriveExpectTx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smemAddr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulkLoad(void* smemDst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smemAddr(smemDst)),
      "l"(gsrc), "r"(bytes), "r"(smemAddr(bar))
      : "memory");
}
// Non-blocking probe of phase `parity` (test_wait: the thread is never
// suspended, so a completed phase is seen at once).
__device__ __forceinline__ bool mbarTryWait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smemAddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier (a TMA copy of local memory
// that never lands means a broken context; the wait still gives up).
static __device__ __noinline__ bool mbarWaitSlow(const DevComm& comm, uint64_t* bar,
                                                 uint32_t parity, int where) {
  const uint64_t start = globalTimerNs();
  for (uint64_t polls = 1;; ++polls) {
    if (mbarTryWait(bar, parity)) return true;
    if ((polls & 63) == 0 && (globalTimerNs() - start > comm.timeoutNs || polls > (1ull << 32))) {
      recordFailure(comm, 5, where, parity, 0);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbarWait(const DevComm& comm, uint64_t* bar, uint32_t parity,
                                         int where) {
  return mbarTryWait(bar, parity) || mbarWaitSlow(comm, bar, parity, where);
}
__device__ __forceinline__ uint4 ldShared16(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smemAddr(p)));
  return v;
}

// A ring of `nb` shared-memory stages, each holding `nsrc` buffers of
// `stageBytes`, filled by one leader thread with TMA bulk copies and drained
// by its team. `used` counts stages consumed so far (identical in every
// thread of the team), which gives each stage's buffer and mbarrier parity.
struct StageRing {
  char* buf;
  uint64_t* full;  // nb mbarriers (arrival count 1)
  uint32_t stageBytes;
  int nb;
  uint64_t used;
  int pieces = 1;  // bulk copies per stage and source
};

// Streams nvec 16-byte vectors of `nsrc` local sources (src(k) -> base
// address, 16-byte aligned) through the ring and calls f(i, v) with v[k] =
// vector i of source k. Stages are issued nb ahead. Per stage the leader
// waits (bounded) for the mbarrier and shares the outcome through
// `teamFlag` (shared, one per team), so the whole team leaves together if a
// stage never lands (recorded as TNCCL_TIMEOUT); after its stage the team
// passes its barrier before the leader refills the buffer.
template <int MAXSRC, typename SrcF, typename F>
__device__ __forceinline__ bool stageStream(const DevComm& comm, const Team& tm, StageRing& R,
                                            int nsrc, uint64_t nvec, SrcF src, F f, int where,
                                            volatile int* teamFlag) {
  const uint64_t vb = R.stageBytes / 16;
  const uint64_t nst = (nvec + vb - 1) / vb;
  auto issue = [&](uint64_t j) {
    const uint64_t g = R.used + j;
    const int b = (int)(g % (uint64_t)R.nb);
    const uint64_t v0 = j * vb;
    const uint32_t bytes = (uint32_t)((nvec - v0 < vb ? nvec - v0 : vb) * 16);
    mbarArriveExpectTx(R.full + b, bytes * (uint32_t)nsrc);
    const uint32_t piece = (bytes / (uint32_t)R.pieces + 15) / 16 * 16;
    for (int k = 0; k < nsrc; ++k)
      for (uint32_t o = 0; o < bytes; o += piece)
        bulkLoad(R.buf + ((size_t)b * MAXSRC + k) * R.stageBytes + o,
                 reinterpret_cast<const char*>(src(k)) + v0 * 16 + o,
                 bytes - o < piece ? bytes - o : piece, R.full + b);
  };
  if (tm.lead())
    for (uint64_t j = 0; j < nst && j < (uint64_t)R.nb; ++j) issue(j);
  bool ok = true;
  for (uint64_t j = 0; j < nst; ++j) {
    const uint64_t g = R.used + j;
    const int b = (int)(g % (uint64_t)R.nb);
    const uint32_t parity = (uint32_t)((g / (uint64_t)R.nb) & 1);
    if (tm.lead()) *teamFlag = mbarWait(comm, R.full + b, parity, where) ? 0 : 1;
    tm.sync();
    if (*teamFlag) {
      ok = false;
      break;
    }
    (void)mbarTryWait(R.full + b, parity);  // completed: acquire in this thread
    const uint64_t v0 = j * vb;
    const uint32_t nv = (uint32_t)(nvec - v0 < vb ? nvec - v0 : vb);
    const char* base = R.buf + (size_t)b * MAXSRC * R.stageBytes;
    for (uint32_t i = tm.tid; i < nv; i += tm.nt) {
      uint4 v[MAXSRC];
#pragma unroll
      for (int k = 0; k < MAXSRC; ++k)
        if (k < nsrc) v[k] = ldShared16(base + (size_t)k * R.stageBytes + (size_t)i * 16);
      f(v0 + i, v);
    }
    tm.sync();
    if (tm.lead() && j + R.nb < nst) issue(j + R.nb);
  }
  R.used += nst;
  return ok;
}

__device__ __forceinline__ uint64_t* flagPtr(char* base, uint64_t off) {
  return reinterpret_cast<uint64_t*>(base + off);
}

// ---------------------------------------------------------------------------
// 16-byte accesses
// ---------------------------------------------------------------------------
// User input: streamed once (evict-first).
__device__ __forceinline__ uint4 ldInput(const void* p) {
  uint4 v;
  asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
// Mailbox payload written by peers: read at L2.
__device__ __forceinline__ uint4 ldMailbox(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st16(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------------------
// Element packing: a 16-byte pack holds V elements of T.
// ---------------------------------------------------------------------------
template <typename T>
struct Pack;

template <>
struct Pack<float> {
  static constexpr int V = 4;
  __device__ __forceinline__ static void unpack(uint4 v, float (&f)[V]) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[V]) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static float toF(float x) { return x; }
  __device__ __forceinline__ static float fromF(float x) { return x; }
};

template <>
struct Pack<__nv_bfloat16> {
  static constexpr int V = 8;
  __device__ __forceinline__ static float2 u2f(uint32_t u) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(h);
  }
  __device__ __forceinline__ static uint32_t f2u(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static void unpack(uint4 v, float (&f)[V]) {
    float2 a = u2f(v.x), b = u2f(v.y), c = u2f(v.z), d = u2f(v.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[V]) {
    return make_uint4(f2u(f[0], f[1]), f2u(f[2], f[3]), f2u(f[4], f[5]), f2u(f[6], f[7]));
  }
  __device__ __forceinline__ static float toF(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 fromF(float x) { return __float2bfloat16_rn(x); }
};

template <>
struct Pack<__half> {
  static constexpr int V = 8;
  __device__ __forceinline__ static float2 u2f(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
  }
  __device__ __forceinline__ static uint32_t f2u(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static void unpack(uint4 v, float (&f)[V]) {
    float2 a = u2f(v.x), b = u2f(v.y), c = u2f(v.z), d = u2f(v.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[V]) {
    return make_uint4(f2u(f[0], f[1]), f2u(f[2], f[3]), f2u(f[4], f[5]), f2u(f[6], f[7]));
  }
  __device__ __forceinline__ static float toF(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half fromF(float x) { return __float2half_rn(x); }
};

// acc = alpha * x, rounded (no FMA contraction: the CPU oracle computes the
// same two roundings).
__device__ __forceinline__ float scaled(float alpha, float x) { return __fmul_rn(alpha, x); }
__device__ __forceinline__ float addRn(float a, float b) { return __fadd_rn(a, b); }

// ---------------------------------------------------------------------------
// NVLS multimem (NVSwitch reduce / multicast)
// ---------------------------------------------------------------------------
// Adds v to a 64-bit counter on every GPU of the multicast object, with
// release semantics (orders this thread's earlier accesses, and those it
// observed through bar.sync, before the add on every copy).
__device__ __forceinline__ void multimemAddRelease(uint64_t* mc, uint64_t v) {
  asm volatile("multimem.red.release.sys.global.add.u64 [%0], %1;" ::"l"(mc), "l"(v) : "memory");
}

template <typename T>
struct Multimem;

template <>
struct Multimem<float> {
  __device__ __forceinline__ static uint4 ldReduce(const void* mc) {
    uint4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(mc)
                 : "memory");
    return v;
  }
  __device__ __forceinline__ static void st(void* mc, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  }
};

template <>
struct Multimem<__nv_bfloat16> {
  __device__ __forceinline__ static uint4 ldReduce(const void* mc) {
    uint4 v;
    asm volatile(
        "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(mc)
        : "memory");
    return v;
  }
  __device__ __forceinline__ static void st(void* mc, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  }
};

template <>
struct Multimem<__half> {
  __device__ __forceinline__ static uint4 ldReduce(const void* mc) {
    uint4 v;
    asm volatile(
        "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(mc)
        : "memory");
    return v;
  }
  __device__ __forceinline__ static void st(void* mc, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
  }
};

}  // namespace dev
}  // namespace tnccl
