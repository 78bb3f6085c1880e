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
      fenceAcqRelSys();
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
    fenceAcqRelSys();
    return true;
  }
  return waitSlow(comm, flag, target, where);
}

// Records a phase boundary of channel c (thread 0 only; no-op when tracing
// is off).
__device__ __forceinline__ void traceMark(const DevComm& comm, int c, int family, int phase,
                                          uint64_t tile) {
  if (comm.trace == nullptr || threadIdx.x != 0) return;
  const uint32_t i = comm.traceCount[c]++;
  uint64_t* rec = comm.trace + ((uint64_t)c * comm.traceEvents + i % comm.traceEvents) * 2;
  rec[0] = globalTimerNs();
  rec[1] = traceTag(family, phase, tile);
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
