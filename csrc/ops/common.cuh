// common.cuh - helpers shared by the model kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace tnops {

extern std::atomic<unsigned long long> gLaunches;

inline int launched(cudaError_t e) {
  if (e == cudaSuccess) gLaunches.fetch_add(1, std::memory_order_relaxed);
  return (int)e;
}

__device__ __forceinline__ float bf2f(uint16_t u) {
  return __uint_as_float((uint32_t)u << 16);
}
__device__ __forceinline__ uint16_t f2bf(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}
// 4 bf16 in a uint2 <-> float4
__device__ __forceinline__ float4 bf4(uint2 u) {
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}
__device__ __forceinline__ uint2 tobf4(float4 f) {
  return make_uint2((uint32_t)f2bf(f.x) | ((uint32_t)f2bf(f.y) << 16),
                    (uint32_t)f2bf(f.z) | ((uint32_t)f2bf(f.w) << 16));
}

__device__ __forceinline__ float warpSum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warpMax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

constexpr int kSMs = 148;

}  // namespace tnops
