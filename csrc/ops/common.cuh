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

// Second pass of the deterministic column sums (bias gradients, LayerNorm
// dweight / dbias): out[c] = sum over p of in[p * ld + c] for c < ncols,
// written to out0[c] for c < split and to out1[c - split] above. A CTA of 32
// warps owns 32 columns; warp w adds rows w, w + 32, w + 64, ... in row order
// (eight independent loads in flight), then warp 0 adds the 32 warp sums in
// warp order. The order depends only on nparts, never on scheduling, and the
// short per-warp chains keep the pass from being latency-bound (a partial
// count of 100-300 rows is common).
constexpr int kColReduceWarps = 32;
namespace {  // one copy per translation unit
__global__ void __launch_bounds__(kColReduceWarps * 32)
    colReduce(const float* __restrict__ in, int nparts, int ld, int ncols, int split,
              float* __restrict__ out0, float* __restrict__ out1) {
  __shared__ float s[kColReduceWarps][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float acc = 0.f;
  if (col < ncols) {
    int p = warp;
    constexpr int U = 8;
    for (; p + (U - 1) * kColReduceWarps < nparts; p += U * kColReduceWarps) {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = in[(size_t)(p + u * kColReduceWarps) * ld + col];
#pragma unroll
      for (int u = 0; u < U; ++u) acc += v[u];
    }
    for (; p < nparts; p += kColReduceWarps) acc += in[(size_t)p * ld + col];
  }
  s[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && col < ncols) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kColReduceWarps; ++w) t += s[w][lane];
    if (col < split)
      out0[col] = t;
    else
      out1[col - split] = t;
  }
}
}  // namespace

}  // namespace tnops
