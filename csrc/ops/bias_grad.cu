// bias_grad.cu - bias gradients of the GPT-2 linear layers, optionally fused
// with the tanh-GELU backward that precedes them.
//
//   tnops_bias_grad:     db[n] = sum_m g[m, n]                   (g bf16, db fp32)
//   tnops_gelu_bwd_bias: gp[m, n] = bf16(gy[m, n] * gelu'(pre[m, n]))
//                        db[n]    = sum_m gp[m, n]
//
// Column sums of an [M, N] row-major bf16 matrix, deterministic: pass 1
// tiles the matrix into (256-column, rowsPer-row) blocks; each warp of a CTA
// owns 256 columns (8 per lane, one 16-byte load per row) and every 8th row
// of the block, 4 rows in flight; the 8 warp sums are added in warp order
// into one fp32 partial per block. Pass 2 adds the partials of a column in
// block order (colReduce, common.cuh). The summation order depends only on
// (M, N), never on scheduling. Rounding of the GELU gradient to bf16 happens before it is
// summed, as when the gradient tensor is materialised and then reduced.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "tnccl_ops.h"

namespace tnops {
namespace {

constexpr int kCols = 256;  // columns per CTA (8 per lane x 32 lanes)
constexpr int kWarps = 8;
constexpr int kUnroll = 4;  // rows in flight per warp

__device__ __forceinline__ void bf16x8ToF(uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Derivative of the tanh approximation of GELU, 0.5 x (1 + tanh(u)) with
// u = k0 (x + k1 x^3), from the product rule:
//   0.5 (1 + t) + 0.5 x (1 - t^2) u',  t = tanh(u),  u' = k0 + 3 k0 k1 x^2.
// With e = e^(-2u) and r = 1 / (1 + e): 0.5 (1 + t) = r and
// 1 - t^2 = 4 r (1 - r) = 4 r (e r), so the derivative is
// r + 2 x r (e r) u': one ex2 and one fast division, and 1 - t^2 comes from
// e r directly, never from 1 - t*t (which cancels where |t| is near 1).
__device__ __forceinline__ float ex2Approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float geluTanhGrad(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
  const float k0k1 = 0.7978845608028654f * 0.044715f;
  const float m2log2e = -2.0f * 1.4426950408889634f;
  const float x2 = x * x;
  // |u| <= 40 keeps e and r finite (e^80 < FLT_MAX); the derivative is 0 or
  // 1 to float precision well before that.
  const float u = fminf(fmaxf(x * fmaf(k0k1, x2, k0), -40.0f), 40.0f);
  const float e = ex2Approx(u * m2log2e);
  const float r = __fdividef(1.0f, 1.0f + e);
  const float du = fmaf(3.0f * k0k1, x2, k0);
  return fmaf(2.0f * x * r * (e * r), du, r);
}

template <bool GELU>
__global__ void __launch_bounds__(kWarps * 32)
    colsumPartial(const uint16_t* __restrict__ gy, const uint16_t* __restrict__ pre,
                  uint16_t* __restrict__ gout, float* __restrict__ partial, int M, int N,
                  int rowsPer) {
  __shared__ float sAcc[kWarps][kCols];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int col0 = blockIdx.x * kCols + lane * 8;
  const int r0 = blockIdx.y * rowsPer;
  const int r1 = min(M, r0 + rowsPer);
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  if (col0 < N) {
    for (int rb = r0 + w; rb < r1; rb += kWarps * kUnroll) {
      uint4 g[kUnroll], p[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int r = rb + u * kWarps;
        if (r < r1) {
          const size_t off = (size_t)r * N + col0;
          g[u] = __ldcs(reinterpret_cast<const uint4*>(gy + off));
          if (GELU) p[u] = __ldcs(reinterpret_cast<const uint4*>(pre + off));
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int r = rb + u * kWarps;
        if (r >= r1) continue;
        float f[8];
        bf16x8ToF(g[u], f);
        if (GELU) {
          float x[8];
          bf16x8ToF(p[u], x);
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint16_t lo = f2bf(f[2 * i] * geluTanhGrad(x[2 * i]));
            const uint16_t hi = f2bf(f[2 * i + 1] * geluTanhGrad(x[2 * i + 1]));
            o[i] = (uint32_t)lo | ((uint32_t)hi << 16);
            f[2 * i] = bf2f(lo);
            f[2 * i + 1] = bf2f(hi);
          }
          *reinterpret_cast<uint4*>(gout + (size_t)r * N + col0) = make_uint4(o[0], o[1], o[2], o[3]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += f[e];
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) sAcc[w][lane * 8 + e] = acc[e];
  __syncthreads();
  const int c = blockIdx.x * kCols + threadIdx.x;
  if (c < N) {
    float s = sAcc[0][threadIdx.x];
#pragma unroll
    for (int k = 1; k < kWarps; ++k) s += sAcc[k][threadIdx.x];
    partial[(size_t)blockIdx.y * N + c] = s;
  }
}

}  // namespace
}  // namespace tnops

using namespace tnops;

// Row blocks: enough CTAs for ~8 per SM, at least 32 rows each.
extern "C" int tnops_colsum_parts(int M, int N) {
  const int colBlocks = (N + kCols - 1) / kCols;
  int parts = (kSMs * 8 + colBlocks - 1) / colBlocks;
  const int maxParts = M / 32 > 0 ? M / 32 : 1;
  return parts < 1 ? 1 : parts > maxParts ? maxParts : parts;
}

static int launchColsum(const uint16_t* gy, const uint16_t* pre, uint16_t* gout, float* db,
                        float* partial, int M, int N, bool gelu, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || N % 8 != 0) return 1;
  // 16-byte pieces of every row: N % 8 == 0 keeps the rows on the boundary
  // when the base pointers are.
  if ((reinterpret_cast<uintptr_t>(gy) | reinterpret_cast<uintptr_t>(pre) |
       reinterpret_cast<uintptr_t>(gout)) & 15)
    return 1;
  const int parts = tnops_colsum_parts(M, N);
  const int rowsPer = (M + parts - 1) / parts;
  const dim3 grid((unsigned)((N + kCols - 1) / kCols), (unsigned)parts);
  if (gelu)
    colsumPartial<true><<<grid, kWarps * 32, 0, stream>>>(gy, pre, gout, partial, M, N, rowsPer);
  else
    colsumPartial<false><<<grid, kWarps * 32, 0, stream>>>(gy, pre, gout, partial, M, N, rowsPer);
  colReduce<<<(N + 31) / 32, kColReduceWarps * 32, 0, stream>>>(partial, parts, N, N, N, db,
                                                                 nullptr);
  gLaunches.fetch_add(2, std::memory_order_relaxed);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// partial: tnops_colsum_parts(M, N) * N floats of scratch.
extern "C" int tnops_bias_grad(const uint16_t* g, float* db, float* partial, int M, int N,
                               cudaStream_t stream) {
  return launchColsum(g, nullptr, nullptr, db, partial, M, N, false, stream);
}

extern "C" int tnops_gelu_bwd_bias(const uint16_t* gy, const uint16_t* pre, uint16_t* gpre,
                                   float* db, float* partial, int M, int N, cudaStream_t stream) {
  return launchColsum(gy, pre, gpre, db, partial, M, N, true, stream);
}
