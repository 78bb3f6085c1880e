// layernorm.cu - fused residual add + LayerNorm (forward and backward) for a
// fp32 residual stream with bf16 activations, one warp per row.
//
// Forward:  x_out = x + delta;  y = (x_out - mean) * rstd * w + b   (bf16)
// Backward: with xhat = (x_out - mean) * rstd and gw = gy * w,
//           dx = g_res + rstd * (gw - mean(gw) - xhat * mean(gw * xhat))
//           dw = sum_rows gy * xhat,  db = sum_rows gy
// dw/db are reduced deterministically: each CTA keeps per-thread column sums,
// combines them in shared memory and writes one partial row; a second kernel
// sums the partial rows in a fixed order. The backward has two kernels: the
// default gives each row to a group of threads with one float4 column group
// per thread (several rows per CTA, cp.async prefetch two rows ahead); the
// other gives each row to one warp (TNOPS_LN_BWD=warp, kept for A/B timing).
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "ln_plan.h"
#include "tnccl_ops.h"

namespace tnops {
namespace {

constexpr int kWarpsPerBlock = 8;
constexpr int kPartialRows = 2 * kSMs;

// K = float4 groups per lane (C <= 128 * K).
template <int K>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    lnFwdKernel(const float* __restrict__ x, const uint16_t* __restrict__ delta,
                const float* __restrict__ w, const float* __restrict__ b, float* __restrict__ xo,
                uint16_t* __restrict__ y, float* __restrict__ mean, float* __restrict__ rstd,
                int rows, int C, float eps) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int C4 = C >> 2;
  const size_t base = (size_t)row * C;
  const float4* xr = reinterpret_cast<const float4*>(x + base);
  float4 v[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = lane + 32 * k;
    if (i < C4) v[k] = xr[i];
  }
  if (delta != nullptr) {
    const uint2* dr = reinterpret_cast<const uint2*>(delta + base);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int i = lane + 32 * k;
      if (i < C4) {
        const float4 d = bf4(dr[i]);
        v[k].x += d.x;
        v[k].y += d.y;
        v[k].z += d.z;
        v[k].w += d.w;
      }
    }
  }
  float s = 0.f;
  float4* xor_ = reinterpret_cast<float4*>(xo + base);
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = lane + 32 * k;
    if (i < C4) {
      xor_[i] = v[k];
      s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
  }
  const float mu = warpSum(s) / (float)C;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = lane + 32 * k;
    if (i < C4) {
      const float a = v[k].x - mu, bb = v[k].y - mu, c = v[k].z - mu, d = v[k].w - mu;
      q += (a * a + bb * bb) + (c * c + d * d);
    }
  }
  const float rs = rsqrtf(warpSum(q) / (float)C + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  uint2* yr = reinterpret_cast<uint2*>(y + base);
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = lane + 32 * k;
    if (i < C4) {
      const float4 ww = w4[i], bb = b4[i];
      float4 o;
      o.x = (v[k].x - mu) * rs * ww.x + bb.x;
      o.y = (v[k].y - mu) * rs * ww.y + bb.y;
      o.z = (v[k].z - mu) * rs * ww.z + bb.z;
      o.w = (v[k].w - mu) * rs * ww.w + bb.w;
      yr[i] = tobf4(o);
    }
  }
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
}

// One warp per row. Every load of a row (gy, x_out, the residual gradient)
// is issued before any of it is used; the per-column dw / db accumulators of
// each warp live in shared memory (one row of C floats per warp and
// quantity), which leaves the registers to the loads in flight. Summation
// order per column: the rows of each warp in row order, then the 8 warps in
// warp order (here), then the CTAs in order (colReduce, common.cuh).
template <int K>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, 2)
    lnBwdKernel(const uint16_t* __restrict__ gy, const float* __restrict__ gres,
                const float* __restrict__ xo, const float* __restrict__ w,
                const float* __restrict__ mean, const float* __restrict__ rstd,
                float* __restrict__ dx, uint16_t* __restrict__ dxb, float* __restrict__ partial,
                int rows, int C) {
  extern __shared__ __align__(16) float sAcc[];  // [dw | db][warp][C]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int C4 = C >> 2;
  const float invC = 1.0f / (float)C;
  float4* myDw = reinterpret_cast<float4*>(sAcc + (size_t)warp * C);
  float4* myDb = reinterpret_cast<float4*>(sAcc + (size_t)(kWarpsPerBlock + warp) * C);
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = lane + 32 * k;
    if (i < C4) {
      myDw[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      myDb[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const int stride = gridDim.x * kWarpsPerBlock;
  for (int row = blockIdx.x * kWarpsPerBlock + warp; row < rows; row += stride) {
    const size_t base = (size_t)row * C;
    const float mu = mean[row], rs = rstd[row];
    const uint2* gr = reinterpret_cast<const uint2*>(gy + base);
    const float4* xr = reinterpret_cast<const float4*>(xo + base);
    const float4* rr = gres ? reinterpret_cast<const float4*>(gres + base) : nullptr;
    uint2 graw[K];
    float4 xv[K], res[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int i = lane + 32 * k;
      if (i < C4) {
        graw[k] = __ldcs(gr + i);
        xv[k] = __ldcs(xr + i);
        res[k] = rr ? __ldcs(rr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float4 g[K], xh[K];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int i = lane + 32 * k;
      if (i < C4) {
        g[k] = bf4(graw[k]);
        xh[k] = make_float4((xv[k].x - mu) * rs, (xv[k].y - mu) * rs, (xv[k].z - mu) * rs,
                            (xv[k].w - mu) * rs);
        const float4 ww = w4[i];
        const float4 gw = make_float4(g[k].x * ww.x, g[k].y * ww.y, g[k].z * ww.z, g[k].w * ww.w);
        s1 += (gw.x + gw.y) + (gw.z + gw.w);
        s2 += (gw.x * xh[k].x + gw.y * xh[k].y) + (gw.z * xh[k].z + gw.w * xh[k].w);
        float4 a = myDw[i], d = myDb[i];
        a.x += g[k].x * xh[k].x;
        a.y += g[k].y * xh[k].y;
        a.z += g[k].z * xh[k].z;
        a.w += g[k].w * xh[k].w;
        d.x += g[k].x;
        d.y += g[k].y;
        d.z += g[k].z;
        d.w += g[k].w;
        myDw[i] = a;
        myDb[i] = d;
      }
    }
    const float m1 = warpSum(s1) * invC, m2 = warpSum(s2) * invC;
    float4* dr = reinterpret_cast<float4*>(dx + base);
    uint2* dbr = dxb ? reinterpret_cast<uint2*>(dxb + base) : nullptr;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int i = lane + 32 * k;
      if (i < C4) {
        const float4 ww = w4[i];
        float4 o;
        o.x = rs * (g[k].x * ww.x - m1 - xh[k].x * m2) + res[k].x;
        o.y = rs * (g[k].y * ww.y - m1 - xh[k].y * m2) + res[k].y;
        o.z = rs * (g[k].z * ww.z - m1 - xh[k].z * m2) + res[k].z;
        o.w = rs * (g[k].w * ww.w - m1 - xh[k].w * m2) + res[k].w;
        dr[i] = o;
        if (dbr) dbr[i] = tobf4(o);
      }
    }
  }
  // Combine the warps of this CTA into one partial row of [dw | db].
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) {
    const int q = c / C, col = c - q * C;
    const float* src = sAcc + (size_t)q * kWarpsPerBlock * C + col;
    float a = 0.f;
#pragma unroll
    for (int wv = 0; wv < kWarpsPerBlock; ++wv) a += src[(size_t)wv * C];
    partial[(size_t)blockIdx.x * 2 * C + c] = a;
  }
}

// ---------------------------------------------------------------------------
// Row-group backward (the default). A group of G threads owns one row at a
// time; each thread owns K consecutive float4 column groups (4K columns:
// K = 2 when C % 8 == 0 and the bf16 rows are 16-byte aligned, else 1), so
// G = 32 * ceil(C / (128 K)). A CTA of R groups runs one per SM and walks
// rows blockIdx.x * R + g, + gridDim.x * R, ... Against one warp per row this
// gives each SM 24-30 warps instead of 8-16 to hide latency, and every
// thread carries a few registers of state instead of a whole row slice;
// K = 2 halves the per-row bookkeeping (row sums, barrier, addressing) per
// column against K = 1, which issue-bound the kernel.
//
// Each thread prefetches its own bytes of the next kGroupStages - 1 rows
// (gy 8K B, x_out and residual gradient 16K B each) into a per-group ring
// of shared-memory stages with cp.async; a thread only ever reads what it
// copied itself, so the copies need no barrier, only cp.async.wait_group.
// The two row sums (of gy * w and of gy * w * xhat) go through one named
// barrier per row and group: warp sums are written to a slot double-
// buffered by row parity, so the next row's writes cannot overwrite values
// another warp is still reading. Summation order per column: each group's
// rows in row order, the groups in group order (here), then the CTAs in
// order (colReduce). Launch geometry and shared-memory layout: ln_plan.h.
// ---------------------------------------------------------------------------
constexpr int kGroupStages = kLnStages;
constexpr int kGroupRedFloats = kLnRedFloats;

__device__ __forceinline__ void cpAsync16(void* dst, const void* src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(src) : "memory");
}
__device__ __forceinline__ void cpAsync8(void* dst, const void* src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(src) : "memory");
}
__device__ __forceinline__ void cpAsyncCommit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cpAsyncWait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void namedBarrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}

template <int K>
__global__ void __launch_bounds__(lnMaxThreads(K), 1)
    lnBwdGroupKernel(const uint16_t* __restrict__ gy, const float* __restrict__ gres,
                     const float* __restrict__ xo, const float* __restrict__ w,
                     const float* __restrict__ mean, const float* __restrict__ rstd,
                     float* __restrict__ dx, uint16_t* __restrict__ dxb,
                     float* __restrict__ partial, int rows, int C, int G, int R) {
  extern __shared__ __align__(16) float sGroup[];
  const int t = threadIdx.x;
  const int grp = t / G;
  const int gt = t - grp * G;  // this thread owns float4 groups K*gt .. K*gt+K-1
  const int lane = t & 31, gwarp = gt >> 5, nwarps = G >> 5;
  const bool act = gt < (C >> 2) / K;
  const float invC = 1.0f / (float)C;
  const int stageBytes = lnStageBytes(K, G);
  char* ring = reinterpret_cast<char*>(sGroup + kGroupRedFloats) +
               (size_t)grp * kGroupStages * stageBytes;
  char* myG = ring + 8 * K * gt;  // + stage * stageBytes
  char* myX = ring + 8 * K * G + 16 * K * gt;
  char* myR = ring + 24 * K * G + 16 * K * gt;
  const int col = 4 * K * gt;     // first column of this thread

  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 wv[K], aw[K], ab[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    wv[k] = act ? reinterpret_cast<const float4*>(w + col)[k] : zero;
    aw[k] = zero;
    ab[k] = zero;
  }
  const int stride = gridDim.x * R;
  const int first = blockIdx.x * R + grp;

  auto issue = [&](int stage, int row) {
    const size_t base = (size_t)row * C + col;
    const int off = stage * stageBytes;
    if (K == 2) {
      cpAsync16(myG + off, gy + base);
    } else {
      cpAsync8(myG + off, gy + base);
    }
#pragma unroll
    for (int k = 0; k < K; ++k) cpAsync16(myX + off + 16 * k, xo + base + 4 * k);
    if (gres) {
#pragma unroll
      for (int k = 0; k < K; ++k) cpAsync16(myR + off + 16 * k, gres + base + 4 * k);
    }
  };
#pragma unroll
  for (int j = 0; j < kGroupStages - 1; ++j) {
    const int row = first + j * stride;
    if (act && row < rows) issue(j, row);
    cpAsyncCommit();
  }
  float mu = 0.f, rs = 0.f;
  if (first < rows) {
    mu = mean[first];
    rs = rstd[first];
  }
  int slot = 0, parity = 0;
  for (int row = first; row < rows; row += stride) {
    const int next = row + stride;
    float nmu = 0.f, nrs = 0.f;
    if (next < rows) {
      nmu = mean[next];
      nrs = rstd[next];
    }
    const int ahead = row + (kGroupStages - 1) * stride;
    if (act && ahead < rows) issue(slot == 0 ? kGroupStages - 1 : slot - 1, ahead);
    cpAsyncCommit();
    cpAsyncWait<kGroupStages - 1>();  // this thread's copies of `row` have landed

    float4 g[K], xh[K], res[K];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      g[k] = zero;
      xh[k] = zero;
      res[k] = zero;
      if (act) {
        const int off = slot * stageBytes;
        g[k] = bf4(reinterpret_cast<const uint2*>(myG + off)[k]);
        const float4 xv = reinterpret_cast<const float4*>(myX + off)[k];
        if (gres) res[k] = reinterpret_cast<const float4*>(myR + off)[k];
        xh[k] = make_float4((xv.x - mu) * rs, (xv.y - mu) * rs, (xv.z - mu) * rs,
                            (xv.w - mu) * rs);
      }
      // g becomes gy * w from here on; the dW / dB sums use gy itself.
      aw[k].x += g[k].x * xh[k].x;
      aw[k].y += g[k].y * xh[k].y;
      aw[k].z += g[k].z * xh[k].z;
      aw[k].w += g[k].w * xh[k].w;
      ab[k].x += g[k].x;
      ab[k].y += g[k].y;
      ab[k].z += g[k].z;
      ab[k].w += g[k].w;
      g[k] = make_float4(g[k].x * wv[k].x, g[k].y * wv[k].y, g[k].z * wv[k].z, g[k].w * wv[k].w);
      s1 += (g[k].x + g[k].y) + (g[k].z + g[k].w);
      s2 += (g[k].x * xh[k].x + g[k].y * xh[k].y) + (g[k].z * xh[k].z + g[k].w * xh[k].w);
    }
    s1 = warpSum(s1);
    s2 = warpSum(s2);
    float2* red = reinterpret_cast<float2*>(sGroup) + (grp * 2 + parity) * kLnMaxWarpsPerGroup;
    if (lane == 0) red[gwarp] = make_float2(s1, s2);
    namedBarrier(1 + grp, G);
    float t1 = 0.f, t2 = 0.f;
#pragma unroll
    for (int k = 0; k < kLnMaxWarpsPerGroup; ++k) {
      if (k < nwarps) {
        const float2 v = red[k];
        t1 += v.x;
        t2 += v.y;
      }
    }
    const float m1 = t1 * invC, m2 = t2 * invC;
    if (act) {
      const size_t base = (size_t)row * C + col;
      float4 o[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        o[k].x = rs * (g[k].x - m1 - xh[k].x * m2) + res[k].x;
        o[k].y = rs * (g[k].y - m1 - xh[k].y * m2) + res[k].y;
        o[k].z = rs * (g[k].z - m1 - xh[k].z * m2) + res[k].z;
        o[k].w = rs * (g[k].w - m1 - xh[k].w * m2) + res[k].w;
        reinterpret_cast<float4*>(dx + base)[k] = o[k];
      }
      if (dxb) {
        if (K == 2) {
          const uint2 lo = tobf4(o[0]), hi = tobf4(o[K - 1]);
          *reinterpret_cast<uint4*>(dxb + base) = make_uint4(lo.x, lo.y, hi.x, hi.y);
        } else {
          *reinterpret_cast<uint2*>(dxb + base) = tobf4(o[0]);
        }
      }
    }
    mu = nmu;
    rs = nrs;
    parity ^= 1;
    slot = slot + 1 == kGroupStages ? 0 : slot + 1;
  }
  cpAsyncWait<0>();
  // Combine the groups of this CTA into one partial row of [dw | db]; the
  // accumulators reuse the stage memory (R * 2C floats <= R * 3 * 40 K G bytes).
  __syncthreads();
  float* acc = sGroup + kGroupRedFloats;
  if (act) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      reinterpret_cast<float4*>(acc + (size_t)grp * 2 * C + col)[k] = aw[k];
      reinterpret_cast<float4*>(acc + (size_t)grp * 2 * C + C + col)[k] = ab[k];
    }
  }
  __syncthreads();
  for (int c = t; c < 2 * C; c += blockDim.x) {
    float a = 0.f;
    for (int q = 0; q < R; ++q) a += acc[(size_t)q * 2 * C + c];
    partial[(size_t)blockIdx.x * 2 * C + c] = a;
  }
}

template <int K>
cudaError_t fwdK(const float* x, const uint16_t* d, const float* w, const float* b, float* xo,
                 uint16_t* y, float* m, float* r, int rows, int C, float eps, cudaStream_t st) {
  const int blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  lnFwdKernel<K><<<blocks, kWarpsPerBlock * 32, 0, st>>>(x, d, w, b, xo, y, m, r, rows, C, eps);
  return cudaGetLastError();
}

template <int K>
cudaError_t bwdK(const uint16_t* gy, const float* gres, const float* xo, const float* w,
                 const float* m, const float* r, float* dx, uint16_t* dxb, float* partial,
                 int rows, int C, cudaStream_t st) {
  int blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (blocks > kPartialRows) blocks = kPartialRows;
  const int smem = 2 * kWarpsPerBlock * C * (int)sizeof(float);  // dw and db rows per warp
  // Opt in to the shared memory once per device (bit d of `done`).
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (!(done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(lnBwdKernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             2 * kWarpsPerBlock * 128 * K * (int)sizeof(float));
    if (e != cudaSuccess) return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  lnBwdKernel<K><<<blocks, kWarpsPerBlock * 32, smem, st>>>(gy, gres, xo, w, m, r, dx, dxb,
                                                           partial, rows, C);
  return cudaGetLastError();
}

// Launches lnBwdGroupKernel<K>; *nparts = the partial rows it writes (<= kSMs).
template <int K>
cudaError_t bwdGroup(const uint16_t* gy, const float* gres, const float* xo, const float* w,
                     const float* m, const float* r, float* dx, uint16_t* dxb, float* partial,
                     int rows, int C, int* nparts, cudaStream_t st) {
  const LnGroupPlan plan = lnGroupPlan(rows, C, K, kSMs);
  *nparts = plan.blocks;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (!(done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(lnBwdGroupKernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kLnMaxSmemBytes);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  lnBwdGroupKernel<K><<<plan.blocks, plan.R * plan.G, plan.smemBytes, st>>>(
      gy, gres, xo, w, m, r, dx, dxb, partial, rows, C, plan.G, plan.R);
  return cudaGetLastError();
}

// TNOPS_LN_BWD=warp selects the one-warp-per-row kernel for every shape (A/B
// timing); by default the row-group kernel takes every aligned input.
bool groupEnabled() {
  static const bool on = [] {
    const char* v = getenv("TNOPS_LN_BWD");
    return v == nullptr || strcmp(v, "warp") != 0;
  }();
  return on;
}

}  // namespace
}  // namespace tnops

using namespace tnops;

extern "C" int tnops_ln_partial_rows(void) { return kPartialRows; }

extern "C" int tnops_ln_fwd(const float* x, const uint16_t* delta, const float* w, const float* b,
                            float* x_out, uint16_t* y, float* mean, float* rstd, int rows, int C,
                            float eps, cudaStream_t stream) {
  if (C % 4 != 0 || C > 128 * 16 || rows <= 0) return (int)cudaErrorInvalidValue;
  // 16-byte pieces of the fp32 rows and parameters, 8-byte pieces of the bf16
  // rows (C % 4 == 0 keeps every row on those boundaries).
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(x_out) |
        reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(b)) & 15) ||
      ((reinterpret_cast<uintptr_t>(delta) | reinterpret_cast<uintptr_t>(y)) & 7))
    return (int)cudaErrorInvalidValue;
  const int K = (C + 127) / 128;
  cudaError_t e;
  switch (K) {
    case 1: e = fwdK<1>(x, delta, w, b, x_out, y, mean, rstd, rows, C, eps, stream); break;
    case 2: e = fwdK<2>(x, delta, w, b, x_out, y, mean, rstd, rows, C, eps, stream); break;
    case 4: case 3: e = fwdK<4>(x, delta, w, b, x_out, y, mean, rstd, rows, C, eps, stream); break;
    case 5: case 6: e = fwdK<6>(x, delta, w, b, x_out, y, mean, rstd, rows, C, eps, stream); break;
    case 7: case 8: e = fwdK<8>(x, delta, w, b, x_out, y, mean, rstd, rows, C, eps, stream); break;
    default: e = fwdK<16>(x, delta, w, b, x_out, y, mean, rstd, rows, C, eps, stream); break;
  }
  return launched(e);
}

extern "C" int tnops_ln_bwd(const uint16_t* gy, const float* g_res, const float* x_out,
                            const float* w, const float* mean, const float* rstd, float* dx,
                            uint16_t* dx_bf16, float* dw, float* db, float* partial, int rows,
                            int C, cudaStream_t stream) {
  if (C % 4 != 0 || C > 128 * 8 || rows <= 0) return (int)cudaErrorInvalidValue;
  const int K = (C + 127) / 128;
  // Both kernels move 4 columns at a time: 8-byte pieces of the bf16 rows and
  // 16-byte pieces of the fp32 rows (C % 4 == 0 keeps every row on those
  // boundaries when the base pointers are).
  const uintptr_t a16 = reinterpret_cast<uintptr_t>(g_res) | reinterpret_cast<uintptr_t>(x_out) |
                        reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(dx);
  const uintptr_t a8 = reinterpret_cast<uintptr_t>(gy) | reinterpret_cast<uintptr_t>(dx_bf16);
  if ((a16 & 15) != 0 || (a8 & 7) != 0) return (int)cudaErrorInvalidValue;
  if (groupEnabled()) {
    int nparts = 0;
    // Two float4 groups per thread where the bf16 rows allow 16-byte pieces.
    const bool pairs = C % 8 == 0 && (a8 & 15) == 0;
    const cudaError_t e =
        pairs ? bwdGroup<2>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C,
                            &nparts, stream)
              : bwdGroup<1>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C,
                            &nparts, stream);
    if (launched(e) != 0) return (int)e;
    colReduce<<<(2 * C + 31) / 32, kColReduceWarps * 32, 0, stream>>>(partial, nparts, 2 * C,
                                                                      2 * C, C, dw, db);
    return launched(cudaGetLastError());
  }
  cudaError_t e;
  switch (K) {
    case 1: e = bwdK<1>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, stream); break;
    case 2: e = bwdK<2>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, stream); break;
    case 3: case 4: e = bwdK<4>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, stream); break;
    case 5: case 6: e = bwdK<6>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, stream); break;
    default: e = bwdK<8>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, stream); break;
  }
  if (launched(e) != 0) return (int)e;
  int nparts = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (nparts > kPartialRows) nparts = kPartialRows;
  // dw = column sums of the first C partial columns, db of the next C.
  colReduce<<<(2 * C + 31) / 32, kColReduceWarps * 32, 0, stream>>>(partial, nparts, 2 * C,
                                                                    2 * C, C, dw, db);
  return launched(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Allocation-free variant of tnops_ln_bwd (declared in tnops_noalloc.h; no
// counterpart in the tiny-nccl reference). The partial-sum scratch is a
// file-scope device array; host code must not pass the array's name to a
// kernel (on the host it is only a stand-in symbol), so its device address is
// looked up once per device with cudaGetSymbolAddress and cached.
// ---------------------------------------------------------------------------
#include <stdio.h>

#include <mutex>

#include "tnops_noalloc.h"

namespace tnops {
namespace {

constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) float gLnBwdScratch[2 * kPartialRows * TNOPS_NOALLOC_MAX_C];
std::mutex gScratchMutex;
float* gScratchAddr[kNoAllocMaxDevices] = {};

}  // namespace
}  // namespace tnops

extern "C" int tnops_ln_bwd_noalloc(const uint16_t* gy, const float* g_res, const float* x_out,
                                    const float* w, const float* mean, const float* rstd,
                                    float* dx, uint16_t* dx_bf16, float* dw, float* db, int rows,
                                    int C, cudaStream_t stream) {
  if (C > TNOPS_NOALLOC_MAX_C) {
    fprintf(stderr,
            "tnops_ln_bwd_noalloc: C = %d exceeds the built-in scratch limit of %d columns\n", C,
            TNOPS_NOALLOC_MAX_C);
    return (int)cudaErrorInvalidValue;
  }
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return (int)e;
  if (device < 0 || device >= kNoAllocMaxDevices) return (int)cudaErrorInvalidDevice;
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(gScratchMutex);
    if (gScratchAddr[device] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, gLnBwdScratch);
      if (e != cudaSuccess) return (int)e;
      gScratchAddr[device] = static_cast<float*>(p);
    }
    scratch = gScratchAddr[device];
  }
  return tnops_ln_bwd(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, dw, db, scratch, rows, C,
                      stream);
}
