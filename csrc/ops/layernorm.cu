// layernorm.cu - fused residual add + LayerNorm (forward and backward) for a
// fp32 residual stream with bf16 activations, one warp per row.
//
// Forward:  x_out = x + delta;  y = (x_out - mean) * rstd * w + b   (bf16)
// Backward: with xhat = (x_out - mean) * rstd and gw = gy * w,
//           dx = g_res + rstd * (gw - mean(gw) - xhat * mean(gw * xhat))
//           dw = sum_rows gy * xhat,  db = sum_rows gy
// dw/db are reduced deterministically: each CTA keeps per-warp column sums,
// combines its warps in shared memory and writes one partial row; a second
// kernel sums the partial rows in a fixed order. The backward has two
// kernels: a pipelined one (rows of C % 8 == 0 staged through shared memory
// with cp.async, several rows in flight per warp) and one that loads each
// row straight into registers (any C % 4 == 0).
#include <stdlib.h>

#include "common.cuh"
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
// Pipelined backward for C % 8 == 0 and 16-byte aligned rows (the usual
// case; the kernel above handles the rest). One CTA of 8 warps per SM; each
// warp owns rows warp + 8 * blockIdx.x + j * (8 * gridDim.x) and keeps its
// next S - 1 rows in flight while it computes the current one: the row's gy,
// x_out and residual gradient are copied global -> shared with 16-byte
// cp.async into a ring of S per-warp stages, so the memory system always
// has requests queued and the warp never waits on a load it has just
// issued. The dW / dB sums stay in registers (the loads no longer occupy
// them). Summation order per column: each warp's rows in row order, the 8
// warps in warp order, then the CTAs in order (colReduce).
// ---------------------------------------------------------------------------
constexpr int kPipeWarps = 8;

__device__ __forceinline__ void cpAsync16(void* dst, const void* src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(src) : "memory");
}
__device__ __forceinline__ void cpAsyncCommit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cpAsyncWait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Stage layout (bytes): gy [2C] | x_out [4C] | g_res [4C]; every part starts
// on a 16-byte boundary because C % 8 == 0.
__device__ __forceinline__ void lnBwdIssueRow(char* st, const uint16_t* gy, const float* xo,
                                              const float* gres, size_t base, int C, int lane) {
  const char* g = reinterpret_cast<const char*>(gy + base);
  const char* x = reinterpret_cast<const char*>(xo + base);
  for (int q = lane; q < (C >> 3); q += 32) cpAsync16(st + 16 * q, g + 16 * q);
  for (int q = lane; q < (C >> 2); q += 32) cpAsync16(st + 2 * C + 16 * q, x + 16 * q);
  if (gres) {
    const char* r = reinterpret_cast<const char*>(gres + base);
    for (int q = lane; q < (C >> 2); q += 32) cpAsync16(st + 6 * C + 16 * q, r + 16 * q);
  }
}

template <int K, int S>
__global__ void __launch_bounds__(kPipeWarps * 32, 1)
    lnBwdPipeKernel(const uint16_t* __restrict__ gy, const float* __restrict__ gres,
                    const float* __restrict__ xo, const float* __restrict__ w,
                    const float* __restrict__ mean, const float* __restrict__ rstd,
                    float* __restrict__ dx, uint16_t* __restrict__ dxb,
                    float* __restrict__ partial, int rows, int C) {
  extern __shared__ __align__(16) char sPipe[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int C4 = C >> 2;
  const float invC = 1.0f / (float)C;
  const size_t stageBytes = (size_t)10 * C;
  char* ring = sPipe + (size_t)warp * S * stageBytes;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const int stride = gridDim.x * kPipeWarps;
  const int first = blockIdx.x * kPipeWarps + warp;

  float4 aw[K], ab[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    aw[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    ab[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // Prologue: rows 0 .. S-2 of this warp, one commit group each (empty
  // groups past the end keep the group count uniform).
#pragma unroll
  for (int j = 0; j < S - 1; ++j) {
    const int row = first + j * stride;
    if (row < rows) lnBwdIssueRow(ring + j * stageBytes, gy, xo, gres, (size_t)row * C, C, lane);
    cpAsyncCommit();
  }
  int slot = 0;
  for (int row = first; row < rows; row += stride) {
    // Refill the stage computed in the previous iteration with the row S-1
    // ahead, then wait for all but the newest S-1 groups: this row's copies.
    const int ahead = row + (S - 1) * stride;
    const int aslot = slot == 0 ? S - 1 : slot - 1;
    if (ahead < rows)
      lnBwdIssueRow(ring + aslot * stageBytes, gy, xo, gres, (size_t)ahead * C, C, lane);
    cpAsyncCommit();
    cpAsyncWait<S - 1>();
    __syncwarp();  // the copies of every lane of the warp are visible

    const char* st = ring + slot * stageBytes;
    const uint2* gs = reinterpret_cast<const uint2*>(st);
    const float4* xs = reinterpret_cast<const float4*>(st + 2 * C);
    const float4* rsm = reinterpret_cast<const float4*>(st + 6 * C);
    const float mu = mean[row], rs = rstd[row];
    float4 g[K], xh[K];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int i = lane + 32 * k;
      if (i < C4) {
        g[k] = bf4(gs[i]);
        const float4 xv = xs[i];
        xh[k] = make_float4((xv.x - mu) * rs, (xv.y - mu) * rs, (xv.z - mu) * rs,
                            (xv.w - mu) * rs);
        const float4 ww = w4[i];
        const float4 gw = make_float4(g[k].x * ww.x, g[k].y * ww.y, g[k].z * ww.z, g[k].w * ww.w);
        s1 += (gw.x + gw.y) + (gw.z + gw.w);
        s2 += (gw.x * xh[k].x + gw.y * xh[k].y) + (gw.z * xh[k].z + gw.w * xh[k].w);
        aw[k].x += g[k].x * xh[k].x;
        aw[k].y += g[k].y * xh[k].y;
        aw[k].z += g[k].z * xh[k].z;
        aw[k].w += g[k].w * xh[k].w;
        ab[k].x += g[k].x;
        ab[k].y += g[k].y;
        ab[k].z += g[k].z;
        ab[k].w += g[k].w;
      }
    }
    const float m1 = warpSum(s1) * invC, m2 = warpSum(s2) * invC;
    const size_t base = (size_t)row * C;
    float4* dr = reinterpret_cast<float4*>(dx + base);
    uint2* dbr = dxb ? reinterpret_cast<uint2*>(dxb + base) : nullptr;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int i = lane + 32 * k;
      if (i < C4) {
        const float4 ww = w4[i];
        const float4 res = gres ? rsm[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 o;
        o.x = rs * (g[k].x * ww.x - m1 - xh[k].x * m2) + res.x;
        o.y = rs * (g[k].y * ww.y - m1 - xh[k].y * m2) + res.y;
        o.z = rs * (g[k].z * ww.z - m1 - xh[k].z * m2) + res.z;
        o.w = rs * (g[k].w * ww.w - m1 - xh[k].w * m2) + res.w;
        dr[i] = o;
        if (dbr) dbr[i] = tobf4(o);
      }
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
    slot = slot + 1 == S ? 0 : slot + 1;
  }
  cpAsyncWait<0>();
  // Combine the warps of this CTA into one partial row of [dw | db], reusing
  // the stages (8 warps x 2C floats = 64 C bytes <= 80 C S bytes).
  __syncthreads();
  float* acc = reinterpret_cast<float*>(sPipe);
  float4* myDw = reinterpret_cast<float4*>(acc + (size_t)warp * C);
  float4* myDb = reinterpret_cast<float4*>(acc + (size_t)(kPipeWarps + warp) * C);
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int i = lane + 32 * k;
    if (i < C4) {
      myDw[i] = aw[k];
      myDb[i] = ab[k];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) {
    const int q = c / C, col = c - q * C;
    const float* src = acc + (size_t)q * kPipeWarps * C + col;
    float a = 0.f;
#pragma unroll
    for (int wv = 0; wv < kPipeWarps; ++wv) a += src[(size_t)wv * C];
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

template <int K, int S>
cudaError_t bwdPipeK(const uint16_t* gy, const float* gres, const float* xo, const float* w,
                     const float* m, const float* r, float* dx, uint16_t* dxb, float* partial,
                     int rows, int C, int* nparts, cudaStream_t st) {
  static_assert(S >= 2, "at least one row in flight while another is computed");
  int blocks = (rows + kPipeWarps - 1) / kPipeWarps;
  if (blocks > kSMs) blocks = kSMs;
  *nparts = blocks;
  const int smem = S * kPipeWarps * 10 * C;
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (!(done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(lnBwdPipeKernel<K, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             S * kPipeWarps * 10 * 128 * K);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  lnBwdPipeKernel<K, S><<<blocks, kPipeWarps * 32, smem, st>>>(gy, gres, xo, w, m, r, dx, dxb,
                                                               partial, rows, C);
  return cudaGetLastError();
}

// TNOPS_LN_BWD_PIPE=0 selects the one-row-per-warp kernel for every shape
// (A/B timing); by default the pipelined kernel takes the shapes it supports.
bool pipeEnabled() {
  static const bool on = [] {
    const char* v = getenv("TNOPS_LN_BWD_PIPE");
    return v == nullptr || v[0] != '0';
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
  const uintptr_t rowAlign = reinterpret_cast<uintptr_t>(gy) |
                             reinterpret_cast<uintptr_t>(g_res) |
                             reinterpret_cast<uintptr_t>(x_out);
  if (C % 8 == 0 && (rowAlign & 15) == 0 && pipeEnabled()) {
    int nparts = 0;
    cudaError_t e;
    switch (K) {
      case 1: e = bwdPipeK<1, 3>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, &nparts, stream); break;
      case 2: e = bwdPipeK<2, 3>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, &nparts, stream); break;
      case 3: case 4: e = bwdPipeK<4, 3>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, &nparts, stream); break;
      case 5: case 6: e = bwdPipeK<6, 3>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, &nparts, stream); break;
      default: e = bwdPipeK<8, 2>(gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, partial, rows, C, &nparts, stream); break;
    }
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
