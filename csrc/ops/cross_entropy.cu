// cross_entropy.cu - fused softmax cross-entropy forward + backward over bf16
// logits, one CTA per row.
//
// Pass 1 streams the row once from HBM and keeps a running (max, sum of
// exponentials) per thread, combined across the CTA; pass 2 re-reads the row
// (now resident in L2) and overwrites it in place with the gradient of the
// mean loss, (softmax - onehot(target)) / valid. HBM traffic is one read and
// one write of the logits, instead of materialising fp32 log-probabilities.
// A row holds V classes followed by (ld - V) padding columns (a vocabulary
// padded to a multiple of 128 keeps the LM-head GEMMs on aligned tensor-core
// kernels); padding columns take no part in the softmax and get gradient 0.
// A row may start at any 2-byte offset: it is split into a scalar head up to
// the first 16-byte boundary, a 16-byte vector body and a scalar tail.
#include <float.h>

#include "common.cuh"
#include "tnccl_ops.h"

namespace tnops {
namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 4;  // 16-byte loads in flight per thread in each pass

struct MaxSum {
  float m, s;
};

constexpr float kLog2e = 1.4426950408889634f;

// 2^x on the hardware approximation (PTX ex2.approx.ftz.f32); the exponent
// arithmetic around it is folded into one FMA per element below.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ MaxSum combine(MaxSum a, MaxSum b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

__device__ __forceinline__ void unpack8(const uint4& u, float* v) {
  v[0] = __uint_as_float(u.x << 16); v[1] = __uint_as_float(u.x & 0xffff0000u);
  v[2] = __uint_as_float(u.y << 16); v[3] = __uint_as_float(u.y & 0xffff0000u);
  v[4] = __uint_as_float(u.z << 16); v[5] = __uint_as_float(u.z & 0xffff0000u);
  v[6] = __uint_as_float(u.w << 16); v[7] = __uint_as_float(u.w & 0xffff0000u);
}

// Running (max, sum of exp(v - max)) over n more values: exp(v - m) is
// 2^(v log2e - m log2e), one FMA and one ex2 per value.
__device__ __forceinline__ void accumulate(MaxSum& st, const float* v, int n) {
  float lm = v[0];
  for (int i = 1; i < n; ++i) lm = fmaxf(lm, v[i]);
  const float m = fmaxf(st.m, lm);
  const float nm = -m * kLog2e;
  float s = st.m == -INFINITY ? 0.f : st.s * ex2(fmaf(st.m, kLog2e, nm));
  for (int i = 0; i < n; ++i) s += ex2(fmaf(v[i], kLog2e, nm));
  st = {m, s};
}

__global__ void __launch_bounds__(kThreads)
    ceKernel(uint16_t* __restrict__ logits, const int64_t* __restrict__ target,
             float* __restrict__ loss, int V, int ld, float invValid) {
  const int r = blockIdx.x;
  uint16_t* row = logits + (size_t)r * ld;
  const int64_t tgt = target[r];
  const uintptr_t addr = reinterpret_cast<uintptr_t>(row);
  int head = (int)(((16 - (addr & 15)) & 15) >> 1);
  if (head > V) head = V;
  const int nvec = (V - head) >> 3;
  const int bodyEnd = head + nvec * 8;
  const uint4* body = reinterpret_cast<const uint4*>(row + head);

  __shared__ float sTarget;
  __shared__ MaxSum sPart[kThreads / 32];
  __shared__ MaxSum sAll;
  if (threadIdx.x == 0) sTarget = (tgt >= 0 && tgt < V) ? bf2f(row[tgt]) : 0.f;

  MaxSum st{-INFINITY, 0.f};
  // kUnroll vectors per thread per step: their loads are all issued before
  // any is used, and one (max, sum) update covers 32 values.
  int i0 = threadIdx.x;
  for (; i0 + (kUnroll - 1) * kThreads < nvec; i0 += kUnroll * kThreads) {
    uint4 u[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) u[j] = body[i0 + j * kThreads];  // stays in L2 for pass 2
    float v[8 * kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) unpack8(u[j], v + 8 * j);
    accumulate(st, v, 8 * kUnroll);
  }
  for (int i = i0; i < nvec; i += kThreads) {
    float v[8];
    unpack8(body[i], v);
    accumulate(st, v, 8);
  }
  for (int i = threadIdx.x; i < head; i += kThreads) {
    float v = bf2f(row[i]);
    accumulate(st, &v, 1);
  }
  for (int i = bodyEnd + threadIdx.x; i < V; i += kThreads) {
    float v = bf2f(row[i]);
    accumulate(st, &v, 1);
  }
  // CTA reduction of (max, sum).
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o)};
    st = combine(st, other);
  }
  if ((threadIdx.x & 31) == 0) sPart[threadIdx.x >> 5] = st;
  __syncthreads();
  if (threadIdx.x < 32) {
    MaxSum t = threadIdx.x < kThreads / 32 ? sPart[threadIdx.x] : MaxSum{-INFINITY, 0.f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      MaxSum other{__shfl_xor_sync(0xffffffffu, t.m, o), __shfl_xor_sync(0xffffffffu, t.s, o)};
      t = combine(t, other);
    }
    if (threadIdx.x == 0) sAll = t;
  }
  __syncthreads();
  const float M = sAll.m;
  const bool valid = tgt >= 0 && tgt < V;
  if (threadIdx.x == 0) loss[r] = valid ? (logf(sAll.s) + M - sTarget) : 0.f;
  const float scale = valid ? invValid : 0.f;
  // p * scale = 2^(a log2e + nb) with nb = -(M log2e + log2 S) + log2 scale;
  // the target column subtracts scale (softmax minus one-hot, scaled).
  const float nb = valid ? -(M * kLog2e) - __log2f(sAll.s) + __log2f(invValid) : 0.f;
  // Pass 2: gradient in place.
  uint4* wbody = reinterpret_cast<uint4*>(row + head);
  auto grad8 = [&](const uint4& u, int i) {
    const int e0 = head + i * 8;
    const uint32_t in[4] = {u.x, u.y, u.z, u.w};
    uint32_t out[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a = __uint_as_float(in[k] << 16), b = __uint_as_float(in[k] & 0xffff0000u);
      float pa = valid ? ex2(fmaf(a, kLog2e, nb)) : 0.f;
      float pb = valid ? ex2(fmaf(b, kLog2e, nb)) : 0.f;
      if (e0 + 2 * k == tgt) pa -= scale;
      if (e0 + 2 * k + 1 == tgt) pb -= scale;
      __nv_bfloat162 h = __floats2bfloat162_rn(pa, pb);
      out[k] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
  };
  i0 = threadIdx.x;
  for (; i0 + (kUnroll - 1) * kThreads < nvec; i0 += kUnroll * kThreads) {
    uint4 u[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) u[j] = wbody[i0 + j * kThreads];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j)
      __stcs(wbody + i0 + j * kThreads, grad8(u[j], i0 + j * kThreads));
  }
  for (int i = i0; i < nvec; i += kThreads) wbody[i] = grad8(wbody[i], i);
  for (int i = threadIdx.x; i < head; i += kThreads) {
    float p = valid ? ex2(fmaf(bf2f(row[i]), kLog2e, nb)) : 0.f;
    if (i == tgt) p -= scale;
    row[i] = f2bf(p);
  }
  for (int i = bodyEnd + threadIdx.x; i < V; i += kThreads) {
    float p = valid ? ex2(fmaf(bf2f(row[i]), kLog2e, nb)) : 0.f;
    if (i == tgt) p -= scale;
    row[i] = f2bf(p);
  }
  for (int i = V + threadIdx.x; i < ld; i += kThreads) row[i] = 0;
}

__global__ void scaleBf16(uint16_t* __restrict__ x, size_t n, const float* __restrict__ scale) {
  const float s = *scale;
  if (s == 1.0f) return;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    x[i] = f2bf(bf2f(x[i]) * s);
}

}  // namespace
}  // namespace tnops

using namespace tnops;

extern "C" int tnops_cross_entropy_fwd_bwd(uint16_t* logits, const int64_t* target, float* loss,
                                           int rows, int V, int ld, int valid,
                                           cudaStream_t stream) {
  if (rows <= 0 || V <= 0 || ld < V) return (int)cudaErrorInvalidValue;
  const float inv = valid > 0 ? 1.0f / (float)valid : 0.f;
  ceKernel<<<rows, kThreads, 0, stream>>>(logits, target, loss, V, ld, inv);
  return launched(cudaGetLastError());
}

extern "C" int tnops_scale_bf16(uint16_t* x, size_t n, const float* scale, cudaStream_t stream) {
  scaleBf16<<<kSMs * 4, 256, 0, stream>>>(x, n, scale);
  return launched(cudaGetLastError());
}
