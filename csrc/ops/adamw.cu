// adamw.cu - multi-tensor AdamW with decoupled weight decay, fp32 state.
//
// One launch covers up to 64 tensors. The grid walks 16 KiB chunks of the
// concatenated tensors; each CTA finds its tensor by scanning the chunk
// prefix table (at most 64 entries) and updates float4 groups:
//   m = b1 m + (1 - b1) g,  v = b2 v + (1 - b2) g^2,
//   p -= lr * ((m / bc1) / (sqrt(v / bc2) + eps) + wd * p),
// and, where the list gives one, writes bf16(p) to the parameter's bf16 copy
// in the same pass (2 more bytes per element instead of a separate cast
// kernel that reads the 4-byte parameter again before the next forward).
// The bias corrections bc1 = 1 - b1^t, bc2 = 1 - b2^t come from the host's
// step t, or (tnops_adamw_dev) from a step counter in device memory, so that
// a launch captured in a CUDA graph uses the step of each replay.
#include <math.h>

#include "common.cuh"
#include "tnccl_ops.h"

namespace tnops {

std::atomic<unsigned long long> gLaunches{0};

namespace {

constexpr int kChunk = 4096;  // elements per CTA iteration

struct AdamArgs {
  tnops_adamw_list list;
  int64_t chunkStart[65];
  float lr, b1, b2, eps, bc1, bc2, gscale;
  const int64_t* stepDev;  // when set, bc1 / bc2 are computed from *stepDev
};

__device__ __forceinline__ void adamElem(float& p, float g, float& m, float& v, float wd,
                                         const AdamArgs& a, float bc1, float bc2) {
  g *= a.gscale;
  m = a.b1 * m + (1.f - a.b1) * g;
  v = a.b2 * v + (1.f - a.b2) * g * g;
  const float mh = m / bc1;
  const float vh = v / bc2;
  p -= a.lr * (mh / (sqrtf(vh) + a.eps) + wd * p);
}

__global__ void __launch_bounds__(256) adamwKernel(const __grid_constant__ AdamArgs a) {
  __shared__ float sBc[2];
  float bc1 = a.bc1, bc2 = a.bc2;
  if (a.stepDev != nullptr) {
    if (threadIdx.x == 0) {
      const double t = (double)*a.stepDev;
      sBc[0] = (float)(1.0 - pow((double)a.b1, t));
      sBc[1] = (float)(1.0 - pow((double)a.b2, t));
    }
    __syncthreads();
    bc1 = sBc[0];
    bc2 = sBc[1];
  }
  const int64_t total = a.chunkStart[a.list.n];
  for (int64_t chunk = blockIdx.x; chunk < total; chunk += gridDim.x) {
    int t = 0;
    while (t + 1 < a.list.n && a.chunkStart[t + 1] <= chunk) ++t;
    const int64_t off = (chunk - a.chunkStart[t]) * kChunk;
    const int64_t n = a.list.numel[t];
    const int64_t end = off + kChunk < n ? off + kChunk : n;
    float* p = a.list.param[t];
    const float* g = a.list.grad[t];
    float* m = a.list.exp_avg[t];
    float* v = a.list.exp_avg_sq[t];
    uint16_t* p16 = a.list.param_bf16[t];
    const float wd = a.list.weight_decay[t];
    const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                       reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(p16) & 7) == 0;
    if (vec) {
      const int64_t v0 = off / 4, v1 = end / 4;
      for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
        float4 pp = reinterpret_cast<float4*>(p)[i];
        const float4 gg = reinterpret_cast<const float4*>(g)[i];
        float4 mm = reinterpret_cast<float4*>(m)[i];
        float4 vv = reinterpret_cast<float4*>(v)[i];
        adamElem(pp.x, gg.x, mm.x, vv.x, wd, a, bc1, bc2);
        adamElem(pp.y, gg.y, mm.y, vv.y, wd, a, bc1, bc2);
        adamElem(pp.z, gg.z, mm.z, vv.z, wd, a, bc1, bc2);
        adamElem(pp.w, gg.w, mm.w, vv.w, wd, a, bc1, bc2);
        reinterpret_cast<float4*>(p)[i] = pp;
        reinterpret_cast<float4*>(m)[i] = mm;
        reinterpret_cast<float4*>(v)[i] = vv;
        if (p16) reinterpret_cast<uint2*>(p16)[i] = tobf4(pp);
      }
      for (int64_t i = v1 * 4 + threadIdx.x; i < end; i += blockDim.x) {
        adamElem(p[i], g[i], m[i], v[i], wd, a, bc1, bc2);
        if (p16) p16[i] = f2bf(p[i]);
      }
    } else {
      for (int64_t i = off + threadIdx.x; i < end; i += blockDim.x) {
        adamElem(p[i], g[i], m[i], v[i], wd, a, bc1, bc2);
        if (p16) p16[i] = f2bf(p[i]);
      }
    }
  }
}

}  // namespace
}  // namespace tnops

using namespace tnops;

static int launchAdamw(const tnops_adamw_list* list, float lr, float beta1, float beta2,
                       float eps, int64_t step, const int64_t* stepDev, float grad_scale,
                       cudaStream_t stream) {
  AdamArgs a;
  a.stepDev = stepDev;
  a.list = *list;
  a.chunkStart[0] = 0;
  for (int t = 0; t < list->n; ++t)
    a.chunkStart[t + 1] = a.chunkStart[t] + (list->numel[t] + kChunk - 1) / kChunk;
  a.lr = lr;
  a.b1 = beta1;
  a.b2 = beta2;
  a.eps = eps;
  a.bc1 = stepDev ? 1.f : (float)(1.0 - pow((double)beta1, (double)step));
  a.bc2 = stepDev ? 1.f : (float)(1.0 - pow((double)beta2, (double)step));
  a.gscale = grad_scale;
  int64_t total = a.chunkStart[list->n];
  int blocks = (int)(total < kSMs * 8 ? total : kSMs * 8);
  if (blocks < 1) blocks = 1;
  adamwKernel<<<blocks, 256, 0, stream>>>(a);
  return launched(cudaGetLastError());
}

extern "C" int tnops_adamw(const tnops_adamw_list* list, float lr, float beta1, float beta2,
                           float eps, int64_t step, float grad_scale, cudaStream_t stream) {
  if (list == nullptr || list->n <= 0 || list->n > 64 || step < 1)
    return (int)cudaErrorInvalidValue;
  return launchAdamw(list, lr, beta1, beta2, eps, step, nullptr, grad_scale, stream);
}

extern "C" int tnops_adamw_dev(const tnops_adamw_list* list, float lr, float beta1, float beta2,
                               float eps, const int64_t* step, float grad_scale,
                               cudaStream_t stream) {
  if (list == nullptr || list->n <= 0 || list->n > 64 || step == nullptr)
    return (int)cudaErrorInvalidValue;
  return launchAdamw(list, lr, beta1, beta2, eps, 0, step, grad_scale, stream);
}

extern "C" unsigned long long tnops_launch_count(void) {
  return gLaunches.load(std::memory_order_relaxed);
}
