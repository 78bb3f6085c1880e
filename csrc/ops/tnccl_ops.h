// tnccl_ops.h - C launchers of the fused model kernels (libtnccl_ops.so).
//
// All launchers are asynchronous on `stream` and return a cudaError_t cast to
// int (0 = success). Shapes are row-major [rows, cols]; bf16 tensors are
// passed as raw 16-bit storage.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

// x_out = x + delta (delta optional, bf16); y = LayerNorm(x_out) * w + b in
// bf16; mean/rstd saved in fp32. x, x_out fp32 [rows, C]; w, b fp32 [C].
// C % 4 == 0 and C <= 2048; x, x_out, w, b 16-byte aligned, delta and y
// 8-byte aligned; anything else returns 1 (invalid argument), no launch.
int tnops_ln_fwd(const float* x, const uint16_t* delta, const float* w, const float* b,
                 float* x_out, uint16_t* y, float* mean, float* rstd, int rows, int C, float eps,
                 cudaStream_t stream);

// Backward of tnops_ln_fwd. gy bf16 [rows, C]; g_res fp32 [rows, C] (gradient
// arriving through the residual stream; may be null = zeros); x_out, mean,
// rstd from the forward. Writes dx fp32 = g_res + dLN/dx, optionally dx_bf16
// (the same value for the bf16 `delta` input), and dw/db fp32 [C] (overwritten,
// deterministic two-stage reduction through `partial`, which must hold
// 2 * tnops_ln_partial_rows() * C floats). C % 4 == 0 and C <= 1024; g_res,
// x_out, w and dx 16-byte aligned, gy and dx_bf16 8-byte aligned; anything
// else returns 1 (invalid argument) without a launch.
int tnops_ln_bwd(const uint16_t* gy, const float* g_res, const float* x_out, const float* w,
                 const float* mean, const float* rstd, float* dx, uint16_t* dx_bf16, float* dw,
                 float* db, float* partial, int rows, int C, cudaStream_t stream);
int tnops_ln_partial_rows(void);

// Fused softmax cross-entropy over bf16 logits [rows, ld] whose first V
// columns are classes (the rest is padding): loss[r] = logsumexp(logits[r,:V])
// - logits[r, target[r]] (fp32), and logits is overwritten in place with
// d(mean loss)/d(logits) = (softmax - onehot)/valid in bf16 (0 in padding
// columns). Rows whose target is negative are ignored (zero loss and
// gradient); `valid` counts the rows that are not, for the mean.
int tnops_cross_entropy_fwd_bwd(uint16_t* logits, const int64_t* target, float* loss, int rows,
                                int V, int ld, int valid, cudaStream_t stream);

// Bias gradient of a linear layer: db[n] = sum_m g[m, n] (g bf16 [M, N],
// db fp32 [N], N a multiple of 8), deterministic two-pass column sum through
// `partial` (tnops_colsum_parts(M, N) * N floats). The bf16 matrices of this
// and the next function must be 16-byte aligned; otherwise, or with N % 8
// != 0, they return 1 without a launch.
int tnops_bias_grad(const uint16_t* g, float* db, float* partial, int M, int N,
                    cudaStream_t stream);
// Fused tanh-GELU backward and bias gradient of the linear layer feeding the
// GELU: gpre = bf16(gy * gelu'(pre)), db[n] = sum_m gpre[m, n].
int tnops_gelu_bwd_bias(const uint16_t* gy, const uint16_t* pre, uint16_t* gpre, float* db,
                        float* partial, int M, int N, cudaStream_t stream);
int tnops_colsum_parts(int M, int N);

// Multiplies a bf16 tensor by the fp32 scalar *scale (device memory); no-op
// on the device when *scale == 1.
int tnops_scale_bf16(uint16_t* x, size_t n, const float* scale, cudaStream_t stream);

// Multi-tensor AdamW step (decoupled weight decay) over up to 64 tensors per
// call: p -= lr * (m_hat / (sqrt(v_hat) + eps) + wd * p). grads may be scaled
// by grad_scale first. bias corrections are computed from `step` (>= 1).
typedef struct {
  int n;
  float* param[64];
  const float* grad[64];
  float* exp_avg[64];
  float* exp_avg_sq[64];
  int64_t numel[64];
  float weight_decay[64];
  // Optional (null entries skip it): a bf16 copy of each updated parameter,
  // written in the same pass, for the next forward's bf16 GEMMs.
  uint16_t* param_bf16[64];
} tnops_adamw_list;

int tnops_adamw(const tnops_adamw_list* list, float lr, float beta1, float beta2, float eps,
                int64_t step, float grad_scale, cudaStream_t stream);
// The same update with the step read from device memory (*step >= 1) when
// the kernel runs: a launch captured in a CUDA graph then takes the step of
// each replay (the caller advances the counter on the same stream).
int tnops_adamw_dev(const tnops_adamw_list* list, float lr, float beta1, float beta2, float eps,
                    const int64_t* step, float grad_scale, cudaStream_t stream);

// bf16 GEMM on the tcgen05 tensor cores with a fused epilogue:
// pre = bf16(x w^T + bias), and with `gelu` act = bf16(gelu_tanh(pre)).
// x [M, K], w [N, K] (nn.Linear layout), bias [N] (may be null), pre / act
// [M, N] (pre may be null with gelu). `persistent`: 0 one CTA per 128 x 256
// tile, 1 one CTA per SM walking the tiles with two TMEM accumulators, 2 CTA
// pairs (cta_group::2) walking 256 x 256 tiles. K % 8 == 0,
// N % 8 == 0, x, w, pre, act 16-byte aligned; 1 (invalid argument) otherwise.
int tnops_gemm_bias_act(const void* x, const void* w, const void* bias, void* pre, void* act,
                        int M, int N, int K, int gelu, int persistent, cudaStream_t stream);
// First failure code recorded by a tcgen05 GEMM (a bounded wait that expired),
// 0 if none; `reset` clears it. Synchronises the device.
unsigned tnops_tcgen05_status(int reset);

// Number of kernels the ops library launched in this process.
unsigned long long tnops_launch_count(void);

#ifdef __cplusplus
}
#endif
