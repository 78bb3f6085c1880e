// ops_ext.cpp - PyTorch binding of the model kernels (csrc/ops). Each entry
// validates its tensors and calls the C launcher on the current CUDA stream;
// a launcher error raises instead of falling back to another implementation.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <vector>

#include "tnccl_ops.h"

namespace py = pybind11;

namespace {

cudaStream_t streamOf(const at::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.get_device()).stream();
}

void need(const at::Tensor& t, at::ScalarType st, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.scalar_type() == st, name, " has dtype ", t.scalar_type(), ", expected ", st);
}

void ok(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " failed: ", cudaGetErrorString((cudaError_t)rc));
}

uint16_t* bf(at::Tensor& t) { return reinterpret_cast<uint16_t*>(t.data_ptr()); }
const uint16_t* bf(const at::Tensor& t) { return reinterpret_cast<const uint16_t*>(t.data_ptr()); }

// x fp32 [rows, C], optional delta bf16 [rows, C] -> x_out, y (bf16), mean, rstd
std::vector<at::Tensor> lnFwd(const at::Tensor& x, const c10::optional<at::Tensor>& delta,
                              const at::Tensor& w, const at::Tensor& b, double eps) {
  need(x, at::kFloat, "x");
  need(w, at::kFloat, "weight");
  need(b, at::kFloat, "bias");
  const int64_t C = x.size(-1);
  const int64_t rows = x.numel() / C;
  TORCH_CHECK(w.numel() == C && b.numel() == C, "LayerNorm parameters must have C elements");
  if (delta) {
    need(*delta, at::kBFloat16, "delta");
    TORCH_CHECK(delta->numel() == x.numel(), "delta must match x");
  }
  c10::cuda::CUDAGuard g(x.device());
  auto xo = at::empty_like(x);
  auto y = at::empty(x.sizes(), x.options().dtype(at::kBFloat16));
  auto mean = at::empty({rows}, x.options());
  auto rstd = at::empty({rows}, x.options());
  ok(tnops_ln_fwd(x.data_ptr<float>(), delta ? bf(*delta) : nullptr, w.data_ptr<float>(),
                  b.data_ptr<float>(), xo.data_ptr<float>(), bf(y), mean.data_ptr<float>(),
                  rstd.data_ptr<float>(), (int)rows, (int)C, (float)eps, streamOf(x)),
     "tnops_ln_fwd");
  return {xo, y, mean, rstd};
}

std::vector<at::Tensor> lnBwd(const at::Tensor& gy, const c10::optional<at::Tensor>& gres,
                              const at::Tensor& xo, const at::Tensor& w, const at::Tensor& mean,
                              const at::Tensor& rstd, bool wantBf16,
                              const c10::optional<at::Tensor>& dwOut,
                              const c10::optional<at::Tensor>& dbOut) {
  need(gy, at::kBFloat16, "grad_y");
  need(xo, at::kFloat, "x_out");
  need(w, at::kFloat, "weight");
  if (gres) need(*gres, at::kFloat, "grad_residual");
  const int64_t C = xo.size(-1);
  const int64_t rows = xo.numel() / C;
  c10::cuda::CUDAGuard g(xo.device());
  auto dx = at::empty_like(xo);
  at::Tensor dxb;
  if (wantBf16) dxb = at::empty(xo.sizes(), xo.options().dtype(at::kBFloat16));
  // dw / db go to the caller's tensors when given (e.g. the parameters'
  // slices of a flat gradient buffer), so that no copy follows.
  auto dw = dwOut ? *dwOut : at::empty({C}, xo.options());
  auto db = dbOut ? *dbOut : at::empty({C}, xo.options());
  need(dw, at::kFloat, "dw_out");
  need(db, at::kFloat, "db_out");
  TORCH_CHECK(dw.numel() == C && db.numel() == C, "ln_bwd: dw_out / db_out need C elements");
  auto partial = at::empty({(int64_t)tnops_ln_partial_rows() * 2 * C}, xo.options());
  ok(tnops_ln_bwd(bf(gy), gres ? gres->data_ptr<float>() : nullptr, xo.data_ptr<float>(),
                  w.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
                  dx.data_ptr<float>(), wantBf16 ? bf(dxb) : nullptr, dw.data_ptr<float>(),
                  db.data_ptr<float>(), partial.data_ptr<float>(), (int)rows, (int)C,
                  streamOf(xo)),
     "tnops_ln_bwd");
  return {dx, wantBf16 ? dxb : at::Tensor(), dw, db};
}

// logits bf16 [rows, ld] with `classes` real columns (overwritten with
// d mean-loss / d logits), targets int64
at::Tensor crossEntropy(at::Tensor logits, const at::Tensor& target, int64_t valid,
                        int64_t classes) {
  need(logits, at::kBFloat16, "logits");
  need(target, at::kLong, "target");
  TORCH_CHECK(logits.dim() == 2 && target.numel() == logits.size(0), "shape mismatch");
  const int64_t ld = logits.size(1);
  if (classes <= 0) classes = ld;
  TORCH_CHECK(classes <= ld, "more classes than logits columns");
  c10::cuda::CUDAGuard g(logits.device());
  auto loss = at::empty({logits.size(0)}, logits.options().dtype(at::kFloat));
  ok(tnops_cross_entropy_fwd_bwd(bf(logits), target.data_ptr<int64_t>(), loss.data_ptr<float>(),
                                 (int)logits.size(0), (int)classes, (int)ld, (int)valid,
                                 streamOf(logits)),
     "tnops_cross_entropy_fwd_bwd");
  return loss;
}

// g bf16 [M, N] -> db fp32 [N] (column sums)
at::Tensor biasGrad(const at::Tensor& g, const c10::optional<at::Tensor>& out) {
  need(g, at::kBFloat16, "grad");
  TORCH_CHECK(g.dim() == 2 && g.size(1) % 8 == 0, "bias_grad: want [M, N] with N % 8 == 0");
  c10::cuda::CUDAGuard guard(g.device());
  const int M = (int)g.size(0), N = (int)g.size(1);
  auto db = out ? *out : at::empty({N}, g.options().dtype(at::kFloat));
  need(db, at::kFloat, "out");
  TORCH_CHECK(db.numel() == N, "bias_grad: out needs N elements");
  auto part = at::empty({(int64_t)tnops_colsum_parts(M, N) * N}, g.options().dtype(at::kFloat));
  ok(tnops_bias_grad(bf(g), db.data_ptr<float>(), part.data_ptr<float>(), M, N, streamOf(g)),
     "tnops_bias_grad");
  return db;
}

// x bf16 [M, K], w bf16 [N, K], bias bf16 [N] or None -> [pre] or, with gelu,
// [pre, act] (bf16 [M, N]) from the tcgen05 GEMM with the fused epilogue.
std::vector<at::Tensor> gemmBiasAct(const at::Tensor& x, const at::Tensor& w,
                                    const c10::optional<at::Tensor>& bias, bool gelu,
                                    int64_t persistent) {
  need(x, at::kBFloat16, "x");
  need(w, at::kBFloat16, "weight");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1),
              "gemm_bias_act: want x [M, K] and weight [N, K]");
  TORCH_CHECK(x.size(1) % 8 == 0 && w.size(0) % 8 == 0,
              "gemm_bias_act: K and N must be multiples of 8");
  if (bias) {
    need(*bias, at::kBFloat16, "bias");
    TORCH_CHECK(bias->numel() == w.size(0), "gemm_bias_act: bias must have N elements");
  }
  c10::cuda::CUDAGuard guard(x.device());
  const int M = (int)x.size(0), N = (int)w.size(0), K = (int)x.size(1);
  auto pre = at::empty({M, N}, x.options());
  at::Tensor act = gelu ? at::empty({M, N}, x.options()) : at::Tensor();
  const int rc = tnops_gemm_bias_act(x.data_ptr(), w.data_ptr(), bias ? bias->data_ptr() : nullptr,
                                     pre.data_ptr(), gelu ? act.data_ptr() : nullptr, M, N, K,
                                     gelu ? 1 : 0, (int)persistent, streamOf(x));
  TORCH_CHECK(rc == 0, "tnops_gemm_bias_act failed (code ", rc, ")");
  if (gelu) return {pre, act};
  return {pre};
}

// gy, pre bf16 [M, N] -> (gpre bf16 [M, N], db fp32 [N])
std::vector<at::Tensor> geluBwdBias(const at::Tensor& gy, const at::Tensor& pre,
                                    const c10::optional<at::Tensor>& dbOut) {
  need(gy, at::kBFloat16, "grad_y");
  need(pre, at::kBFloat16, "pre");
  TORCH_CHECK(gy.dim() == 2 && gy.sizes() == pre.sizes() && gy.size(1) % 8 == 0,
              "gelu_bwd_bias: want equal [M, N] with N % 8 == 0");
  c10::cuda::CUDAGuard guard(gy.device());
  const int M = (int)gy.size(0), N = (int)gy.size(1);
  auto gpre = at::empty_like(gy);
  auto db = dbOut ? *dbOut : at::empty({N}, gy.options().dtype(at::kFloat));
  need(db, at::kFloat, "db_out");
  TORCH_CHECK(db.numel() == N, "gelu_bwd_bias: db_out needs N elements");
  auto part = at::empty({(int64_t)tnops_colsum_parts(M, N) * N}, gy.options().dtype(at::kFloat));
  ok(tnops_gelu_bwd_bias(bf(gy), bf(pre), bf(gpre), db.data_ptr<float>(), part.data_ptr<float>(),
                         M, N, streamOf(gy)),
     "tnops_gelu_bwd_bias");
  return {gpre, db};
}

void scaleBf16(at::Tensor x, const at::Tensor& scale) {
  need(x, at::kBFloat16, "x");
  need(scale, at::kFloat, "scale");
  c10::cuda::CUDAGuard g(x.device());
  ok(tnops_scale_bf16(bf(x), (size_t)x.numel(), scale.data_ptr<float>(), streamOf(x)),
     "tnops_scale_bf16");
}

void adamw(const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& grads,
           const std::vector<at::Tensor>& m, const std::vector<at::Tensor>& v,
           const std::vector<double>& wd, double lr, double b1, double b2, double eps,
           int64_t step, double gscale, const c10::optional<at::Tensor>& stepDev,
           const std::vector<at::Tensor>& bf16Copies) {
  TORCH_CHECK(bf16Copies.empty() || bf16Copies.size() == params.size(),
              "adamw: param_bf16 must be empty or one tensor per parameter");
  if (stepDev.has_value()) {
    TORCH_CHECK(stepDev->is_cuda() && stepDev->scalar_type() == at::kLong &&
                    stepDev->numel() == 1,
                "adamw: step_tensor must be one int64 on the GPU");
  }
  const size_t n = params.size();
  TORCH_CHECK(grads.size() == n && m.size() == n && v.size() == n && wd.size() == n,
              "adamw: list lengths differ");
  if (n == 0) return;
  c10::cuda::CUDAGuard g(params[0].device());
  cudaStream_t st = streamOf(params[0]);
  for (size_t base = 0; base < n; base += 64) {
    tnops_adamw_list L{};
    L.n = (int)std::min<size_t>(64, n - base);
    for (int i = 0; i < L.n; ++i) {
      const size_t k = base + (size_t)i;
      need(params[k], at::kFloat, "param");
      need(grads[k], at::kFloat, "grad");
      need(m[k], at::kFloat, "exp_avg");
      need(v[k], at::kFloat, "exp_avg_sq");
      L.param[i] = params[k].data_ptr<float>();
      L.grad[i] = grads[k].data_ptr<float>();
      L.exp_avg[i] = m[k].data_ptr<float>();
      L.exp_avg_sq[i] = v[k].data_ptr<float>();
      L.numel[i] = params[k].numel();
      L.weight_decay[i] = (float)wd[k];
      if (!bf16Copies.empty()) {
        const at::Tensor& c = bf16Copies[k];
        TORCH_CHECK(c.scalar_type() == at::kBFloat16 && c.is_contiguous() &&
                        c.numel() == params[k].numel() && c.device() == params[k].device(),
                    "adamw: param_bf16 must be contiguous bf16 of the parameter's size");
        L.param_bf16[i] = reinterpret_cast<uint16_t*>(c.data_ptr());
      }
    }
    if (stepDev.has_value())
      ok(tnops_adamw_dev(&L, (float)lr, (float)b1, (float)b2, (float)eps,
                         stepDev->data_ptr<int64_t>(), (float)gscale, st),
         "tnops_adamw_dev");
    else
      ok(tnops_adamw(&L, (float)lr, (float)b1, (float)b2, (float)eps, step, (float)gscale, st),
         "tnops_adamw");
  }
}

}  // namespace

void registerOps(py::module_& m) {
  py::module_ ops = m.def_submodule("ops", "fused sm_100a model kernels");
  ops.attr("available") = true;
  ops.def("ln_fwd", &lnFwd, py::arg("x"), py::arg("delta"), py::arg("weight"), py::arg("bias"),
          py::arg("eps"));
  ops.def("ln_bwd", &lnBwd, py::arg("grad_y"), py::arg("grad_residual"), py::arg("x_out"),
          py::arg("weight"), py::arg("mean"), py::arg("rstd"), py::arg("want_bf16"),
          py::arg("dw_out") = py::none(), py::arg("db_out") = py::none());
  ops.def("cross_entropy_fwd_bwd", &crossEntropy, py::arg("logits"), py::arg("target"),
          py::arg("valid"), py::arg("classes") = 0);
  ops.def("bias_grad", &biasGrad, py::arg("grad"), py::arg("out") = py::none());
  ops.def("gelu_bwd_bias", &geluBwdBias, py::arg("grad_y"), py::arg("pre"),
          py::arg("db_out") = py::none());
  ops.def("gemm_bias_act", &gemmBiasAct, py::arg("x"), py::arg("weight"), py::arg("bias"),
          py::arg("gelu"), py::arg("persistent") = 0);
  ops.def("tcgen05_status", [](bool reset) { return tnops_tcgen05_status(reset ? 1 : 0); },
          py::arg("reset") = false);
  ops.def("scale_bf16_", &scaleBf16);
  ops.def("adamw", &adamw, py::arg("params"), py::arg("grads"), py::arg("exp_avg"),
          py::arg("exp_avg_sq"), py::arg("weight_decay"), py::arg("lr"), py::arg("beta1"),
          py::arg("beta2"), py::arg("eps"), py::arg("step"), py::arg("grad_scale"),
          py::arg("step_tensor") = py::none(),
          py::arg("param_bf16") = std::vector<at::Tensor>());
  ops.def("launch_count", []() { return tnops_launch_count(); });
}
