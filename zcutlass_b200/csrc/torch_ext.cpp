// PyTorch operator registration for the zcutlass GEMM (CUDA dispatch key only).
//
//   torch.ops.zcutlass_torch.gemm(A, B, C=None, bias=None, alpha=1.0, beta=0.0) -> D
//       same schema, checks and error behaviour as the reference op
//       (python/zcutlass_torch/csrc/zcutlass_torch.cpp:36-89, 153-156 in
//       supercatking/zcutlass): 2-D contiguous CUDA tensors, f16/bf16, D
//       allocated with at::empty, current CUDA stream, RuntimeError on failure.
//   torch.ops.zcutlass.gemm      the same op under the namespace the product spec names
//   torch.ops.zcutlass.gemm_out  writes into a caller-provided D (no allocation)
//   torch.ops.zcutlass.linear(x, weight, bias=None) -> y
//       nn.functional.linear semantics: weight is the PyTorch [N, K] layout and
//       is consumed directly as a column-major B (no transposed copy).
//
// This file only adapts tensors to zcutlass::gemm; all kernels live in libzcutlass.so.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <optional>

#include "zcutlass/gemm.hpp"

namespace {

zcutlass::DType dtype_of(const at::Tensor& t) {
  if (t.scalar_type() == at::kHalf) return zcutlass::DType::F16;
  if (t.scalar_type() == at::kBFloat16) return zcutlass::DType::BF16;
  TORCH_CHECK(false, "zcutlass only supports float16 and bfloat16 tensors");
}

void check_2d_cuda_contiguous(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 2, name, " must be rank-2");
  TORCH_CHECK(t.is_contiguous(), name, " must be row-major contiguous");
  (void)dtype_of(t);
}

void check_operands(const at::Tensor& a, const at::Tensor& b, const std::optional<at::Tensor>& c,
                    const std::optional<at::Tensor>& bias) {
  check_2d_cuda_contiguous(a, "A");
  check_2d_cuda_contiguous(b, "B");
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "A and B dtype must match");
  TORCH_CHECK(a.size(1) == b.size(0), "A.shape[1] must equal B.shape[0]");
  TORCH_CHECK(a.device() == b.device(), "A and B must be on the same CUDA device");
  if (c.has_value()) {
    check_2d_cuda_contiguous(*c, "C");
    TORCH_CHECK(c->scalar_type() == a.scalar_type(), "C dtype must match A/B");
    TORCH_CHECK(c->device() == a.device(), "C must be on the same CUDA device");
    TORCH_CHECK(c->size(0) == a.size(0) && c->size(1) == b.size(1),
                "C shape must be [A.shape[0], B.shape[1]]");
  }
  if (bias.has_value()) {
    TORCH_CHECK(bias->is_cuda(), "bias must be a CUDA tensor");
    TORCH_CHECK(bias->dim() == 1, "bias must be rank-1");
    TORCH_CHECK(bias->is_contiguous(), "bias must be contiguous");
    TORCH_CHECK(bias->scalar_type() == a.scalar_type(), "bias dtype must match A/B");
    TORCH_CHECK(bias->device() == a.device(), "bias must be on the same CUDA device");
    TORCH_CHECK(bias->size(0) == b.size(1), "bias length must equal B.shape[1]");
  }
}

void run_gemm(const at::Tensor& a, const at::Tensor& b, const std::optional<at::Tensor>& c,
              const std::optional<at::Tensor>& bias, double alpha, double beta, at::Tensor& d) {
  const zcutlass::DType t = dtype_of(a);
  zcutlass::GemmDesc desc{a.size(0),
                          b.size(1),
                          a.size(1),
                          a.stride(0),
                          b.stride(0),
                          c.has_value() ? c->stride(0) : b.size(1),
                          d.stride(0),
                          t,
                          t,
                          t,
                          t,
                          static_cast<float>(alpha),
                          static_cast<float>(beta),
                          bias.has_value() ? bias->data_ptr() : nullptr,
                          at::cuda::getCurrentCUDAStream().stream()};
  const zcutlass::Status status = zcutlass::gemm(
      desc, a.data_ptr(), b.data_ptr(), c.has_value() ? c->data_ptr() : nullptr, d.data_ptr());
  TORCH_CHECK(status == zcutlass::Status::Success, "zcutlass::gemm failed: ",
              zcutlass::status_to_string(status));
}

at::Tensor gemm_op(const at::Tensor& a, const at::Tensor& b, const std::optional<at::Tensor>& c,
                   const std::optional<at::Tensor>& bias, double alpha, double beta) {
  check_operands(a, b, c, bias);
  const c10::cuda::CUDAGuard guard(a.device());
  at::Tensor d = at::empty({a.size(0), b.size(1)}, a.options());
  run_gemm(a, b, c, bias, alpha, beta, d);
  return d;
}

void gemm_out_op(const at::Tensor& a, const at::Tensor& b, const std::optional<at::Tensor>& c,
                 const std::optional<at::Tensor>& bias, double alpha, double beta, at::Tensor d) {
  check_operands(a, b, c, bias);
  check_2d_cuda_contiguous(d, "D");
  TORCH_CHECK(d.scalar_type() == a.scalar_type(), "D dtype must match A/B");
  TORCH_CHECK(d.device() == a.device(), "D must be on the same CUDA device");
  TORCH_CHECK(d.size(0) == a.size(0) && d.size(1) == b.size(1),
              "D shape must be [A.shape[0], B.shape[1]]");
  const c10::cuda::CUDAGuard guard(a.device());
  run_gemm(a, b, c, bias, alpha, beta, d);
}

// y[..., N] = x[..., K] @ weight[N, K]^T + bias
at::Tensor linear_op(const at::Tensor& x, const at::Tensor& weight,
                     const std::optional<at::Tensor>& bias) {
  TORCH_CHECK(x.is_cuda() && weight.is_cuda(), "x and weight must be CUDA tensors");
  TORCH_CHECK(weight.dim() == 2 && weight.is_contiguous(), "weight must be a contiguous [N, K] matrix");
  TORCH_CHECK(x.dim() >= 1 && x.size(-1) == weight.size(1), "x.shape[-1] must equal weight.shape[1]");
  TORCH_CHECK(x.scalar_type() == weight.scalar_type(), "x and weight dtype must match");
  TORCH_CHECK(x.device() == weight.device(), "x and weight must be on the same CUDA device");
  const zcutlass::DType t = dtype_of(x);
  if (bias.has_value()) {
    TORCH_CHECK(bias->is_cuda() && bias->dim() == 1 && bias->is_contiguous(),
                "bias must be a contiguous rank-1 CUDA tensor");
    TORCH_CHECK(bias->scalar_type() == x.scalar_type(), "bias dtype must match x");
    TORCH_CHECK(bias->size(0) == weight.size(0), "bias length must equal weight.shape[0]");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const at::Tensor x2 = x.reshape({-1, x.size(-1)}).contiguous();
  const int64_t m = x2.size(0), k = x2.size(1), n = weight.size(0);
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = n;
  at::Tensor y = at::empty({m, n}, x.options());
  zcutlass::GemmDesc desc{m, n, k, x2.stride(0), weight.stride(0), n, n, t, t, t, t, 1.0f, 0.0f,
                          bias.has_value() ? bias->data_ptr() : nullptr,
                          at::cuda::getCurrentCUDAStream().stream()};
  desc.b_layout = zcutlass::layout::LayoutKind::ColumnMajor;
  const zcutlass::Status status =
      zcutlass::gemm(desc, x2.data_ptr(), weight.data_ptr(), nullptr, y.data_ptr());
  TORCH_CHECK(status == zcutlass::Status::Success, "zcutlass::linear failed: ",
              zcutlass::status_to_string(status));
  return y.view(out_shape);
}

}  // namespace

TORCH_LIBRARY(zcutlass_torch, m) {
  m.def("gemm(Tensor A, Tensor B, Tensor? C=None, Tensor? bias=None, float alpha=1.0, float beta=0.0) -> Tensor");
}

TORCH_LIBRARY_IMPL(zcutlass_torch, CUDA, m) { m.impl("gemm", gemm_op); }

TORCH_LIBRARY(zcutlass, m) {
  m.def("gemm(Tensor A, Tensor B, Tensor? C=None, Tensor? bias=None, float alpha=1.0, float beta=0.0) -> Tensor");
  m.def("gemm_out(Tensor A, Tensor B, Tensor? C, Tensor? bias, float alpha, float beta, Tensor(a!) D) -> ()");
  m.def("linear(Tensor x, Tensor weight, Tensor? bias=None) -> Tensor");
}

TORCH_LIBRARY_IMPL(zcutlass, CUDA, m) {
  m.impl("gemm", gemm_op);
  m.impl("gemm_out", gemm_out_op);
  m.impl("linear", linear_op);
}
