// torch adapters for the sm_100a kernels: argument checks, stream/device selection and the
// Python module definition (vdn_minimax_h3_b200._C). The kernels themselves live in the
// .cu files behind the raw-pointer API of launchers.h.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "launchers.h"

namespace vdn {
namespace {

void check_2d_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16, got ", t.scalar_type());
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have a contiguous last dimension");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0, name, " row stride must be a multiple of 16 bytes");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned");
}

const float* opt_f32(const c10::optional<torch::Tensor>& t, int64_t n, const char* name) {
  if (!t) return nullptr;
  TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() &&
                  t->numel() == n,
              name, " must be a contiguous fp32 CUDA tensor of ", n, " elements");
  return t->data_ptr<float>();
}

int* err_ptr(const torch::Tensor& err) {
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt && err.numel() >= 1,
              "err must be an int32 CUDA tensor");
  return err.data_ptr<int>();
}

GemmArgs gemm_args(const torch::Tensor& A, const torch::Tensor& B) {
  check_2d_bf16(A, "A");
  check_2d_bf16(B, "B");
  TORCH_CHECK(A.size(1) == B.size(1), "K mismatch: A ", A.sizes(), " B ", B.sizes());
  TORCH_CHECK(A.size(1) % 8 == 0, "K must be a multiple of 8");
  GemmArgs a;
  a.A = A.data_ptr();
  a.B = B.data_ptr();
  a.lda = A.stride(0);
  a.ldb = B.stride(0);
  a.M = (int)A.size(0);
  a.N = (int)B.size(0);
  a.K = (int)A.size(1);
  return a;
}

}  // namespace

void gemm_bf16(torch::Tensor A, torch::Tensor B, torch::Tensor out,
               c10::optional<torch::Tensor> bias, bool accumulate, torch::Tensor err) {
  GemmArgs a = gemm_args(A, B);
  check_2d_bf16(out, "out");
  TORCH_CHECK(out.size(0) == a.M && out.size(1) == a.N, "out shape mismatch");
  c10::cuda::CUDAGuard g(A.device());
  launch_gemm_bf16(a, accumulate ? 3 : 0, out.data_ptr(), out.stride(0),
                   opt_f32(bias, a.N, "bias"), nullptr, 0, nullptr, err_ptr(err),
                   at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gemm_bf16_residual(torch::Tensor A, torch::Tensor B, torch::Tensor X,
                        c10::optional<torch::Tensor> bias, torch::Tensor gate,
                        torch::Tensor gate_idx, torch::Tensor err) {
  GemmArgs a = gemm_args(A, B);
  check_2d_bf16(X, "X");
  check_2d_bf16(gate, "gate");
  TORCH_CHECK(X.size(0) == a.M && X.size(1) == a.N, "X shape mismatch");
  TORCH_CHECK(gate.size(1) >= a.N, "gate table narrower than N");
  TORCH_CHECK(gate_idx.is_cuda() && gate_idx.scalar_type() == at::kInt &&
                  gate_idx.is_contiguous() && gate_idx.numel() >= a.M,
              "gate_idx must be contiguous int32 [M]");
  c10::cuda::CUDAGuard g(A.device());
  launch_gemm_bf16(a, 1, X.data_ptr(), X.stride(0), opt_f32(bias, a.N, "bias"),
                   gate.data_ptr(), gate.stride(0), gate_idx.data_ptr<int>(), err_ptr(err),
                   at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gemm_bf16_swiglu(torch::Tensor A, torch::Tensor B, torch::Tensor H,
                      c10::optional<torch::Tensor> bias, torch::Tensor err) {
  GemmArgs a = gemm_args(A, B);
  check_2d_bf16(H, "H");
  TORCH_CHECK(a.N % 256 == 0, "swiglu GEMM needs N % 256 == 0 (interleaved value|gate tiles)");
  TORCH_CHECK(H.size(0) == a.M && H.size(1) == a.N / 2, "H shape mismatch");
  c10::cuda::CUDAGuard g(A.device());
  launch_gemm_bf16(a, 2, H.data_ptr(), H.stride(0), opt_f32(bias, a.N, "bias"), nullptr, 0,
                   nullptr, err_ptr(err), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace vdn

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "VDN-H3 sm_100a kernels";
  m.def("gemm_bf16", &vdn::gemm_bf16, "bf16 tcgen05 GEMM: out (+)= A @ B^T (+ bias)");
  m.def("gemm_bf16_residual", &vdn::gemm_bf16_residual,
        "bf16 tcgen05 GEMM with gated-residual epilogue: X += gate[idx] * (A @ B^T + bias)");
  m.def("gemm_bf16_swiglu", &vdn::gemm_bf16_swiglu,
        "bf16 tcgen05 GEMM with SwiGLU epilogue over interleaved value|gate weight tiles");
}
