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

void check_2d_bytes(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.element_size() == 1 && t.dim() == 2 && t.stride(1) == 1, name,
              " must be a 2-D one-byte (E4M3) CUDA tensor with contiguous rows");
  TORCH_CHECK(t.stride(0) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " rows must be 16-byte aligned");
}
void check_sf(const torch::Tensor& t, int64_t nbytes, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.element_size() == 1 && t.is_contiguous() && t.numel() >= nbytes &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              name, " must be a contiguous 16-byte aligned byte tensor of >= ", nbytes, " bytes");
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

// out (+)= op(A) @ op(B)^T where a_mn means A is held as [K, M] and b_mn means B is held as
// [K, N] (the input / weight gradients of a Linear without transposed copies).
void gemm_bf16_layout(torch::Tensor A, torch::Tensor B, torch::Tensor out, bool a_mn, bool b_mn,
                      bool accumulate, torch::Tensor err) {
  check_2d_bf16(A, "A");
  check_2d_bf16(B, "B");
  check_2d_bf16(out, "out");
  GemmArgs a;
  a.A = A.data_ptr();
  a.B = B.data_ptr();
  a.lda = A.stride(0);
  a.ldb = B.stride(0);
  const int64_t M = a_mn ? A.size(1) : A.size(0), ka = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0), kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(ka == kb, "K mismatch: A ", A.sizes(), " B ", B.sizes(), " (a_mn ", a_mn,
              ", b_mn ", b_mn, ")");
  TORCH_CHECK(M < (1ll << 31) && N < (1ll << 31) && ka < (1ll << 31), "GEMM extent too large");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "out must be [", M, ", ", N, "], got ",
              out.sizes());
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)ka;
  if (a.K == 0) {
    if (!accumulate) out.zero_();
    return;
  }
  c10::cuda::CUDAGuard g(A.device());
  launch_gemm_bf16_layout(a, a_mn, b_mn, accumulate, out.data_ptr(), out.stride(0), err_ptr(err),
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

namespace {
GemmRoute build_route(int64_t M, int64_t N, const torch::Tensor& route,
                      const std::vector<int64_t>& route_ld, int64_t q0, int64_t q1, int64_t k0,
                      int64_t k1, const c10::optional<torch::Tensor>& norm_q,
                      const c10::optional<torch::Tensor>& norm_k, double qk_eps,
                      const c10::optional<torch::Tensor>& cosv,
                      const c10::optional<torch::Tensor>& sinv) {
  TORCH_CHECK(N % 8 == 0, "routed GEMM needs N % 8 == 0");
  TORCH_CHECK(route.is_cuda() && route.scalar_type() == at::kLong && route.is_contiguous() &&
                  route.dim() == 2 && route.size(1) == N / 8,
              "route must be a contiguous int64 CUDA tensor [planes, N/8]");
  const int planes = (int)route.size(0);
  TORCH_CHECK(planes >= 1 && planes <= 8 && (int)route_ld.size() == planes,
              "1..8 route planes, one row stride each");
  GemmRoute r{};
  r.route = reinterpret_cast<const long long*>(route.data_ptr<int64_t>());
  r.planes = planes;
  for (int i = 0; i < planes; ++i) {
    TORCH_CHECK(route_ld[i] % 8 == 0, "route row strides must be multiples of 8 elements");
    r.route_ld[i] = route_ld[i];
  }
  r.q0 = (int)q0;
  r.q1 = (int)q1;
  r.k0 = (int)k0;
  r.k1 = (int)k1;
  if (q1 > q0 || k1 > k0) {
    TORCH_CHECK(planes >= 2, "q/k processing needs plane 1 for the processed heads");
    TORCH_CHECK(q0 % 128 == 0 && q1 % 128 == 0 && k0 % 128 == 0 && k1 % 128 == 0 && q1 <= N &&
                    k1 <= N,
                "q/k column ranges must lie on 128-column head boundaries");
    TORCH_CHECK(norm_q && norm_k && cosv && sinv, "q/k processing needs norms and rope tables");
    for (const auto* t : {&*cosv, &*sinv}) {
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->dim() == 2 &&
                      t->size(0) >= M && t->size(1) == 128 && t->stride(1) == 1 &&
                      t->stride(0) % 4 == 0 &&
                      reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                  "rope tables must be fp32 [M, 128] with 16-byte aligned rows");
    }
    TORCH_CHECK(cosv->stride(0) == sinv->stride(0), "rope tables must share a row stride");
    r.norm_q = opt_f32(norm_q, 128, "norm_q");
    r.norm_k = opt_f32(norm_k, 128, "norm_k");
    r.qk_eps = (float)qk_eps;
    r.rope_cos = cosv->data_ptr<float>();
    r.rope_sin = sinv->data_ptr<float>();
    r.ld_rope = cosv->stride(0);
  }
  return r;
}
}  // namespace

void gemm_bf16_routed(torch::Tensor A, torch::Tensor B, c10::optional<torch::Tensor> bias,
                      torch::Tensor route, std::vector<int64_t> route_ld, int64_t q0, int64_t q1,
                      int64_t k0, int64_t k1, c10::optional<torch::Tensor> norm_q,
                      c10::optional<torch::Tensor> norm_k, double qk_eps,
                      c10::optional<torch::Tensor> cosv, c10::optional<torch::Tensor> sinv,
                      torch::Tensor err) {
  GemmArgs a = gemm_args(A, B);
  GemmRoute r = build_route(a.M, a.N, route, route_ld, q0, q1, k0, k1, norm_q, norm_k, qk_eps,
                            cosv, sinv);
  c10::cuda::CUDAGuard g(A.device());
  launch_gemm_bf16_routed(a, r, opt_f32(bias, a.N, "bias"), err_ptr(err),
                          at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


void gemm_fp8(torch::Tensor A, torch::Tensor B, torch::Tensor sfa, torch::Tensor sfb, int64_t mode,
              c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> bias,
              c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> gate_idx,
              c10::optional<torch::Tensor> q_out, c10::optional<torch::Tensor> q_sf,
              torch::Tensor err) {
  check_2d_bytes(A, "A");
  check_2d_bytes(B, "B");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K, "K mismatch");
  TORCH_CHECK(K % 128 == 0 && N % 32 == 0, "fp8 GEMM needs K % 128 == 0 and N % 32 == 0");
  check_sf(sfa, ((M + 127) / 128) * (K / 128) * 512, "sfa");
  check_sf(sfb, ((N + 255) / 256) * (K / 128) * 1024, "sfb");
  GemmFp8Args a{A.data_ptr(), B.data_ptr(), A.stride(0), B.stride(0), sfa.data_ptr(),
                sfb.data_ptr(), (int)M, (int)N, (int)K};
  void* op = nullptr;
  int64_t ldo = 0;
  const void* gp = nullptr;
  int64_t ldg = 0;
  const int* gi = nullptr;
  void* qp = nullptr;
  int64_t ldq = 0;
  void* qs = nullptr;
  if (mode == 0 || mode == 1) {
    TORCH_CHECK(out.has_value(), "out required");
    check_2d_bf16(*out, "out");
    TORCH_CHECK(out->size(0) == M && out->size(1) == N, "out shape mismatch");
    op = out->data_ptr();
    ldo = out->stride(0);
    if (mode == 1) {
      TORCH_CHECK(gate && gate_idx, "residual epilogue needs gate and gate_idx");
      check_2d_bf16(*gate, "gate");
      TORCH_CHECK(gate->size(1) >= N, "gate table narrower than N");
      TORCH_CHECK(gate_idx->is_cuda() && gate_idx->scalar_type() == at::kInt &&
                      gate_idx->is_contiguous() && gate_idx->numel() >= M,
                  "gate_idx must be contiguous int32 [M]");
      gp = gate->data_ptr();
      ldg = gate->stride(0);
      gi = gate_idx->data_ptr<int>();
    }
  } else if (mode == 2) {
    TORCH_CHECK(N % 256 == 0, "swiglu fp8 GEMM needs N % 256 == 0");
    TORCH_CHECK(q_out && q_sf, "swiglu fp8 GEMM needs q_out and q_sf");
    check_2d_bytes(*q_out, "q_out");
    TORCH_CHECK(q_out->size(0) == M && q_out->size(1) == N / 2, "q_out shape mismatch");
    check_sf(*q_sf, ((M + 127) / 128) * ((N / 2) / 128) * 512, "q_sf");
    qp = q_out->data_ptr();
    ldq = q_out->stride(0);
    qs = q_sf->data_ptr();
  } else {
    TORCH_CHECK(false, "unknown fp8 GEMM mode ", mode);
  }
  c10::cuda::CUDAGuard g(A.device());
  launch_gemm_fp8(a, (int)mode, op, ldo, opt_f32(bias, N, "bias"), gp, ldg, gi, qp, ldq, qs,
                  err_ptr(err), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gemm_fp8_routed(torch::Tensor A, torch::Tensor B, torch::Tensor sfa, torch::Tensor sfb,
                     c10::optional<torch::Tensor> bias, torch::Tensor route,
                     std::vector<int64_t> route_ld, int64_t q0, int64_t q1, int64_t k0, int64_t k1,
                     c10::optional<torch::Tensor> norm_q, c10::optional<torch::Tensor> norm_k,
                     double qk_eps, c10::optional<torch::Tensor> cosv,
                     c10::optional<torch::Tensor> sinv, torch::Tensor err) {
  check_2d_bytes(A, "A");
  check_2d_bytes(B, "B");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K, "K mismatch");
  TORCH_CHECK(K % 128 == 0 && N % 32 == 0, "fp8 GEMM needs K % 128 == 0 and N % 32 == 0");
  check_sf(sfa, ((M + 127) / 128) * (K / 128) * 512, "sfa");
  check_sf(sfb, ((N + 255) / 256) * (K / 128) * 1024, "sfb");
  GemmFp8Args a{A.data_ptr(), B.data_ptr(), A.stride(0), B.stride(0), sfa.data_ptr(),
                sfb.data_ptr(), (int)M, (int)N, (int)K};
  GemmRoute r = build_route(M, N, route, route_ld, q0, q1, k0, k1, norm_q, norm_k, qk_eps, cosv,
                            sinv);
  c10::cuda::CUDAGuard g(A.device());
  launch_gemm_fp8_routed(a, r, opt_f32(bias, N, "bias"), err_ptr(err),
                         at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void quant_rows(torch::Tensor x, torch::Tensor q, torch::Tensor sf) {
  check_2d_bf16(x, "x");
  check_2d_bytes(q, "q");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(q.size(0) == M && q.size(1) == K, "q shape mismatch");
  TORCH_CHECK(K % 128 == 0, "quantiser needs K % 128 == 0");
  check_sf(sf, ((M + 127) / 128) * (K / 128) * 512, "sf");
  c10::cuda::CUDAGuard g(x.device());
  launch_quant_rows(x.data_ptr(), x.stride(0), (int)M, (int)K, q.data_ptr(), q.stride(0),
                    sf.data_ptr(), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adaln_rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> w, double eps, torch::Tensor table,
                   int64_t shift_col, int64_t scale_col, torch::Tensor idx,
                   c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> q,
                   c10::optional<torch::Tensor> qsf) {
  check_2d_bf16(x, "x");
  check_2d_bf16(table, "table");
  const int T = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0, "hidden size must be a multiple of 8");
  TORCH_CHECK(out || q, "adaln_rmsnorm needs a bf16 and/or an E4M3 output");
  if (out) {
    check_2d_bf16(*out, "out");
    TORCH_CHECK(out->size(0) == T && out->size(1) == D, "out shape mismatch");
  }
  if (q) {
    TORCH_CHECK(D % 256 == 0, "the E4M3 output needs D % 256 == 0");
    check_2d_bytes(*q, "q");
    TORCH_CHECK(q->size(0) == T && q->size(1) == D, "q shape mismatch");
    TORCH_CHECK(qsf.has_value(), "the E4M3 output needs its scale-factor buffer");
    check_sf(*qsf, ((T + 127) / 128) * (D / 128) * 512, "qsf");
  }
  TORCH_CHECK(shift_col % 8 == 0 && scale_col % 8 == 0, "table columns must be 8-aligned");
  TORCH_CHECK(shift_col + D <= table.size(1) && scale_col + D <= table.size(1), "table too narrow");
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt && idx.is_contiguous() &&
                  idx.numel() >= T, "idx must be contiguous int32 [T]");
  c10::cuda::CUDAGuard g(x.device());
  const float* wp = opt_f32(w, D, "w");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(wp) % 16 == 0, "norm weight must be 16-byte aligned");
  launch_adaln_rmsnorm(x.data_ptr(), x.stride(0), wp, (float)eps, table.data_ptr(),
                       table.stride(0), (int)shift_col, (int)scale_col, idx.data_ptr<int>(),
                       out ? out->data_ptr() : nullptr, out ? out->stride(0) : 0, T, D,
                       at::cuda::getCurrentCUDAStream(), q ? q->data_ptr() : nullptr,
                       q ? q->stride(0) : 0, q ? qsf->data_ptr() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adaln_rmsnorm_dst(torch::Tensor x, c10::optional<torch::Tensor> w, double eps,
                       torch::Tensor table, int64_t shift_col, int64_t scale_col, torch::Tensor idx,
                       int64_t row0, std::vector<torch::Tensor> outs, std::vector<torch::Tensor> qs,
                       std::vector<torch::Tensor> sfs) {
  check_2d_bf16(x, "x");
  check_2d_bf16(table, "table");
  const int T = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 256 == 0, "adaln_rmsnorm_dst needs D % 256 == 0");
  TORCH_CHECK(outs.size() <= 2 && qs.size() <= 2 && qs.size() == sfs.size() &&
                  (outs.size() + qs.size()) > 0,
              "one or two bf16 and/or E4M3 destinations");
  NormDst dst{};
  dst.row0 = row0;
  for (size_t i = 0; i < outs.size(); ++i) {
    check_2d_bf16(outs[i], "out");
    TORCH_CHECK(outs[i].size(1) == D && outs[i].size(0) >= row0 + T, "out too small");
    TORCH_CHECK(i == 0 || outs[i].stride(0) == outs[0].stride(0), "outs share a row stride");
    dst.out[i] = reinterpret_cast<__nv_bfloat16*>(outs[i].data_ptr());
    dst.ldo = outs[i].stride(0);
  }
  for (size_t i = 0; i < qs.size(); ++i) {
    check_2d_bytes(qs[i], "q");
    TORCH_CHECK(qs[i].size(1) == D && qs[i].size(0) >= row0 + T, "q too small");
    TORCH_CHECK(i == 0 || qs[i].stride(0) == qs[0].stride(0), "qs share a row stride");
    check_sf(sfs[i], ((qs[i].size(0) + 127) / 128) * (D / 128) * 512, "sf");
    dst.q[i] = reinterpret_cast<uint8_t*>(qs[i].data_ptr());
    dst.qsf[i] = reinterpret_cast<uint8_t*>(sfs[i].data_ptr());
    dst.ldq = qs[i].stride(0);
  }
  TORCH_CHECK(shift_col % 8 == 0 && scale_col % 8 == 0, "table columns must be 8-aligned");
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt && idx.is_contiguous() &&
                  idx.numel() >= T, "idx must be contiguous int32 [T]");
  c10::cuda::CUDAGuard g(x.device());
  const float* wp = opt_f32(w, D, "w");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(wp) % 16 == 0, "norm weight must be 16-byte aligned");
  launch_adaln_rmsnorm_dst(x.data_ptr(), x.stride(0), wp, (float)eps, table.data_ptr(),
                           table.stride(0), (int)shift_col, (int)scale_col, idx.data_ptr<int>(),
                           dst, T, D, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gemm_f32_scatter(torch::Tensor A, torch::Tensor B, c10::optional<torch::Tensor> sfa,
                      c10::optional<torch::Tensor> sfb, torch::Tensor out,
                      std::vector<int64_t> bases, int64_t row0, int64_t rows, torch::Tensor err) {
  // bf16 partial products stored to their row owners (bf16 operands, or E4M3 with sfa/sfb)
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 &&
                  out.stride(1) == 1 && out.stride(0) % 8 == 0,
              "out must be bf16 2-D with 16-byte aligned rows");
  RowScatter sc{};
  TORCH_CHECK(bases.size() <= (size_t)kMaxScatterRanks, "at most 8 owners");
  sc.n = (int)bases.size();
  for (size_t i = 0; i < bases.size(); ++i) {
    TORCH_CHECK(bases[i] % 16 == 0, "scatter destinations must be 16-byte aligned");
    sc.base[i] = reinterpret_cast<__nv_bfloat16*>(bases[i]);
  }
  sc.row0 = row0;
  sc.rows_per_rank = (int)rows;
  c10::cuda::CUDAGuard g(A.device());
  if (sfa) {
    check_2d_bytes(A, "A");
    check_2d_bytes(B, "B");
    const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
    TORCH_CHECK(K % 128 == 0 && N % 32 == 0 && B.size(1) == K, "fp8 shapes");
    TORCH_CHECK(sc.n || (out.size(0) == M && out.size(1) == N), "out shape mismatch");
    check_sf(*sfa, ((M + 127) / 128) * (K / 128) * 512, "sfa");
    check_sf(*sfb, ((N + 255) / 256) * (K / 128) * 1024, "sfb");
    GemmFp8Args a{A.data_ptr(), B.data_ptr(), A.stride(0), B.stride(0), sfa->data_ptr(),
                  sfb->data_ptr(), (int)M, (int)N, (int)K};
    launch_gemm_fp8_f32_scatter(a, out.data_ptr(), out.stride(0), sc, err_ptr(err),
                                at::cuda::getCurrentCUDAStream());
  } else {
    GemmArgs a = gemm_args(A, B);
    TORCH_CHECK(a.N % 32 == 0, "N % 32 == 0");
    TORCH_CHECK(sc.n || (out.size(0) == a.M && out.size(1) == a.N), "out shape mismatch");
    launch_gemm_bf16_f32_scatter(a, out.data_ptr(), out.stride(0), sc, err_ptr(err),
                                 at::cuda::getCurrentCUDAStream());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void residual_combine(torch::Tensor x, torch::Tensor a, torch::Tensor b,
                      c10::optional<torch::Tensor> bias, torch::Tensor gate, torch::Tensor idx) {
  check_2d_bf16(x, "x");
  check_2d_bf16(gate, "gate");
  const int R = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0, "D % 8 == 0");
  for (const auto* t : {&a, &b}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 &&
                    t->size(0) >= R && t->size(1) == D && t->stride(1) == 1 &&
                    t->stride(0) == a.stride(0) && t->stride(0) % 8 == 0,
                "partials must be bf16 [>=R, D] with one 16-byte aligned row stride");
  }
  TORCH_CHECK(gate.size(1) >= D, "gate table narrower than D");
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt && idx.is_contiguous() &&
                  idx.numel() >= R, "idx must be contiguous int32 [R]");
  c10::cuda::CUDAGuard g(x.device());
  launch_residual_combine(x.data_ptr(), x.stride(0), a.data_ptr(), b.data_ptr(),
                          a.stride(0), opt_f32(bias, D, "bias"), gate.data_ptr(), gate.stride(0),
                          idx.data_ptr<int>(), R, D, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// peers: optional addresses (int64) of the peers' fp32 slot arrays; the sums go to
// peers[p] + slot_offset (elements) instead of `out`, frames outside this shard skipped.
void frame_sums(torch::Tensor x, int64_t row0, int64_t video_start, int64_t F, int64_t S,
                torch::Tensor out, std::vector<int64_t> peers, int64_t slot_offset) {
  check_2d_bf16(x, "x");
  const int D = x.size(1);
  TORCH_CHECK(D % 8 == 0, "D must be a multiple of 8");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() &&
                  out.numel() == F * D, "out must be contiguous fp32 [F, D]");
  TORCH_CHECK((int)peers.size() <= kMaxScatterRanks, "at most 8 peer destinations");
  FrameSumDst dst{};
  dst.n = (int)peers.size();
  dst.offset = slot_offset;
  for (int p = 0; p < dst.n; ++p) dst.base[p] = reinterpret_cast<float*>(peers[p]);
  c10::cuda::CUDAGuard g(x.device());
  launch_frame_sums(x.data_ptr(), x.stride(0), row0, x.size(0), video_start, (int)F, (int)S, D,
                    out.data_ptr<float>(), at::cuda::getCurrentCUDAStream(), &dst);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_prep(torch::Tensor src, int64_t H, torch::Tensor w, double eps, torch::Tensor cosv,
             torch::Tensor sinv, torch::Tensor out) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.dim() == 2 &&
                  src.stride(1) == 1, "src must be bf16 [T, H*d] with contiguous rows");
  check_2d_bf16(out, "out");
  const int T = src.size(0);
  const int d = src.size(1) / H;
  TORCH_CHECK(d * H == src.size(1) && d % 2 == 0 && d <= 256, "bad head_dim");
  TORCH_CHECK(src.stride(0) % 2 == 0, "src row stride must be even");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kFloat && w.numel() == d, "w fp32 [d]");
  TORCH_CHECK(cosv.scalar_type() == at::kFloat && sinv.scalar_type() == at::kFloat &&
                  cosv.is_contiguous() && sinv.is_contiguous() && cosv.size(0) >= T,
              "cos/sin must be contiguous fp32 [T, rot]");
  const int rot = cosv.size(1);
  TORCH_CHECK(rot <= d && rot % 2 == 0, "rotary dim must be even and <= head_dim");
  c10::cuda::CUDAGuard g(src.device());
  launch_qk_prep(src.data_ptr(), src.stride(0), T, (int)H, d, w.data_ptr<float>(), (float)eps,
                 cosv.data_ptr<float>(), sinv.data_ptr<float>(), rot, out.data_ptr(),
                 out.stride(0), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


namespace {
void check_heads(const torch::Tensor& t, const char* name, int64_t T, int64_t H) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 3, name,
              " must be a bf16 CUDA [T, H, d] tensor");
  TORCH_CHECK(t.size(0) == T && t.size(1) == H && t.size(2) == 128, name,
              " must be [T, H, 128], got ", t.sizes());
  TORCH_CHECK(t.stride(2) == 1 && t.stride(1) == 128, name,
              " must have contiguous heads (stride(1)=128, stride(2)=1)");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              name, " row stride / base must be 16-byte aligned");
}
}  // namespace

namespace {
// Row-owner scatter from Python: one base address per owner rank (the owner's buffer at
// row 0 and this producer's first column), the packed row of output row 0, the shard
// height. An empty base list means no scatter.
RowScatter make_scatter(const std::vector<int64_t>& base, int64_t row0, int64_t rows) {
  RowScatter sc{};
  TORCH_CHECK(base.size() <= (size_t)kMaxScatterRanks, "at most 8 scatter ranks");
  sc.n = (int)base.size();
  for (size_t i = 0; i < base.size(); ++i) {
    TORCH_CHECK(base[i] % 16 == 0, "scatter destinations must be 16-byte aligned");
    sc.base[i] = reinterpret_cast<__nv_bfloat16*>(base[i]);
  }
  sc.row0 = row0;
  sc.rows_per_rank = (int)rows;
  TORCH_CHECK(sc.n == 0 || rows > 0, "scatter needs a positive shard height");
  return sc;
}

void check_out_or_scatter(const torch::Tensor& out, const RowScatter& sc, int64_t ld,
                          int64_t rows, int64_t cols) {
  check_2d_bf16(out, "out");
  if (sc.n == 0) {
    TORCH_CHECK(out.size(0) == rows && out.size(1) == cols, "out must be [", rows, ", ", cols, "]");
  } else {
    TORCH_CHECK(out.stride(0) == ld && ld % 8 == 0, "scatter row stride must match out's");
  }
}
}  // namespace

void window_attention(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor tiles,
                      torch::Tensor kv, c10::optional<torch::Tensor> gate, torch::Tensor out,
                      double scale, torch::Tensor err, std::vector<int64_t> scatter_base,
                      int64_t scatter_row0, int64_t scatter_rows,
                      c10::optional<torch::Tensor> trace, c10::optional<torch::Tensor> lse) {
  const int64_t T = q.size(0), H = q.size(1);
  if (lse)
    TORCH_CHECK(lse->is_cuda() && lse->scalar_type() == at::kFloat && lse->is_contiguous() &&
                    lse->numel() == H * T, "lse must be contiguous fp32 [H, T]");
  check_heads(q, "q", T, H);
  check_heads(k, "k", T, H);
  check_heads(v, "v", T, H);
  const RowScatter sc = make_scatter(scatter_base, scatter_row0, scatter_rows);
  check_out_or_scatter(out, sc, out.stride(0), T, H * 128);
  if (trace)
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                    trace->numel() >= 12 * 64 + 4,
                "trace must be a contiguous int64 CUDA tensor of >= 772 entries");
  TORCH_CHECK(tiles.is_cuda() && tiles.scalar_type() == at::kInt && tiles.is_contiguous() &&
                  tiles.dim() == 2 && tiles.size(1) == 4, "tiles must be int32 [n, 4]");
  TORCH_CHECK(kv.is_cuda() && kv.scalar_type() == at::kInt && kv.is_contiguous() &&
                  kv.dim() == 2 && kv.size(1) == 8, "kv must be int32 [n_seg, 8]");
  const void* gp = nullptr;
  int64_t ldg = 0;
  if (gate) {
    TORCH_CHECK(gate->is_cuda() && gate->scalar_type() == at::kBFloat16 && gate->dim() == 2 &&
                    gate->size(0) == T && gate->size(1) == H && gate->stride(1) == 1,
                "gate logits must be bf16 [T, H] with contiguous heads");
    gp = gate->data_ptr();
    ldg = gate->stride(0);
  }
  c10::cuda::CUDAGuard g(q.device());
  launch_window_attention(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(),
                          v.stride(0), (int)T, (int)H, tiles.data_ptr<int>(), (int)tiles.size(0),
                          kv.data_ptr<int>(), gp, ldg, out.data_ptr(), out.stride(0),
                          (float)scale, err_ptr(err), at::cuda::getCurrentCUDAStream(), &sc,
                          trace ? reinterpret_cast<long long*>(trace->data_ptr<int64_t>()) : nullptr,
                          lse ? lse->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Window-attention backward: gradients of q, k, v (ungated attention) from dout, the
// forward output o and its lse; delta [H, T] is scratch the dq pass fills for the dkv pass.
void window_attention_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                          torch::Tensor dout, torch::Tensor lse, torch::Tensor delta,
                          torch::Tensor dq, torch::Tensor dk, torch::Tensor dv,
                          torch::Tensor q_tiles, torch::Tensor kv_ranges, torch::Tensor k_tiles,
                          torch::Tensor q_ranges, double scale, torch::Tensor err) {
  const int64_t T = q.size(0), H = q.size(1);
  for (auto* t : {&q, &k, &v, &o, &dout, &dq, &dk, &dv}) check_heads(*t, "attention tensor", T, H);
  TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous() &&
                  lse.numel() == H * T, "lse must be contiguous fp32 [H, T]");
  TORCH_CHECK(delta.is_cuda() && delta.scalar_type() == at::kFloat && delta.is_contiguous() &&
                  delta.numel() == H * T, "delta must be contiguous fp32 [H, T]");
  for (auto* t : {&q_tiles, &k_tiles})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kInt && t->is_contiguous() && t->dim() == 2 &&
                    t->size(1) == 4, "tiles must be int32 [n, 4]");
  for (auto* t : {&kv_ranges, &q_ranges})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kInt && t->is_contiguous() && t->dim() == 2 &&
                    t->size(1) == 8, "ranges must be int32 [n_seg, 8]");
  AttnBwdArgs a{};
  a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr(); a.o = o.data_ptr(); a.dout = dout.data_ptr();
  a.ldq = q.stride(0); a.ldk = k.stride(0); a.ldv = v.stride(0); a.ldo = o.stride(0); a.lddo = dout.stride(0);
  a.dq = dq.data_ptr(); a.dk = dk.data_ptr(); a.dv = dv.data_ptr();
  a.lddq = dq.stride(0); a.lddk = dk.stride(0); a.lddv = dv.stride(0);
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.T = (int)T;
  a.H = (int)H;
  a.q_tiles = q_tiles.data_ptr<int>();
  a.n_q_tiles = (int)q_tiles.size(0);
  a.kv_ranges = kv_ranges.data_ptr<int>();
  a.k_tiles = k_tiles.data_ptr<int>();
  a.n_k_tiles = (int)k_tiles.size(0);
  a.q_ranges = q_ranges.data_ptr<int>();
  a.scale = (float)scale;
  a.err = err_ptr(err);
  c10::cuda::CUDAGuard g(q.device());
  launch_attention_bwd(a, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


namespace {
// [N, H, 128] bf16 view with contiguous heads -> (base, row stride)
void check_rows_heads(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be bf16 CUDA");
  TORCH_CHECK(t.dim() == 3 && t.size(2) == 128 && t.stride(2) == 1 && t.stride(1) == 128, name,
              " must be [N, H, 128] with contiguous heads");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              name, " row stride / base must be 16-byte aligned");
}
void check_f32(const torch::Tensor& t, const char* name, int64_t numel) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == numel,
              name, " must be a contiguous fp32 CUDA tensor of ", numel, " elements, got ", t.sizes());
}
cudaStream_t cur() { return at::cuda::getCurrentCUDAStream(); }
}  // namespace

void lb_activate(torch::Tensor in, torch::Tensor out, bool l2) {
  check_rows_heads(in, "in");
  check_rows_heads(out, "out");
  TORCH_CHECK(in.sizes() == out.sizes(), "shape mismatch");
  c10::cuda::CUDAGuard g(in.device());
  launch_lb_activate(in.data_ptr(), in.stride(0), in.size(0), in.size(1), out.data_ptr(),
                     out.stride(0), l2, cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lb_conv_features(torch::Tensor in, torch::Tensor wsp, torch::Tensor wtm, torch::Tensor out,
                      int64_t F, int64_t gh, int64_t gw, bool l2, torch::Tensor err,
                      c10::optional<torch::Tensor> tmp) {
  check_rows_heads(in, "in");
  check_rows_heads(out, "out");
  const int64_t H = in.size(1);
  TORCH_CHECK(in.size(0) == F * gh * gw, "rows != F * gh * gw");
  check_f32(wsp, "w_spatial", H * 128 * 25);
  check_f32(wtm, "w_temporal", H * 128 * 5);
  c10::cuda::CUDAGuard g(in.device());
  if (tmp) {
    // two passes through a bf16 intermediate of the output's shape
    check_rows_heads(*tmp, "tmp");
    TORCH_CHECK(tmp->size(0) == in.size(0) && tmp->size(1) == H, "tmp must match in");
    launch_lb_conv2(in.data_ptr(), in.stride(0), wsp.data_ptr<float>(), wtm.data_ptr<float>(),
                    tmp->data_ptr(), tmp->stride(0), out.data_ptr(), out.stride(0), (int)F,
                    (int)gh, (int)gw, (int)H, l2, err_ptr(err), cur());
  } else {
    launch_lb_conv(in.data_ptr(), in.stride(0), wsp.data_ptr<float>(), wtm.data_ptr<float>(),
                   out.data_ptr(), out.stride(0), (int)F, (int)gh, (int)gw, (int)H, l2,
                   err_ptr(err), cur());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Backward of the AdaLN-modulated RMSNorm: x / dy / dx [T, D] bf16 rows (16-byte aligned),
// w fp32 [D] or None, table bf16 [n, >= scale_col + D] with 16-byte aligned rows, idx int32 [T].
void adaln_rmsnorm_bwd(torch::Tensor x, torch::Tensor dy, c10::optional<torch::Tensor> w,
                       double eps, torch::Tensor table, int64_t scale_col, torch::Tensor idx,
                       torch::Tensor dx) {
  for (const torch::Tensor* t : {&x, &dy, &dx}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 &&
                    t->stride(1) == 1 && (t->stride(0) * 2) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "x, dy, dx must be bf16 CUDA [T, D] with 16-byte aligned rows");
    TORCH_CHECK(t->sizes() == x.sizes(), "x, dy, dx must have one shape");
  }
  const int64_t T = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0, "D must be a multiple of 8");
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kBFloat16 && table.dim() == 2 &&
                  table.stride(1) == 1 && (table.stride(0) * 2) % 16 == 0 && scale_col % 8 == 0 &&
                  scale_col + D <= table.size(1) &&
                  reinterpret_cast<uintptr_t>(table.data_ptr()) % 16 == 0,
              "table must be bf16 CUDA [n, >= scale_col + D], aligned rows and column");
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt && idx.is_contiguous() &&
                  idx.numel() == T, "idx must be int32 CUDA [T]");
  const float* wp = nullptr;
  if (w) {
    check_f32(*w, "w", D);
    wp = w->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(x.device());
  launch_adaln_rmsnorm_bwd(x.data_ptr(), x.stride(0), dy.data_ptr(), dy.stride(0), wp, (float)eps,
                           table.data_ptr(), table.stride(0), (int)scale_col, idx.data_ptr<int>(),
                           dx.data_ptr(), dx.stride(0), (int)T, (int)D, cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Backward of the two-pass short conv: in / tmp / dy / dx [N, H, 128] bf16 rows (N = F*gh*gw),
// wsp [25 * C] and wtm [C * 5] fp32 as given to the forward, dtmp fp32 scratch [N * C],
// dwsp / dwtm fp32 accumulators of the weights' shapes (zeroed by the caller).
void lb_conv_features_bwd(torch::Tensor in, torch::Tensor tmp, torch::Tensor dy, torch::Tensor wsp,
                          torch::Tensor wtm, torch::Tensor dtmp, torch::Tensor dx,
                          torch::Tensor dwsp, torch::Tensor dwtm, int64_t F, int64_t gh,
                          int64_t gw, bool l2) {
  check_rows_heads(in, "in");
  check_rows_heads(tmp, "tmp");
  check_rows_heads(dy, "dy");
  check_rows_heads(dx, "dx");
  const int64_t H = in.size(1), N = in.size(0), C = H * 128;
  TORCH_CHECK(N == F * gh * gw, "rows != F * gh * gw");
  TORCH_CHECK(tmp.sizes() == in.sizes() && dy.sizes() == in.sizes() && dx.sizes() == in.sizes(),
              "in, tmp, dy, dx must have one shape");
  check_f32(wsp, "w_spatial", C * 25);
  check_f32(wtm, "w_temporal", C * 5);
  check_f32(dtmp, "dtmp", N * C);
  check_f32(dwsp, "dw_spatial", C * 25);
  check_f32(dwtm, "dw_temporal", C * 5);
  c10::cuda::CUDAGuard g(in.device());
  launch_lb_conv2_bwd(in.data_ptr(), in.stride(0), tmp.data_ptr(), tmp.stride(0), dy.data_ptr(),
                      dy.stride(0), wsp.data_ptr<float>(), wtm.data_ptr<float>(),
                      dtmp.data_ptr<float>(), dx.data_ptr(), dx.stride(0), dwsp.data_ptr<float>(),
                      dwtm.data_ptr<float>(), (int)F, (int)gh, (int)gw, (int)H, l2, cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lb_frame_stats(torch::Tensor k, torch::Tensor v, torch::Tensor beta, torch::Tensor A,
                    torch::Tensor B, torch::Tensor err) {
  // k, v: [F, S, H, 128] views whose (F, S) rows are one row stride apart
  TORCH_CHECK(k.dim() == 4 && v.dim() == 4 && k.sizes() == v.sizes(), "k, v must be [F, S, H, 128]");
  const int64_t F = k.size(0), S = k.size(1), H = k.size(2);
  TORCH_CHECK(k.stride(0) == S * k.stride(1) && v.stride(0) == S * v.stride(1),
              "frames must be consecutive rows");
  check_rows_heads(k.view({F * S, H, 128}), "k");
  check_rows_heads(v.view({F * S, H, 128}), "v");
  check_f32(beta, "beta", F * S * H);
  check_f32(A, "A", F * H * 16384);
  check_f32(B, "B", F * H * 16384);
  c10::cuda::CUDAGuard g(k.device());
  launch_lb_frame_stats(k.data_ptr(), k.stride(1), v.data_ptr(), v.stride(1), (int)F, (int)S,
                        (int)H, beta.data_ptr<float>(), A.data_ptr<float>(), B.data_ptr<float>(),
                        err_ptr(err), cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lb_spd_factor(torch::Tensor A, torch::Tensor B, torch::Tensor alpha, torch::Tensor trans,
                   torch::Tensor inj, double a_scale, double b_scale, torch::Tensor err) {
  const int64_t n = A.numel() / 16384;
  TORCH_CHECK(A.size(-1) == 128 && A.size(-2) == 128, "A must be [..., 128, 128]");
  check_f32(A, "A", n * 16384);
  check_f32(B, "B", n * 16384);
  check_f32(alpha, "alpha", n * 128);
  check_f32(trans, "trans", n * 16384);
  check_f32(inj, "inj", n * 16384);
  c10::cuda::CUDAGuard g(A.device());
  launch_lb_spd_factor(A.data_ptr<float>(), B.data_ptr<float>(), alpha.data_ptr<float>(),
                       trans.data_ptr<float>(), inj.data_ptr<float>(), (int)n, (float)a_scale,
                       (float)b_scale, cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// suffix = None runs the prefix recurrence only (one direction).
void lb_scan(torch::Tensor trans, torch::Tensor inj, c10::optional<torch::Tensor> start,
             torch::Tensor prefix, c10::optional<torch::Tensor> suffix, torch::Tensor err) {
  TORCH_CHECK(trans.dim() == 4 && trans.size(2) == 128 && trans.size(3) == 128, "trans [F,H,128,128]");
  const int64_t F = trans.size(0), H = trans.size(1);
  check_f32(trans, "trans", F * H * 16384);
  check_f32(inj, "inj", F * H * 16384);
  check_f32(prefix, "prefix", F * H * 16384);
  float* qp = nullptr;
  if (suffix) {
    check_f32(*suffix, "suffix", F * H * 16384);
    qp = suffix->data_ptr<float>();
  }
  const float* sp = nullptr;
  if (start) {
    check_f32(*start, "start", H * 16384);
    sp = start->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(trans.device());
  launch_lb_scan(trans.data_ptr<float>(), inj.data_ptr<float>(), sp, (int)F, (int)H,
                 prefix.data_ptr<float>(), qp, err_ptr(err), cur(), suffix ? 2 : 1);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lb_gather(torch::Tensor prefix, torch::Tensor suffix, torch::Tensor idx, torch::Tensor ab,
               torch::Tensor aa, c10::optional<torch::Tensor> start, torch::Tensor out) {
  const int64_t F = prefix.size(0), H = prefix.size(1);
  check_f32(prefix, "prefix", F * H * 16384);
  check_f32(suffix, "suffix", F * H * 16384);
  check_f32(ab, "alpha_before", F * H * 128);
  check_f32(aa, "alpha_after", F * H * 128);
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt && idx.is_contiguous() &&
                  idx.numel() == F * 4, "idx must be int32 [F, 4]");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
                  out.numel() == F * H * 16384, "out must be contiguous bf16 [F, H, 128, 128]");
  const float* sp = nullptr;
  if (start) {
    check_f32(*start, "start", H * 16384);
    sp = start->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(prefix.device());
  launch_lb_gather(prefix.data_ptr<float>(), suffix.data_ptr<float>(), idx.data_ptr<int>(),
                   ab.data_ptr<float>(), aa.data_ptr<float>(), sp, (int)F, (int)H, out.data_ptr(),
                   cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void lb_readout(torch::Tensor q, torch::Tensor state, torch::Tensor w, torch::Tensor gate,
                torch::Tensor out, double eps, bool gate_logits, torch::Tensor err,
                std::vector<int64_t> scatter_base, int64_t scatter_row0, int64_t scatter_rows) {
  TORCH_CHECK(q.dim() == 4, "q must be [F, S, H, 128]");
  const int64_t F = q.size(0), S = q.size(1), H = q.size(2);
  TORCH_CHECK(q.stride(0) == S * q.stride(1), "q frames must be consecutive rows");
  check_rows_heads(q.view({F * S, H, 128}), "q");
  TORCH_CHECK(state.is_cuda() && state.scalar_type() == at::kBFloat16 && state.is_contiguous() &&
                  state.numel() == F * H * 16384, "state must be contiguous bf16 [F, H, 128, 128]");
  check_f32(w, "norm weight", 128);
  TORCH_CHECK(gate.dim() == 3 && gate.size(0) == F * S && gate.size(1) == H, "gate [F*S, H, 128]");
  check_rows_heads(gate, "gate");
  const RowScatter sc = make_scatter(scatter_base, scatter_row0, scatter_rows);
  check_out_or_scatter(out, sc, out.stride(0), F * S, H * 128);
  c10::cuda::CUDAGuard g(q.device());
  launch_lb_readout(q.data_ptr(), q.stride(1), state.data_ptr(), (int)F, (int)S, (int)H,
                    w.data_ptr<float>(), gate.data_ptr(), gate.stride(0), gate_logits,
                    out.data_ptr(), out.stride(0), (float)eps, err_ptr(err), cur(), &sc);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace vdn

// ---------------------------------------------------------------- symmetric memory
namespace vdn {

py::tuple symm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  char handle[64];
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  void* p = symm_malloc((size_t)nbytes, handle);
  return py::make_tuple((int64_t)reinterpret_cast<uintptr_t>(p), py::bytes(handle, 64));
}

int64_t symm_open_handle(py::bytes handle, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  std::string h = handle;
  TORCH_CHECK(h.size() == 64, "IPC handle must be 64 bytes");
  return (int64_t)reinterpret_cast<uintptr_t>(symm_open(h.data()));
}

void symm_close_handle(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  symm_close(reinterpret_cast<void*>(ptr));
}

void symm_free_ptr(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  symm_free(reinterpret_cast<void*>(ptr));
}

torch::Tensor bytes_at(int64_t ptr, int64_t nbytes, int64_t device) {
  // A non-owning uint8 tensor over [ptr, ptr + nbytes) on `device` (local or peer memory
  // mapped into this process). The region's owner controls its lifetime.
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), {nbytes}, [](void*) {}, opts);
}

// out = scale * sum_p srcs[p][offset : offset + out.numel()] (fp32; srcs are the ranks'
// copies of one symmetric buffer, as int64 addresses on out's device).
void symm_reduce_scatter(std::vector<int64_t> srcs, int64_t offset, torch::Tensor out,
                         double scale) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous(),
              "out must be a contiguous fp32 CUDA tensor");
  std::vector<const float*> p;
  for (auto a : srcs) p.push_back(reinterpret_cast<const float*>(a));
  c10::cuda::CUDAGuard g(out.device());
  launch_symm_reduce_scatter(p.data(), (int)p.size(), offset, out.numel(), (float)scale,
                             out.data_ptr<float>(), at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[q * shard_bytes, (q + 1) * shard_bytes) = the shard at srcs[q], for every rank q != rank.
void symm_all_gather(std::vector<int64_t> srcs, int64_t rank, torch::Tensor out, int64_t shard_bytes) {
  TORCH_CHECK(out.is_cuda() && out.is_contiguous(), "out must be a contiguous CUDA tensor");
  const int P = (int)srcs.size();
  TORCH_CHECK((int64_t)out.numel() * out.element_size() >= (int64_t)P * shard_bytes,
              "out is smaller than ranks x shard_bytes");
  std::vector<const void*> p;
  for (auto a : srcs) p.push_back(reinterpret_cast<const void*>(a));
  c10::cuda::CUDAGuard g(out.device());
  launch_symm_all_gather(p.data(), P, (int)rank, shard_bytes, out.data_ptr(),
                         at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void symm_barrier(int64_t counter, int64_t local_flags, torch::Tensor peer_flags, int64_t rank,
                  int64_t timeout_ns, torch::Tensor err) {
  TORCH_CHECK(peer_flags.is_cuda() && peer_flags.scalar_type() == at::kLong &&
                  peer_flags.is_contiguous(), "peer_flags must be int64 CUDA [P]");
  const int P = (int)peer_flags.numel();
  TORCH_CHECK(rank >= 0 && rank < P, "rank out of range");
  c10::cuda::CUDAGuard g(peer_flags.device());
  launch_symm_barrier(reinterpret_cast<unsigned long long*>(counter),
                      reinterpret_cast<unsigned long long*>(local_flags),
                      reinterpret_cast<unsigned long long* const*>(peer_flags.data_ptr<int64_t>()),
                      (int)rank, P, (long long)timeout_ns, err_ptr(err),
                      at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace vdn

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("symm_alloc", &vdn::symm_alloc, "cudaMalloc + IPC handle: (ptr, handle bytes)");
  m.def("symm_open", &vdn::symm_open_handle, "map a peer's IPC handle: ptr");
  m.def("symm_close", &vdn::symm_close_handle, "unmap a peer region");
  m.def("symm_free", &vdn::symm_free_ptr, "free this rank's region");
  m.def("bytes_at", &vdn::bytes_at, "non-owning uint8 tensor over device memory");
  m.def("symm_barrier", &vdn::symm_barrier, "bounded all-ranks flag barrier over peer memory");
  m.doc() = "VDN-H3 sm_100a kernels";
  m.def("gemm_bf16", &vdn::gemm_bf16, "bf16 tcgen05 GEMM: out (+)= A @ B^T (+ bias)");
  m.def("gemm_bf16_layout", &vdn::gemm_bf16_layout,
        "bf16 tcgen05 GEMM with MN-major operands: out (+)= op(A) @ op(B)^T",
        py::arg("A"), py::arg("B"), py::arg("out"), py::arg("a_mn"), py::arg("b_mn"),
        py::arg("accumulate"), py::arg("err"));
  m.def("gemm_bf16_residual", &vdn::gemm_bf16_residual,
        "bf16 tcgen05 GEMM with gated-residual epilogue: X += gate[idx] * (A @ B^T + bias)");
  m.def("gemm_bf16_swiglu", &vdn::gemm_bf16_swiglu,
        "bf16 tcgen05 GEMM with SwiGLU epilogue over interleaved value|gate weight tiles");
  m.def("gemm_bf16_routed", &vdn::gemm_bf16_routed,
        "bf16 tcgen05 GEMM whose epilogue scatters 8-column groups through a route table and "
        "applies QK RMSNorm + RoPE to the q/k heads");
  m.def("gemm_fp8", &vdn::gemm_fp8,
        "block-scaled E4M3 tcgen05 GEMM (UE8M0 scale factors in TMEM); epilogue modes 0 store, "
        "1 gated residual, 2 swiglu -> E4M3 + scale factors");
  m.def("gemm_fp8_routed", &vdn::gemm_fp8_routed,
        "block-scaled E4M3 GEMM with the routed epilogue (column routes, QK-norm + RoPE)");
  m.def("quant_rows", &vdn::quant_rows, "bf16 rows -> E4M3 with one UE8M0 scale per 1x128 block");
  m.def("adaln_rmsnorm_dst", &vdn::adaln_rmsnorm_dst,
        "AdaLN-RMSNorm into up to two destinations (local + peer) at a row offset, bf16 and/or E4M3");
  m.def("gemm_f32_scatter", &vdn::gemm_f32_scatter,
        "GEMM whose bf16 partial rows go to their owners (row-parallel GEMM -> reduce-scatter)");
  m.def("residual_combine", &vdn::residual_combine,
        "x += gate[idx] * (partial_a + partial_b + bias)");
  m.def("adaln_rmsnorm", &vdn::adaln_rmsnorm, "RMSNorm * w * (1 + scale[idx]) + shift[idx]");
  m.def("frame_sums", &vdn::frame_sums, "per-frame fp32 column sums of video rows",
        py::arg("x"), py::arg("row0"), py::arg("video_start"), py::arg("F"), py::arg("S"),
        py::arg("out"), py::arg("peers") = std::vector<int64_t>{}, py::arg("slot_offset") = 0);
  m.def("qk_prep", &vdn::qk_prep, "per-head RMSNorm + rotate-half RoPE");
  m.def("window_attention", &vdn::window_attention,
        "tcgen05 window softmax attention over an AttentionPlan (gated epilogue)");
  m.def("symm_all_gather", &vdn::symm_all_gather,
        "all-gather of equal shards read from peers' symmetric memory",
        py::arg("srcs"), py::arg("rank"), py::arg("out"), py::arg("shard_bytes"));
  m.def("symm_reduce_scatter", &vdn::symm_reduce_scatter,
        "reduce-scatter by peer loads over a symmetric buffer (fp32 sum, scaled)");
  m.def("window_attention_bwd", &vdn::window_attention_bwd,
        "tcgen05 window attention backward (dq pass over the plan, dk/dv pass over the "
        "transposed plan)");
  m.def("attention_set_variant", &vdn::attention_set_variant,
        "window attention exponential-pass variant 0..7 (1: packed f32x2, the default; 2-4: "
        "polynomial share; 5-7: timing diagnostics)");
  m.def("attention_variant", &vdn::attention_variant, "current window attention variant");
  m.def("gemm_fp8_set_trace", [](c10::optional<torch::Tensor> t) {
    vdn::gemm_fp8_set_trace(t ? reinterpret_cast<long long*>(t->data_ptr()) : nullptr);
  }, "fp8 GEMM diagnostics: int64 [148 * 8] per-CTA wait cycles, or None");
  m.def("lb_activate", &vdn::lb_activate, "SiLU [+ L2] over 128-wide heads");
  m.def("lb_conv_features", &vdn::lb_conv_features, "separable 5x5x5 depthwise conv + SiLU [+ L2]; "
        "w_spatial is [C, 25] for the fused kernel, [25, C] (tap-major) when tmp is given",
        py::arg("in"), py::arg("wsp"), py::arg("wtm"), py::arg("out"), py::arg("F"), py::arg("gh"),
        py::arg("gw"), py::arg("l2"), py::arg("err"), py::arg("tmp") = py::none());
  m.def("lb_frame_stats", &vdn::lb_frame_stats, "tcgen05 per-frame delta-rule statistics A, B");
  m.def("lb_spd_factor", &vdn::lb_spd_factor, "batched (I + aA)^-1, transition and injection");
  m.def("adaln_rmsnorm_bwd", &vdn::adaln_rmsnorm_bwd, "backward (dx) of the AdaLN RMSNorm");
  m.def("lb_conv_features_bwd", &vdn::lb_conv_features_bwd,
        "backward of the two-pass short conv (dx, dw_spatial, dw_temporal)");
  m.def("lb_scan", &vdn::lb_scan, "bidirectional serial state recurrences");
  m.def("lb_scan_set_cluster", &vdn::lb_scan_set_cluster,
        "scan cluster size: 0 = by head count, else 1, 2, 4 or 8");
  m.def("lb_gather", &vdn::lb_gather, "window-complement state gather with alpha bridge");
  m.def("lb_readout", &vdn::lb_readout, "tcgen05 readout q.S^T + RMSNorm * w * gate");
}
