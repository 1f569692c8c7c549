// Raw-pointer launch API of the CUDA translation units. The .cu files include only CUDA
// headers (fast nvcc builds); ops.cpp adapts torch tensors onto these.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vdn {

struct GemmArgs {
  const void* A;   // [M, K] bf16, row stride lda (elements)
  const void* B;   // [N, K] bf16, row stride ldb
  int64_t lda, ldb;
  int M, N, K;
};

// mode: 0 store, 1 gated residual, 2 swiglu (interleaved), 3 accumulate
void launch_gemm_bf16(const GemmArgs& a, int mode, void* out, int64_t ldo, const float* bias,
                      const void* gate, int64_t ldg, const int* gate_idx, int* err,
                      cudaStream_t stream);

}  // namespace vdn
