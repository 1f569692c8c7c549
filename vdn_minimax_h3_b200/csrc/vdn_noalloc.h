// C entry points that allocate no device memory (no cudaMalloc / cudaFree, no allocating
// library call): intermediates live in fixed, file-scope device scratch arrays.
//
// vdn_delta_stats_factor_noalloc
//   The delta-rule statistics and factorisation of the linear branch in one call:
//     A_fh = sum_s beta k k^T,  B_fh = sum_s (beta v) k^T            (scratch, fp32)
//     trans_fh = diag(alpha_fh) (I + a_scale A_fh)^-1,  inj_fh = b_scale B_fh (I + a_scale A_fh)^-1
//   with the same kernels as the allocating path (lb_frame_stats + lb_spd_factor), so the
//   results are identical to ops.linear_branch.frame_statistics + factor_apply.
//   Inputs (device pointers): k, v bf16 token-major rows [F*S, H*128] with row strides ldk /
//   ldv (elements, multiple of 8, 16-byte aligned bases); beta fp32 [F*S*H]; alpha fp32
//   [F*H*128]. Outputs: trans, inj fp32 [F, H, 128, 128].
//   Limit: F * H <= VDN_NOALLOC_MAX_MATS (the scratch holds that many 128 x 128 pairs,
//   2 x 64 KB each: 16 MB); larger requests return VDN_NOALLOC_TOO_LARGE and launch nothing.
//   Nothing in the scratch needs to start at zero: each call clears the scratch error word
//   before its kernels run, and the statistics kernel writes all of A and B -- unless it
//   gives up on a bounded wait. Then it records a code in the error word and skips its
//   stores, the factor kernel reads the previous call's A / B, and trans / inj are invalid:
//   after the stream finishes, check vdn_noalloc_read_device_error and discard the outputs
//   whenever the word is nonzero.
//   A CUDA error already pending on the calling host thread is left in place and the call
//   returns VDN_NOALLOC_CUDA_ERROR without launching, so an earlier, unrelated failure is
//   never reported as this call's nor cleared by it.
//   The scratch is shared by every call on a device: calls that overlap in time (different
//   streams, or host threads, without ordering between them) race on it.
//   The first call on a device resolves the scratch addresses (cudaGetSymbolAddress) and
//   sets kernel attributes; make that first call before any stream capture.
// Returns 0 on success or a VDN_NOALLOC_* code; vdn_noalloc_error_string names it.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VDN_NOALLOC_MAX_MATS 128

enum {
  VDN_NOALLOC_OK = 0,
  VDN_NOALLOC_TOO_LARGE = 1,     // F * H above VDN_NOALLOC_MAX_MATS
  VDN_NOALLOC_BAD_ARGUMENT = 2,  // null pointer, misaligned base or stride, empty shape
  VDN_NOALLOC_CUDA_ERROR = 3,    // symbol lookup or launch failed
};

int vdn_delta_stats_factor_noalloc(const void* k, int64_t ldk, const void* v, int64_t ldv,
                                   const float* beta, const float* alpha, int F, int S, int H,
                                   float a_scale, float b_scale, float* trans, float* inj,
                                   cudaStream_t stream);

// Copies the scratch error word (a kernel's bounded-wait failure code, 0 if none) to *code;
// synchronous, call after the stream has finished. Returns a VDN_NOALLOC_* code.
int vdn_noalloc_read_device_error(int* code);

const char* vdn_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
