// Allocation-free C entry point for the delta-rule statistics + factorisation (the contract
// is in vdn_noalloc.h). The A / B statistics between the two kernels live in file-scope
// device arrays instead of freshly allocated buffers; the kernels are the ones the
// allocating path uses (linear_branch.cu), reached through their launchers.
#include "launchers.h"
#include "vdn_noalloc.h"

namespace {

constexpr int kMatFloats = 128 * 128;
constexpr int kMaxDevices = 64;

// 2 x 128 x 64 KB = 16 MB of statistics scratch, plus the kernels' error word.
static __device__ __align__(256) float g_noalloc_A[VDN_NOALLOC_MAX_MATS * kMatFloats];
static __device__ __align__(256) float g_noalloc_B[VDN_NOALLOC_MAX_MATS * kMatFloats];
static __device__ __align__(256) int g_noalloc_err[64];

struct ScratchAddrs {
  bool ready;
  float* A;
  float* B;
  int* err;
};
ScratchAddrs g_addrs[kMaxDevices];  // resolved once per device

int resolve(int dev, ScratchAddrs** out) {
  if (dev < 0 || dev >= kMaxDevices) return VDN_NOALLOC_CUDA_ERROR;
  ScratchAddrs& s = g_addrs[dev];
  if (!s.ready) {
    void* a = nullptr;
    void* b = nullptr;
    void* e = nullptr;
    if (cudaGetSymbolAddress(&a, g_noalloc_A) != cudaSuccess ||
        cudaGetSymbolAddress(&b, g_noalloc_B) != cudaSuccess ||
        cudaGetSymbolAddress(&e, g_noalloc_err) != cudaSuccess)
      return VDN_NOALLOC_CUDA_ERROR;
    s.A = static_cast<float*>(a);
    s.B = static_cast<float*>(b);
    s.err = static_cast<int*>(e);
    s.ready = true;
  }
  *out = &s;
  return VDN_NOALLOC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int vdn_delta_stats_factor_noalloc(
    const void* k, int64_t ldk, const void* v, int64_t ldv, const float* beta, const float* alpha,
    int F, int S, int H, float a_scale, float b_scale, float* trans, float* inj,
    cudaStream_t stream) {
  if (F <= 0 || S <= 0 || H <= 0) return VDN_NOALLOC_BAD_ARGUMENT;
  if ((int64_t)F * H > VDN_NOALLOC_MAX_MATS) return VDN_NOALLOC_TOO_LARGE;
  if (!k || !v || !beta || !alpha || !trans || !inj) return VDN_NOALLOC_BAD_ARGUMENT;
  if (!aligned16(k) || !aligned16(v) || !aligned16(trans) || !aligned16(inj) || ldk % 8 ||
      ldv % 8 || ldk < (int64_t)H * 128 || ldv < (int64_t)H * 128)
    return VDN_NOALLOC_BAD_ARGUMENT;
  // An error already pending on this host thread belongs to the caller: refuse to run
  // (leaving it pending) rather than report it as ours or clear it.
  if (cudaPeekAtLastError() != cudaSuccess) return VDN_NOALLOC_CUDA_ERROR;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return VDN_NOALLOC_CUDA_ERROR;
  ScratchAddrs* s = nullptr;
  const int rc = resolve(dev, &s);
  if (rc != VDN_NOALLOC_OK) return rc;
  if (cudaMemsetAsync(s->err, 0, sizeof(int), stream) != cudaSuccess) return VDN_NOALLOC_CUDA_ERROR;
  try {
    vdn::launch_lb_frame_stats(k, ldk, v, ldv, F, S, H, beta, s->A, s->B, s->err, stream);
    vdn::launch_lb_spd_factor(s->A, s->B, alpha, trans, inj, F * H, a_scale, b_scale, stream);
  } catch (...) {
    return VDN_NOALLOC_CUDA_ERROR;
  }
  // nothing was pending at entry, so an error here comes from this call's launches
  return cudaGetLastError() == cudaSuccess ? VDN_NOALLOC_OK : VDN_NOALLOC_CUDA_ERROR;
}

extern "C" __attribute__((visibility("default"))) int vdn_noalloc_read_device_error(int* code) {
  if (!code) return VDN_NOALLOC_BAD_ARGUMENT;
  return cudaMemcpyFromSymbol(code, g_noalloc_err, sizeof(int)) == cudaSuccess
             ? VDN_NOALLOC_OK
             : VDN_NOALLOC_CUDA_ERROR;
}

extern "C" __attribute__((visibility("default"))) const char* vdn_noalloc_error_string(int code) {
  switch (code) {
    case VDN_NOALLOC_OK: return "ok";
    case VDN_NOALLOC_TOO_LARGE:
      return "F * H exceeds VDN_NOALLOC_MAX_MATS (128): the fixed statistics scratch is full";
    case VDN_NOALLOC_BAD_ARGUMENT: return "null pointer, misaligned pointer or stride, or empty shape";
    case VDN_NOALLOC_CUDA_ERROR: return "CUDA error while resolving the scratch or launching";
    default: return "unknown code";
  }
}
