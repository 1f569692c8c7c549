// Backward of the AdaLN-modulated RMSNorm (sm_100a), the training path of
//   y = RMSNorm(x) * w * (1 + scale[idx[r]]) + shift[idx[r]]
// (reference: the H3 block's norm1 / norm2 with the AdaLN modulation, fused_block.py:41-44;
// the reference differentiates it through autograd). With r = (mean(x^2) + eps)^-1/2 and
// g = dy * w * (1 + scale[idx]):   dx = r g - (r^3 / D) x sum(g x).
// One warp per row; two streaming passes over the row (sums, then dx), the second served
// mostly from L1/L2; fp32 arithmetic, bf16 in and out.
#include <cuda_bf16.h>

#include "common.cuh"
#include "launchers.h"

namespace vdn {

__device__ __forceinline__ void norm_bwd_load(const __nv_bfloat16* x, const __nv_bfloat16* dy,
                                              const __nv_bfloat16* srow, const float* w, int c,
                                              float xv[8], float gv[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(x + c * 8);
  const uint4 b = *reinterpret_cast<const uint4*>(dy + c * 8);
  const uint4 s = *reinterpret_cast<const uint4*>(srow + c * 8);
  const uint32_t* au = reinterpret_cast<const uint32_t*>(&a);
  const uint32_t* bu = reinterpret_cast<const uint32_t*>(&b);
  const uint32_t* su = reinterpret_cast<const uint32_t*>(&s);
  float wv[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
  if (w) {
    const float4 wa = __ldg(reinterpret_cast<const float4*>(w + c * 8));
    const float4 wb = __ldg(reinterpret_cast<const float4*>(w + c * 8 + 4));
    wv[0] = wa.x; wv[1] = wa.y; wv[2] = wa.z; wv[3] = wa.w;
    wv[4] = wb.x; wv[5] = wb.y; wv[6] = wb.z; wv[7] = wb.w;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    xv[2 * j] = bf16_lo(au[j]);
    xv[2 * j + 1] = bf16_hi(au[j]);
    gv[2 * j] = bf16_lo(bu[j]) * wv[2 * j] * (1.f + bf16_lo(su[j]));
    gv[2 * j + 1] = bf16_hi(bu[j]) * wv[2 * j + 1] * (1.f + bf16_hi(su[j]));
  }
}

__global__ void __launch_bounds__(256) adaln_rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ dy,
    int64_t ldy, const float* __restrict__ w, float eps, const __nv_bfloat16* __restrict__ table,
    int64_t ldt, int scale_col, const int* __restrict__ idx, __nv_bfloat16* __restrict__ dx,
    int64_t ldo, int T, int D) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;                       // whole warp: no block barriers below
  const int nvec = D >> 3;
  const __nv_bfloat16* xr = x + (int64_t)row * ldx;
  const __nv_bfloat16* gr = dy + (int64_t)row * ldy;
  const __nv_bfloat16* sr = table + (int64_t)idx[row] * ldt + scale_col;
  float ss = 0.f, dot = 0.f;
  for (int c = lane; c < nvec; c += 32) {
    float xv[8], gv[8];
    norm_bwd_load(xr, gr, sr, w, c, xv, gv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ss = fmaf(xv[j], xv[j], ss);
      dot = fmaf(gv[j], xv[j], dot);
    }
  }
  ss = warp_sum(ss);
  dot = warp_sum(dot);
  const float r = rsqrtf(ss / (float)D + eps);
  const float k = r * r * r * dot / (float)D;
  __nv_bfloat16* orow = dx + (int64_t)row * ldo;
  for (int c = lane; c < nvec; c += 32) {
    float xv[8], gv[8];
    norm_bwd_load(xr, gr, sr, w, c, xv, gv);
    uint4 o;
    uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      ou[j] = pack_bf16(r * gv[2 * j] - k * xv[2 * j], r * gv[2 * j + 1] - k * xv[2 * j + 1]);
    *reinterpret_cast<uint4*>(orow + c * 8) = o;
  }
}

void launch_adaln_rmsnorm_bwd(const void* x, int64_t ldx, const void* dy, int64_t ldy,
                              const float* w, float eps, const void* table, int64_t ldt,
                              int scale_col, const int* idx, void* dx, int64_t ldo, int T, int D,
                              cudaStream_t stream) {
  if (T == 0 || D == 0) return;
  adaln_rmsnorm_bwd_kernel<<<(T + 7) / 8, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<const __nv_bfloat16*>(dy),
      ldy, w, eps, reinterpret_cast<const __nv_bfloat16*>(table), ldt, scale_col, idx,
      reinterpret_cast<__nv_bfloat16*>(dx), ldo, T, D);
}

}  // namespace vdn
