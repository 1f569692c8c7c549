// Backward of the linear branch's separable short conv (sm_100a): the training path of
// features = act(temporal5(spatial5x5(x))), act = SiLU [then L2 over the head's 128
// channels]. Reference parity: src/models/linear_attention/features.py:133-209 (the
// reference differentiates its cuDNN depthwise conv + Inductor temporal/activation code
// through autograd). The forward runs the two-pass kernels of linear_branch.cu, whose bf16
// spatial intermediate `tmp` is kept for this pass.
//
//   lb_temporal_bwd_kernel  one warp per (head, position), lane = 4 channels, streaming the
//                           frames: recompute u = temporal5(tmp) in registers, take the
//                           activation's backward (warp reductions for the L2 norm), emit the
//                           transposed temporal conv dtmp[f] = sum_dt w[dt] du[f - dt + 2]
//                           from a five-frame register ring, and accumulate dw_temporal in
//                           registers (one atomic per channel and tap per warp at the end).
//   lb_spatial_bwd_kernel   block = (frame, head), thread = channel: slides a 5 x 5 window of
//                           dtmp and of x along each grid row (10 loads per position),
//                           dx = sum w[i][j] dtmp[y-i+2][x-j+2] (the flipped stencil) and
//                           dw_spatial[i][j] += dtmp[y][x] x[y+i-2][x+j-2] in registers.
// Zero padding in space and time matches the forward's; fp32 accumulation throughout.
#include <cuda_bf16.h>

#include "common.cuh"
#include "launchers.h"

namespace vdn {

constexpr int TB_WARPS = 8;

__device__ __forceinline__ float4 ld_bf16x4(const __nv_bfloat16* p) {
  const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
  return make_float4(bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y));
}

__device__ __forceinline__ float f4_get(const float4& v, int c) {
  return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}

__global__ void __launch_bounds__(TB_WARPS * 32) lb_temporal_bwd_kernel(
    const __nv_bfloat16* __restrict__ tmp, int64_t ldt, const __nv_bfloat16* __restrict__ dy,
    int64_t ldy, const float* __restrict__ wtm, float* __restrict__ dtmp,
    float* __restrict__ dwtm, int F, int S, int H, int l2) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * TB_WARPS + warp;
  if (h >= H) return;                       // whole warp: no block barriers below
  const int64_t C = (int64_t)H * 128;
  const int64_t chan = (int64_t)h * 128 + lane * 4;
  float w[5][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int dt = 0; dt < 5; ++dt) w[dt][c] = __ldg(wtm + (chan + c) * 5 + dt);
  float dw[5][4];
#pragma unroll
  for (int dt = 0; dt < 5; ++dt)
#pragma unroll
    for (int c = 0; c < 4; ++c) dw[dt][c] = 0.f;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int pos = blockIdx.x; pos < S; pos += gridDim.x) {
    auto load_t = [&](int f) {
      return f < F ? ld_bf16x4(tmp + ((int64_t)f * S + pos) * ldt + chan) : zero;
    };
    float4 t[5];                            // tmp of frames fo-2 .. fo+2
    t[0] = zero;
    t[1] = zero;
    t[2] = load_t(0);
    t[3] = load_t(1);
    t[4] = load_t(2);
    float4 d[5] = {zero, zero, zero, zero, zero};   // d[4] = du[fo], ..., d[0] = du[fo-4]
    for (int fo = 0; fo < F + 2; ++fo) {
      float du[4] = {0.f, 0.f, 0.f, 0.f};
      if (fo < F) {                         // warp-uniform
        const float4 g4 = ld_bf16x4(dy + ((int64_t)fo * S + pos) * ldy + chan);
        float u[4], sg[4], s[4], g[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float acc = 0.f;
#pragma unroll
          for (int dt = 0; dt < 5; ++dt) acc = fmaf(w[dt][c], f4_get(t[dt], c), acc);
          u[c] = acc;
          sg[c] = 1.0f / (1.0f + expf(-acc));
          s[c] = acc * sg[c];
          g[c] = f4_get(g4, c);
        }
        float ds[4];
        if (l2) {
          const float ss = warp_sum(s[0] * s[0] + s[1] * s[1] + s[2] * s[2] + s[3] * s[3]);
          const float inv = rsqrtf(fmaxf(ss, 1e-12f));
          float y[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) y[c] = s[c] * inv;
          const float dot = warp_sum(y[0] * g[0] + y[1] * g[1] + y[2] * g[2] + y[3] * g[3]);
          const bool clamped = !(ss > 1e-12f);   // the norm's floor: a constant scale
#pragma unroll
          for (int c = 0; c < 4; ++c) ds[c] = clamped ? inv * g[c] : inv * (g[c] - y[c] * dot);
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) ds[c] = g[c];
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          du[c] = ds[c] * sg[c] * (1.0f + u[c] * (1.0f - sg[c]));   // SiLU'
#pragma unroll
          for (int dt = 0; dt < 5; ++dt) dw[dt][c] = fmaf(du[c], f4_get(t[dt], c), dw[dt][c]);
        }
      }
      d[0] = d[1];
      d[1] = d[2];
      d[2] = d[3];
      d[3] = d[4];
      d[4] = make_float4(du[0], du[1], du[2], du[3]);
      const int fe = fo - 2;                // dtmp[fe] = sum_dt w[dt] du[fe - dt + 2]
      if (fe >= 0) {
        float o[4];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          o[c] = w[0][c] * f4_get(d[4], c) + w[1][c] * f4_get(d[3], c) +
                 w[2][c] * f4_get(d[2], c) + w[3][c] * f4_get(d[1], c) +
                 w[4][c] * f4_get(d[0], c);
        *reinterpret_cast<float4*>(dtmp + ((int64_t)fe * S + pos) * C + chan) =
            make_float4(o[0], o[1], o[2], o[3]);
      }
      t[0] = t[1];
      t[1] = t[2];
      t[2] = t[3];
      t[3] = t[4];
      t[4] = load_t(fo + 3);
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int dt = 0; dt < 5; ++dt) atomicAdd(dwtm + (chan + c) * 5 + dt, dw[dt][c]);
}

__global__ void __launch_bounds__(128) lb_spatial_bwd_kernel(
    const __nv_bfloat16* __restrict__ in, int64_t ldi, const float* __restrict__ dtmp,
    const float* __restrict__ wsp, __nv_bfloat16* __restrict__ dx, int64_t ldx,
    float* __restrict__ dwsp, int gh, int gw, int C) {
  const int f = blockIdx.x;
  const int c = blockIdx.y * 128 + threadIdx.x;
  const int S = gh * gw;
  const int64_t fbase = (int64_t)f * S;
  float w[25], dw[25];
#pragma unroll
  for (int k = 0; k < 25; ++k) {
    w[k] = __ldg(wsp + (int64_t)k * C + c);
    dw[k] = 0.f;
  }
  auto G = [&](int y, int x) -> float {
    return (y >= 0 && y < gh && x >= 0 && x < gw) ? __ldg(dtmp + (fbase + y * gw + x) * C + c)
                                                  : 0.f;
  };
  auto X = [&](int y, int x) -> float {
    if (y < 0 || y >= gh || x < 0 || x >= gw) return 0.f;
    const unsigned short b =
        __ldg(reinterpret_cast<const unsigned short*>(in + (fbase + y * gw + x) * ldi + c));
    return __uint_as_float((uint32_t)b << 16);
  };
  for (int y = 0; y < gh; ++y) {
    // inside the x loop: gwin[r][k] = dtmp(y + r - 2, x + k - 2), xwin likewise for x;
    // before it, columns -3 .. 1 (the first shift drops column -3 and loads column 2)
    float gwin[5][5], xwin[5][5];
#pragma unroll
    for (int r = 0; r < 5; ++r)
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        gwin[r][k] = G(y + r - 2, k - 3);
        xwin[r][k] = X(y + r - 2, k - 3);
      }
    for (int x = 0; x < gw; ++x) {
      // bring column x + 2 in: the window now covers columns x-2 .. x+2
#pragma unroll
      for (int r = 0; r < 5; ++r) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          gwin[r][k] = gwin[r][k + 1];
          xwin[r][k] = xwin[r][k + 1];
        }
        gwin[r][4] = G(y + r - 2, x + 2);
        xwin[r][4] = X(y + r - 2, x + 2);
      }
      float acc = 0.f;
      const float gc = gwin[2][2];
#pragma unroll
      for (int i = 0; i < 5; ++i)
#pragma unroll
        for (int j = 0; j < 5; ++j) {
          acc = fmaf(w[i * 5 + j], gwin[4 - i][4 - j], acc);
          dw[i * 5 + j] = fmaf(gc, xwin[i][j], dw[i * 5 + j]);
        }
      dx[(fbase + y * gw + x) * ldx + c] = __float2bfloat16_rn(acc);
    }
  }
#pragma unroll
  for (int k = 0; k < 25; ++k) atomicAdd(dwsp + (int64_t)k * C + c, dw[k]);
}

void launch_lb_conv2_bwd(const void* in, int64_t ldi, const void* tmp, int64_t ldt,
                         const void* dy, int64_t ldy, const float* wsp, const float* wtm,
                         float* dtmp, void* dx, int64_t ldx, float* dwsp, float* dwtm, int F,
                         int gh, int gw, int H, int l2, cudaStream_t stream) {
  if (!F || !gh || !gw || !H) return;
  const int S = gh * gw;
  const int pos_blocks = S < 256 ? S : 256;
  lb_temporal_bwd_kernel<<<dim3(pos_blocks, (H + TB_WARPS - 1) / TB_WARPS), TB_WARPS * 32, 0,
                           stream>>>(reinterpret_cast<const __nv_bfloat16*>(tmp), ldt,
                                     reinterpret_cast<const __nv_bfloat16*>(dy), ldy, wtm, dtmp,
                                     dwtm, F, S, H, l2);
  lb_spatial_bwd_kernel<<<dim3(F, H), 128, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(in), ldi, dtmp, wsp,
      reinterpret_cast<__nv_bfloat16*>(dx), ldx, dwsp, gh, gw, H * 128);
}

}  // namespace vdn
