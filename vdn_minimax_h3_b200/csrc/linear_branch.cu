// The linear branch's kernels (sm_100a). Reference parity, per kernel:
//
//   lb_activate       SiLU [+ L2 over the head dim]     linear_attention/features.py:47-67
//   lb_conv_features  5x5 depthwise spatial conv, 5-tap temporal conv, SiLU [+ L2], one
//                     pass (features.py:133-209 + ops/temporal_conv.py; the reference runs
//                     cuDNN for the spatial half and a Triton kernel for the rest)
//   lb_frame_stats    A = sum_s beta k k^T, B = sum_s beta v k^T per (frame, head) on
//                     tcgen05 (scan.py:79-167). A needs fp32 accuracy: beta*k is split into
//                     bf16 hi + lo and both halves accumulate into one fp32 TMEM tile, so A
//                     carries ~16 mantissa bits of the products (the reference: TF32, 10).
//   lb_spd_factor     (I + a A)^-1 by Gauss-Jordan in fp32 shared memory (SPD: no pivoting),
//                     transition = diag(alpha) inv, injection = (b B) inv (delta_rule.py:31-89)
//   lb_scan           both serial recurrences S_t = S_{t-1} T_t + inj_t (scan.py:170-255)
//   lb_gather         window complement + alpha bridge (scan.py:261-396)
//   lb_readout        q . S^T on tcgen05, then RMSNorm * w * sigmoid(gate) and the store in
//                     token order (branch.py:440-458, kernels.py:8-57)
#include "common.cuh"
#include "launchers.h"
#include "tma.cuh"

namespace vdn {

// ------------------------------------------------------------------------- activation
__global__ void __launch_bounds__(256) lb_activate_kernel(const __nv_bfloat16* __restrict__ in,
                                                          int64_t ldi, int N, int H,
                                                          __nv_bfloat16* __restrict__ out,
                                                          int64_t ldo, int l2) {
  const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= (int64_t)N * H) return;
  const int row = (int)(item / H), h = (int)(item % H);
  const uint2 v = *reinterpret_cast<const uint2*>(in + (int64_t)row * ldi + h * 128 + lane * 4);
  float y[4] = {siluf_(bf16_lo(v.x)), siluf_(bf16_hi(v.x)), siluf_(bf16_lo(v.y)), siluf_(bf16_hi(v.y))};
  if (l2) {
    float ss = warp_sum(y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3]);
    const float inv = 1.f / fmaxf(sqrtf(ss), 1e-6f);
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] *= inv;
  }
  *reinterpret_cast<uint2*>(out + (int64_t)row * ldo + h * 128 + lane * 4) =
      make_uint2(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]));
}

void launch_lb_activate(const void* in, int64_t ldi, int N, int H, void* out, int64_t ldo, int l2,
                        cudaStream_t stream) {
  const int64_t items = (int64_t)N * H;
  if (!items) return;
  lb_activate_kernel<<<(unsigned)((items + 7) / 8), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(in), ldi, N, H, reinterpret_cast<__nv_bfloat16*>(out),
      ldo, l2);
}

// --------------------------------------------------------------- separable short conv
// Block = (grid row y, head h, chunk of LB_FC frames); warp w owns positions 4w..4w+3 of the
// row, lane owns 4 channels, so a warp covers the head's 128 channels and the L2 norm is a
// warp reduction. The five input rows y-2..y+2 of a frame (all positions, the head's 128
// channels) are staged in shared memory by TMA (one box per row, issued by one thread) in
// a LB_STAGES-deep ring of frames, so later frames are in flight while this frame's 25
// spatial taps run; rows and positions outside the grid stay zero (the convolution's zero
// padding). The five latest spatial results per output sit in a register ring for the
// temporal taps. Frames are chunked (2-frame halo each side).
constexpr int LB_FC = 16;
constexpr int LB_PPW = 4;                 // positions per warp
constexpr int LB_MAXW = 48;               // widest supported grid row
constexpr int LB_XPAD = LB_MAXW + 4;      // staged positions per row (2 halo each side)
constexpr int LB_ROW_BYTES = LB_XPAD * 256;        // one staged row: 128 bf16 per position
constexpr int LB_STAGE_BYTES = 5 * LB_ROW_BYTES;   // five input rows of one frame
constexpr int LB_STAGES = 3;
constexpr int LB_CONV_SMEM = LB_STAGES * LB_STAGE_BYTES + 1024 /*align*/ + 64 /*barriers*/;

__global__ void __launch_bounds__(384) lb_conv_kernel(
    const __grid_constant__ CUtensorMap tmIn, const float* __restrict__ wsp,
    const float* __restrict__ wtm, __nv_bfloat16* __restrict__ out, int64_t ldo, int F, int gh,
    int gw, int H, int l2, int* err) {
  extern __shared__ uint8_t lb_smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(lb_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + LB_STAGES * LB_STAGE_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + LB_STAGES);
  __shared__ __align__(16) float s_wsp[25][128];
  __shared__ __align__(16) float s_wtm[5][128];
  const int y = blockIdx.x, h = blockIdx.y;
  const int f0 = blockIdx.z * LB_FC;
  const int S = gh * gw;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nthr = blockDim.x;
  for (int i = tid; i < 25 * 128; i += nthr) {
    const int tap = i / 128, c = i % 128;
    s_wsp[tap][c] = wsp[(int64_t)(h * 128 + c) * 25 + tap];
  }
  for (int i = tid; i < 5 * 128; i += nthr) {
    const int tap = i / 128, c = i % 128;
    s_wtm[tap][c] = wtm[(int64_t)(h * 128 + c) * 5 + tap];
  }
  // zero the ring once: halo positions and rows outside the grid are never written
  for (int i = tid; i < LB_STAGES * LB_STAGE_BYTES / 16; i += nthr)
    reinterpret_cast<uint4*>(stages)[i] = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    for (int s = 0; s < LB_STAGES; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  fence_proxy_async_smem();   // the zeros are visible to the TMA writes that follow
  __syncthreads();
  const int f_end = min(F, f0 + LB_FC);
  const int f_first = max(f0 - 2, 0), f_last = min(f_end + 2, F);  // frames with input
  const int n_in = f_last - f_first;
  int rows_valid = 0;
  for (int i = 0; i < 5; ++i) rows_valid += (y + i - 2 >= 0 && y + i - 2 < gh) ? 1 : 0;
  auto issue = [&](int ii) {   // input frame f_first + ii into stage ii % LB_STAGES
    const int st = ii % LB_STAGES;
    const int f = f_first + ii;
    uint8_t* base = stages + st * LB_STAGE_BYTES;
    mbar_arrive_expect_tx(&full[st], (uint32_t)(rows_valid * gw * 256));
    for (int i = 0; i < 5; ++i) {
      const int yy = y + i - 2;
      if (yy < 0 || yy >= gh) continue;
      tma_load_2d(base + i * LB_ROW_BYTES + 2 * 256, &tmIn, &full[st], h * 128, f * S + yy * gw);
    }
  };
  if (tid == 0) {
    tma_prefetch_desc(&tmIn);
    for (int ii = 0; ii < min(LB_STAGES, n_in); ++ii) issue(ii);
  }

  const int x0 = warp * LB_PPW;
  const bool active = x0 < gw;
  const int c0 = lane * 4;
  const int64_t chan = (int64_t)h * 128 + c0;
  float ring[5][LB_PPW][4];
#pragma unroll
  for (int a = 0; a < 5; ++a)
#pragma unroll
    for (int q = 0; q < LB_PPW; ++q)
#pragma unroll
      for (int b = 0; b < 4; ++b) ring[a][q][b] = 0.f;
  float tw[5][4];
#pragma unroll
  for (int dt = 0; dt < 5; ++dt) {
    const float4 t = *reinterpret_cast<const float4*>(&s_wtm[dt][c0]);
    tw[dt][0] = t.x;
    tw[dt][1] = t.y;
    tw[dt][2] = t.z;
    tw[dt][3] = t.w;
  }
  int issued = min(LB_STAGES, n_in);
  for (int f = f0 - 2; f < f_end + 2; ++f) {
    const bool have = f >= f_first && f < f_last;
    const int ii = f - f_first;
    bool ok = true;
    if (have) ok = mbar_wait(&full[ii % LB_STAGES], (uint32_t)((ii / LB_STAGES) & 1), abort_flag, err,
                             kErrTimeoutProducer);
    float sp[LB_PPW][4];
#pragma unroll
    for (int q = 0; q < LB_PPW; ++q)
#pragma unroll
      for (int b = 0; b < 4; ++b) sp[q][b] = 0.f;
    if (have && ok && active) {
      const uint8_t* base = stages + (ii % LB_STAGES) * LB_STAGE_BYTES + c0 * 2;
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        float win[LB_PPW + 4][4];
#pragma unroll
        for (int u = 0; u < LB_PPW + 4; ++u) {
          const uint2 v = *reinterpret_cast<const uint2*>(base + i * LB_ROW_BYTES + (x0 + u) * 256);
          win[u][0] = bf16_lo(v.x);
          win[u][1] = bf16_hi(v.x);
          win[u][2] = bf16_lo(v.y);
          win[u][3] = bf16_hi(v.y);
        }
#pragma unroll
        for (int j = 0; j < 5; ++j) {
          const float4 w = *reinterpret_cast<const float4*>(&s_wsp[i * 5 + j][c0]);
#pragma unroll
          for (int q = 0; q < LB_PPW; ++q) {
            sp[q][0] = fmaf(w.x, win[q + j][0], sp[q][0]);
            sp[q][1] = fmaf(w.y, win[q + j][1], sp[q][1]);
            sp[q][2] = fmaf(w.z, win[q + j][2], sp[q][2]);
            sp[q][3] = fmaf(w.w, win[q + j][3], sp[q][3]);
          }
        }
      }
    }
    // every thread is done with this stage (and agrees on aborting) before it is refilled
    if (__syncthreads_or(!ok)) break;
    if (tid == 0 && have && issued < n_in && ii + LB_STAGES == issued) issue(issued++);
#pragma unroll
    for (int q = 0; q < LB_PPW; ++q)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        ring[0][q][b] = ring[1][q][b];
        ring[1][q][b] = ring[2][q][b];
        ring[2][q][b] = ring[3][q][b];
        ring[3][q][b] = ring[4][q][b];
        ring[4][q][b] = sp[q][b];
      }
    const int fo = f - 2;
    if (fo < f0 || !active) continue;
#pragma unroll
    for (int q = 0; q < LB_PPW; ++q) {
      const int x = x0 + q;
      float o[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        float t = 0.f;
#pragma unroll
        for (int dt = 0; dt < 5; ++dt) t = fmaf(tw[dt][b], ring[dt][q][b], t);
        o[b] = siluf_(t);
      }
      if (l2) {
        const float ss = warp_sum(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
        const float inv = 1.f / fmaxf(sqrtf(ss), 1e-6f);
#pragma unroll
        for (int b = 0; b < 4; ++b) o[b] *= inv;
      }
      if (x < gw)
        *reinterpret_cast<uint2*>(out + ((int64_t)fo * S + (int64_t)y * gw + x) * ldo + chan) =
            make_uint2(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]));
    }
  }
  // an aborted block waits (bounded) for its own copies in flight before exiting
  if (tid == 0 && *abort_flag) {
    const long long t0 = clock64();
    for (int ii = max(0, issued - LB_STAGES); ii < issued; ++ii) {
      while (!mbar_try_wait(&full[ii % LB_STAGES], (uint32_t)((ii / LB_STAGES) & 1)) &&
             clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  }
}

void launch_lb_conv(const void* in, int64_t ldi, const float* wsp, const float* wtm, void* out,
                    int64_t ldo, int F, int gh, int gw, int H, int l2, int* err,
                    cudaStream_t stream) {
  if (!F || !gh || !gw) return;
  if (gw > LB_MAXW) throw std::runtime_error("short conv: grid width above 48 is not supported");
  static std::atomic<uint64_t> attr{0};
  if (attr_needed(attr)) {
    cudaFuncSetAttribute(lb_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LB_CONV_SMEM);
    attr_done(attr);
  }
  // rows = packed tokens of the F frames, one 128-channel head per box column
  CUtensorMap tm = make_tmap_2d(in, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H * 128,
                                (uint64_t)F * gh * gw, ldi * 2, 128, gw, CU_TENSOR_MAP_SWIZZLE_NONE);
  const int warps = (gw + LB_PPW - 1) / LB_PPW;
  dim3 grid(gh, H, (F + LB_FC - 1) / LB_FC);
  lb_conv_kernel<<<grid, warps * 32, LB_CONV_SMEM, stream>>>(
      tm, wsp, wtm, reinterpret_cast<__nv_bfloat16*>(out), ldo, F, gh, gw, H, l2, err);
}

// ------------------------------------------------- separable short conv, two passes
// Pass 1 (lb_spatial_kernel): the 5x5 depthwise spatial conv, bf16 result (the reference's
// spatial conv also hands a bf16 tensor to its temporal conv). Block = (chunk of SP_FC
// frames, head h, channel half); warp w owns positions 4w..4w+3 of a grid row, lane 2
// channels, whose 25 taps stay in registers as packed fp32 pairs (fma.rn.f32x2). The block
// walks its frames' grid rows in order; every input row (gw positions x 64 channels) is
// brought into shared memory once by TMA into an 8-slot row ring with 3 rows of prefetch,
// and output row y reads rows y-2..y+2 (one 128-byte wavefront per position). ~50 KB of
// shared memory and <= 93 registers give two to three blocks per SM.
// Pass 2 (lb_temporal_kernel): 5-tap temporal conv + SiLU [+ L2 over the head's 128
// channels]; one warp per (position, head) streams the frames with a register ring, so
// every intermediate element is read once.
constexpr int SP_SLOTS = 8;
constexpr int SP_AHEAD = 3;               // rows of prefetch beyond the five in use
constexpr int SP_FC = 4;                  // frames per block
constexpr int SP_CH = 64;                 // channels per block (half a head)
constexpr int SP_ROW_BYTES = LB_XPAD * SP_CH * 2;
constexpr int SP_SMEM = SP_SLOTS * SP_ROW_BYTES + 1024 /*align*/ + 128 /*barriers*/;

__global__ void __launch_bounds__(LB_MAXW / LB_PPW * 32, 2) lb_spatial_kernel(
    const __grid_constant__ CUtensorMap tmIn, const float* __restrict__ wsp, int C,
    __nv_bfloat16* __restrict__ tmp, int64_t ldt, int F, int gh, int gw, int* err) {
  extern __shared__ uint8_t lb_smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(lb_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + SP_SLOTS * SP_ROW_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + SP_SLOTS);
  const int h = blockIdx.y, half = blockIdx.z;
  const int col0 = h * 128 + half * SP_CH;           // first channel of this block
  const int f0 = blockIdx.x * SP_FC, f1 = min(F, f0 + SP_FC);
  const int S = gh * gw;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nthr = blockDim.x;
  // halo positions (2 each side) are never written by TMA: zero the ring once
  for (int i = tid; i < SP_SLOTS * SP_ROW_BYTES / 16; i += nthr)
    reinterpret_cast<uint4*>(ring)[i] = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    for (int i = 0; i < SP_SLOTS; ++i) mbar_init(&full[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  fence_proxy_async_smem();
  __syncthreads();
  const int n_loads = (f1 - f0) * gh;     // load L = grid row (f0 + L / gh, L % gh)
  int issued = 0;
  auto issue_upto = [&](int limit) {
    limit = min(limit, n_loads);
    for (; issued < limit; ++issued) {
      const int slot = issued % SP_SLOTS;
      const int f = f0 + issued / gh, y = issued % gh;
      mbar_arrive_expect_tx(&full[slot], (uint32_t)(gw * SP_CH * 2));
      tma_load_2d(ring + slot * SP_ROW_BYTES + 2 * SP_CH * 2, &tmIn, &full[slot], col0,
                  f * S + y * gw);
    }
  };
  if (tid == 0) {
    tma_prefetch_desc(&tmIn);
    issue_upto(3 + SP_AHEAD);
  }
  // this lane's two channels: 25 taps as packed pairs, one 8-byte load each from the
  // tap-major weights [25, C]
  const int c = 2 * lane;
  unsigned long long wt[25];
#pragma unroll
  for (int t = 0; t < 25; ++t)
    wt[t] = __ldg(reinterpret_cast<const unsigned long long*>(wsp + (int64_t)t * C + col0 + c));
  const int x0 = warp * LB_PPW;
  const bool active = x0 < gw;
  int waited = 0;
  bool ok = true;
  for (int o = 0; o < n_loads; ++o) {
    const int fr = o / gh, y = o - fr * gh;
    const int base = fr * gh;
    // rows o-2..o+2 of this frame are in use; load o+5 reuses the slot of o-3, which the
    // previous output row was the last to read (all threads passed the barrier below)
    if (tid == 0) issue_upto(o + 3 + SP_AHEAD);
    const int need = min(o + 3, base + gh);
    for (; waited < need && ok; ++waited)
      ok = mbar_wait(&full[waited % SP_SLOTS], (uint32_t)((waited / SP_SLOTS) & 1), abort_flag, err,
                     kErrTimeoutProducer);
    if (ok && active) {
      unsigned long long acc[LB_PPW];
#pragma unroll
      for (int q = 0; q < LB_PPW; ++q) acc[q] = 0ull;
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        const int yy = y + i - 2;
        if (yy < 0 || yy >= gh) continue;   // block-uniform: the zero padding rows
        const uint8_t* rowp = ring + ((base + yy) % SP_SLOTS) * SP_ROW_BYTES + c * 2;
        unsigned long long win[LB_PPW + 4];
#pragma unroll
        for (int u = 0; u < LB_PPW + 4; ++u)
          win[u] = f2_from_bf16x2(*reinterpret_cast<const uint32_t*>(rowp + (x0 + u) * SP_CH * 2));
#pragma unroll
        for (int j = 0; j < 5; ++j)
#pragma unroll
          for (int q = 0; q < LB_PPW; ++q) acc[q] = f2_fma(wt[i * 5 + j], win[q + j], acc[q]);
      }
      const int64_t row0 = (int64_t)(f0 + fr) * S + (int64_t)y * gw;
#pragma unroll
      for (int q = 0; q < LB_PPW; ++q) {
        if (x0 + q >= gw) break;
        float a0, a1;
        f2_unpack(acc[q], a0, a1);
        *reinterpret_cast<uint32_t*>(tmp + (row0 + x0 + q) * ldt + col0 + c) = pack_bf16(a0, a1);
      }
    }
    if (__syncthreads_or(!ok)) break;
  }
  // an aborted block waits (bounded) for its own copies in flight before exiting
  if (tid == 0 && *abort_flag) {
    const long long t0 = clock64();
    for (int L = max(0, issued - SP_SLOTS); L < issued; ++L) {
      while (!mbar_try_wait(&full[L % SP_SLOTS], (uint32_t)((L / SP_SLOTS) & 1)) &&
             clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  }
}

constexpr int TC_WARPS = 8;
// SiLU with the approximate divide (bf16 output)
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__global__ void __launch_bounds__(TC_WARPS * 32, 4) lb_temporal_kernel(
    const __nv_bfloat16* __restrict__ tmp, int64_t ldt, const float* __restrict__ wtm,
    __nv_bfloat16* __restrict__ out, int64_t ldo, int F, int S, int H, int l2) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = blockIdx.x, h = blockIdx.y * TC_WARPS + warp;
  if (h >= H) return;
  const int64_t chan = (int64_t)h * 128 + lane * 4;
  float tw[5][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int dt = 0; dt < 5; ++dt) tw[dt][c] = __ldg(wtm + (chan + c) * 5 + dt);
  const __nv_bfloat16* src = tmp + (int64_t)pos * ldt + chan;
  __nv_bfloat16* dst = out + (int64_t)pos * ldo + chan;
  const int64_t fs_in = (int64_t)S * ldt, fs_out = (int64_t)S * ldo;
  // ring slot of frame f is f % 5: with the loop unrolled by 5 every slot index is a
  // constant, so the ring never moves
  uint2 ring[5];
  ring[3] = ring[4] = make_uint2(0, 0);                     // frames -2, -1
  auto load = [&](int f) {
    return f < F ? __ldg(reinterpret_cast<const uint2*>(src + f * fs_in)) : make_uint2(0, 0);
  };
  ring[0] = load(0);
  ring[1] = load(1);
  ring[2] = load(2);
  for (int f0 = 0; f0 < F; f0 += 5) {
    // frames f0+3 .. f0+7 into slots 3, 4, 0, 1, 2 as they free up
    uint2 nxt[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) nxt[k] = load(f0 + 3 + k);
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const int fo = f0 + k;                  // output frame: inputs fo-2 .. fo+2
      if (fo >= F) break;
      // slot of frame fo+2 is (k+2) % 5; it holds frame fo+2 once the previous step stored
      if (k >= 1) ring[(k + 2) % 5] = nxt[k - 1];
      float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int dt = 0; dt < 5; ++dt) {
        const uint2 v = ring[(k + dt + 3) % 5];    // frame fo + dt - 2
        o[0] = fmaf(tw[dt][0], bf16_lo(v.x), o[0]);
        o[1] = fmaf(tw[dt][1], bf16_hi(v.x), o[1]);
        o[2] = fmaf(tw[dt][2], bf16_lo(v.y), o[2]);
        o[3] = fmaf(tw[dt][3], bf16_hi(v.y), o[3]);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) o[c] = silu_fast(o[c]);
      if (l2) {
        // x / max(||x||, 1e-6) == x * rsqrt(max(||x||^2, 1e-12))
        const float ss = warp_sum(o[0] * o[0] + o[1] * o[1] + o[2] * o[2] + o[3] * o[3]);
        const float inv = rsqrtf(fmaxf(ss, 1e-12f));
#pragma unroll
        for (int c = 0; c < 4; ++c) o[c] *= inv;
      }
      *reinterpret_cast<uint2*>(dst + fo * fs_out) =
          make_uint2(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]));
    }
    // frame f0+7 (slot (f0+7) % 5 == 2) is needed by the next group's first output
    ring[2] = nxt[4];
  }
}

void launch_lb_conv2(const void* in, int64_t ldi, const float* wsp, const float* wtm, void* tmp,
                     int64_t ldt, void* out, int64_t ldo, int F, int gh, int gw, int H, int l2,
                     int* err, cudaStream_t stream) {
  if (!F || !gh || !gw) return;
  if (gw > LB_MAXW) throw std::runtime_error("short conv: grid width above 44 is not supported");
  static std::atomic<uint64_t> attr{0};
  if (attr_needed(attr)) {
    cudaFuncSetAttribute(lb_spatial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SP_SMEM);
    // two blocks per SM need the largest shared-memory carveout
    cudaFuncSetAttribute(lb_spatial_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
    attr_done(attr);
  }
  CUtensorMap tm = make_tmap_2d(in, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H * 128,
                                (uint64_t)F * gh * gw, ldi * 2, SP_CH, gw, CU_TENSOR_MAP_SWIZZLE_NONE);
  const int warps = (gw + LB_PPW - 1) / LB_PPW;
  lb_spatial_kernel<<<dim3((F + SP_FC - 1) / SP_FC, H, 128 / SP_CH), warps * 32, SP_SMEM, stream>>>(
      tm, wsp, H * 128, reinterpret_cast<__nv_bfloat16*>(tmp), ldt, F, gh, gw, err);
  lb_temporal_kernel<<<dim3(gh * gw, (H + TC_WARPS - 1) / TC_WARPS), TC_WARPS * 32, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(tmp), ldt, wtm, reinterpret_cast<__nv_bfloat16*>(out),
      ldo, F, gh * gw, H, l2);
}

// ------------------------------------------------------------------ frame statistics
// CTA = (frame, head). 64-token chunks through a 2-stage ring: k and v by TMA (MN-major,
// 128B swizzle); the 128 threads write beta*k (hi, lo) and beta*v in the same layout; one
// thread issues MMAs into two TMEM accumulators (A: cols 0-127, B: cols 128-255).
constexpr int FS_CHUNK = 64;
constexpr int FS_TILE = FS_CHUNK * 128 * 2;              // 16 KB
constexpr int FS_STAGE = 5 * FS_TILE;                    // k, v, hi, lo, bv
constexpr int FS_SMEM = 2 * FS_STAGE + 1024 + 256;

__global__ void __launch_bounds__(128, 1)
    lb_frame_stats_kernel(const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const float* __restrict__ beta,
                          int S, int H, float* __restrict__ Aout, float* __restrict__ Bout,
                          int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * FS_STAGE);
  uint64_t* mma_bar = full + 2;
  uint64_t* done = full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int f = blockIdx.x / H, h = blockIdx.x % H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nchunks = (S + FS_CHUNK - 1) / FS_CHUNK;

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&mma_bar[0], 1);
    mbar_init(&mma_bar[1], 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto issue = [&](int c) {
    uint8_t* st = smem + (c & 1) * FS_STAGE;
    const int row = f * S + c * FS_CHUNK;
    mbar_arrive_expect_tx(&full[c & 1], 2 * FS_TILE);  // k and v, two boxes each
    tma_load_2d(st, &tmK, &full[c & 1], h * 128, row);
    tma_load_2d(st + FS_TILE / 2, &tmK, &full[c & 1], h * 128 + 64, row);
    tma_load_2d(st + FS_TILE, &tmV, &full[c & 1], h * 128, row);
    tma_load_2d(st + FS_TILE + FS_TILE / 2, &tmV, &full[c & 1], h * 128 + 64, row);
  };
  if (tid == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    issue(0);
    if (nchunks > 1) issue(1);
  }
  constexpr uint32_t idesc = umma_idesc_bf16(128, 128, true, true);
  bool ok = true;
  int last_issued[2] = {0, nchunks > 1 ? 1 : -1};
  for (int c = 0; c < nchunks; ++c) {
    const int s = c & 1;
    uint8_t* st = smem + s * FS_STAGE;
    const bool got = mbar_wait(&full[s], (c >> 1) & 1, abort_flag, err, kErrTimeoutEpilogue);
    if (__syncthreads_or(!got)) {     // block-uniform: every thread leaves together
      ok = false;
      break;
    }
    // beta-weighted operands, 16 bytes (8 channels of one token) at a time, written at the
    // same swizzled offsets the TMA used for k and v
    const int ntok = min(FS_CHUNK, S - c * FS_CHUNK);
    for (int i = tid; i < FS_CHUNK * 16; i += 128) {
      const int o = i * 16;
      const int t = (o % (FS_TILE / 2)) / 128;
      const float b = t < ntok ? beta[((int64_t)f * S + c * FS_CHUNK + t) * H + h] : 0.f;
      const uint4 kk = *reinterpret_cast<const uint4*>(st + o);
      const uint4 vv = *reinterpret_cast<const uint4*>(st + FS_TILE + o);
      const uint32_t* ku = reinterpret_cast<const uint32_t*>(&kk);
      const uint32_t* vu = reinterpret_cast<const uint32_t*>(&vv);
      uint32_t hi[4], lo[4], bv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float k0 = bf16_lo(ku[j]) * b, k1 = bf16_hi(ku[j]) * b;
        const __nv_bfloat162 hh = __floats2bfloat162_rn(k0, k1);
        hi[j] = *reinterpret_cast<const uint32_t*>(&hh);
        lo[j] = pack_bf16(k0 - __bfloat162float(hh.x), k1 - __bfloat162float(hh.y));
        const __nv_bfloat162 vb = *reinterpret_cast<const __nv_bfloat162*>(&vu[j]);
        const __nv_bfloat162 bb = __floats2bfloat162_rn(b, b);
        const __nv_bfloat162 pr = __hmul2(vb, bb);  // bf16 product, as the reference's v*beta
        bv[j] = *reinterpret_cast<const uint32_t*>(&pr);
      }
      *reinterpret_cast<uint4*>(st + 2 * FS_TILE + o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(st + 3 * FS_TILE + o) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      *reinterpret_cast<uint4*>(st + 4 * FS_TILE + o) = make_uint4(bv[0], bv[1], bv[2], bv[3]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    bool fail = false;
    if (tid == 0) {
      tc_fence_after();
      const uint32_t aK = smem_u32(st), aHi = smem_u32(st + 2 * FS_TILE),
                     aLo = smem_u32(st + 3 * FS_TILE), aBv = smem_u32(st + 4 * FS_TILE);
#pragma unroll
      for (int k = 0; k < FS_CHUNK / 16; ++k) {
        const uint32_t off = k * 2048;
        const uint64_t dk = umma_desc_mnmajor_sw128(aK + off, FS_TILE / 2);
        umma_f16_ss(tmem, umma_desc_mnmajor_sw128(aHi + off, FS_TILE / 2), dk, idesc, (c | k) != 0);
        umma_f16_ss(tmem, umma_desc_mnmajor_sw128(aLo + off, FS_TILE / 2), dk, idesc, 1u);
        umma_f16_ss(tmem + 128, umma_desc_mnmajor_sw128(aBv + off, FS_TILE / 2), dk, idesc, (c | k) != 0);
      }
      umma_commit(&mma_bar[s]);
      if (c + 2 < nchunks) {
        // stage s is rewritten only after the MMAs reading it are done
        if (mbar_wait(&mma_bar[s], (c >> 1) & 1, abort_flag, err, kErrTimeoutMma)) {
          issue(c + 2);
          last_issued[s] = c + 2;
        } else {
          fail = true;
        }
      }
    }
    if (__syncthreads_or(fail)) {
      ok = false;
      break;
    }
  }
  if (!ok && tid == 0) {
    // let the copies this thread issued land before the CTA exits
    long long t0 = clock64();
    for (int st = 0; st < 2; ++st) {
      if (last_issued[st] < 0) continue;
      while (!mbar_try_wait(&full[st], (last_issued[st] >> 1) & 1) &&
             clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  }
  if (tid == 0) {
    umma_commit(done);
  }
  if (mbar_wait(done, 0, abort_flag, err, kErrTimeoutEpilogue) && ok) {
    tc_fence_after();
    const int row = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float* arow = Aout + (((int64_t)f * H + h) * 128 + row) * 128;
    float* brow = Bout + (((int64_t)f * H + h) * 128 + row) * 128;
#pragma unroll 1
    for (int cc = 0; cc < 128; cc += 32) {
      uint32_t u[32];
      tmem_ld32(tmem + lane_off + cc, u);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(arow + cc)[q] =
            make_float4(__uint_as_float(u[4 * q]), __uint_as_float(u[4 * q + 1]),
                        __uint_as_float(u[4 * q + 2]), __uint_as_float(u[4 * q + 3]));
      tmem_ld32(tmem + lane_off + 128 + cc, u);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(brow + cc)[q] =
            make_float4(__uint_as_float(u[4 * q]), __uint_as_float(u[4 * q + 1]),
                        __uint_as_float(u[4 * q + 2]), __uint_as_float(u[4 * q + 3]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

void launch_lb_frame_stats(const void* k, int64_t ldk, const void* v, int64_t ldv, int F, int S,
                           int H, const float* beta, float* A, float* B, int* err,
                           cudaStream_t stream) {
  if (!F || !S || !H) return;
  static std::atomic<uint64_t> attr{0};
  if (attr_needed(attr)) {
    cudaFuncSetAttribute(lb_frame_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FS_SMEM);
    attr_done(attr);
  }
  const uint64_t cols = (uint64_t)H * 128, rows = (uint64_t)F * S;
  CUtensorMap tk = make_tmap_2d(k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, ldk * 2, 64, FS_CHUNK);
  CUtensorMap tv = make_tmap_2d(v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, ldv * 2, 64, FS_CHUNK);
  lb_frame_stats_kernel<<<F * H, 128, FS_SMEM, stream>>>(tk, tv, beta, S, H, A, B, err);
}

// ---------------------------------------------------------------------- SPD factor
// Gauss-Jordan inversion with the matrix held in registers: thread (ti, tj) of 16 x 16 owns
// the 8 x 8 block rows 8ti.., cols 8tj..; step k broadcasts only pivot column k and pivot
// row k through shared memory. SPD (I + aA): no row exchanges needed.
constexpr int SPD_LD = 132;                       // padded row stride (16-byte aligned rows)
constexpr int SPD_BK = 32;                        // B columns staged per chunk
constexpr int SPD_SMEM = (128 * SPD_LD + SPD_BK * SPD_LD + 2 * 128) * 4;

__global__ void __launch_bounds__(256) lb_spd_factor_kernel(
    const float* __restrict__ A, const float* __restrict__ B, const float* __restrict__ alpha,
    float* __restrict__ trans, float* __restrict__ inj, float a_scale, float b_scale) {
  extern __shared__ float sm[];
  float* colk = sm;            // [128]
  float* rowk = sm + 128;      // [128]
  float* Ms = sm + 256;        // [128][SPD_LD] final inverse, for the injection product
  float* Bt = Ms + 128 * SPD_LD;  // [SPD_BK][SPD_LD] a chunk of B^T (k-major)
  const int64_t mat = blockIdx.x;
  const float* a = A + mat * 16384;
  const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
  float m[8][8];
  // M = I + a_scale * (A + A^T) / 2: A staged through shared memory (coalesced 16-byte
  // global loads), the transposed block read back with 16-byte shared loads
  for (int e = tid * 4; e < 16384; e += 256 * 4) {
    const float4 v = *reinterpret_cast<const float4*>(a + e);
    *reinterpret_cast<float4*>(Ms + (e >> 7) * SPD_LD + (e & 127)) = v;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v0 = *reinterpret_cast<const float4*>(Ms + (ti * 8 + i) * SPD_LD + tj * 8);
    const float4 v1 = *reinterpret_cast<const float4*>(Ms + (ti * 8 + i) * SPD_LD + tj * 8 + 4);
    m[i][0] = v0.x; m[i][1] = v0.y; m[i][2] = v0.z; m[i][3] = v0.w;
    m[i][4] = v1.x; m[i][5] = v1.y; m[i][6] = v1.z; m[i][7] = v1.w;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 t0 = *reinterpret_cast<const float4*>(Ms + (tj * 8 + j) * SPD_LD + ti * 8);
    const float4 t1 = *reinterpret_cast<const float4*>(Ms + (tj * 8 + j) * SPD_LD + ti * 8 + 4);
    const float tv[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m[i][j] = a_scale * 0.5f * (m[i][j] + tv[i]) + ((ti * 8 + i) == (tj * 8 + j) ? 1.f : 0.f);
  }
  __syncthreads();
  // Step k of Gauss-Jordan as ONE uniform rank-1 update: with c the pivot column, r the
  // pivot row and p = M[k][k], set c'_k = p - 1 and r'_k = p + 1; then
  // M -= c' r'^T / p gives the eliminated entries, the scaled pivot row r/p, the column
  // -c/p and the new pivot 1/p at once -- one FFMA per element, no per-element branches.
  for (int k = 0; k < 128; ++k) {
    const int kb = k >> 3, kk = k & 7;
    if (tj == kb) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c == kk) {
#pragma unroll
          for (int i = 0; i < 8; ++i) colk[ti * 8 + i] = m[i][c];
        }
      }
    }
    if (ti == kb) {
#pragma unroll
      for (int rr0 = 0; rr0 < 8; ++rr0) {
        if (rr0 == kk) {
#pragma unroll
          for (int j = 0; j < 8; ++j) rowk[tj * 8 + j] = m[rr0][j];
        }
      }
    }
    __syncthreads();
    const float piv = colk[k];
    const float inv_p = __frcp_rn(piv);
    // the pivot column and row through 16-byte loads (bank-conflict-free)
    const float4 c0 = *reinterpret_cast<const float4*>(colk + ti * 8);
    const float4 c1 = *reinterpret_cast<const float4*>(colk + ti * 8 + 4);
    const float4 r0 = *reinterpret_cast<const float4*>(rowk + tj * 8);
    const float4 r1 = *reinterpret_cast<const float4*>(rowk + tj * 8 + 4);
    const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
    float cr[8], rr[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) cr[i] = (ti * 8 + i == k) ? piv - 1.f : cv[i];
#pragma unroll
    for (int j = 0; j < 8; ++j) rr[j] = ((tj * 8 + j == k) ? piv + 1.f : rv[j]) * inv_p;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) m[i][j] = fmaf(-cr[i], rr[j], m[i][j]);
    __syncthreads();
  }
  // symmetrise through shared memory, transition = diag(alpha) inv
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) Ms[(ti * 8 + i) * SPD_LD + tj * 8 + j] = m[i][j];
  __syncthreads();
  const float* al = alpha + mat * 128;
  float* tr = trans + mat * 16384;
#pragma unroll
  for (int j = 0; j < 8; ++j) {   // row tj*8+j of M holds column tj*8+j of M^T
    const float4 t0 = *reinterpret_cast<const float4*>(Ms + (tj * 8 + j) * SPD_LD + ti * 8);
    const float4 t1 = *reinterpret_cast<const float4*>(Ms + (tj * 8 + j) * SPD_LD + ti * 8 + 4);
    const float tv[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i][j] = 0.5f * (m[i][j] + tv[i]);
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = ti * 8 + i;
    const float ar = al[r];
#pragma unroll
    for (int j = 0; j < 8; ++j) Ms[r * SPD_LD + tj * 8 + j] = m[i][j];
    float4* dst = reinterpret_cast<float4*>(tr + r * 128 + tj * 8);
    dst[0] = make_float4(ar * m[i][0], ar * m[i][1], ar * m[i][2], ar * m[i][3]);
    dst[1] = make_float4(ar * m[i][4], ar * m[i][5], ar * m[i][6], ar * m[i][7]);
  }
  __syncthreads();
  // injection = (b_scale * B) @ inv, B staged k-major through shared memory in chunks so
  // the inner loop is four 16-byte shared loads per 64 FMAs
  const float* bm = B + mat * 16384;
  float* out = inj + mat * 16384;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) m[i][j] = 0.f;
  for (int k0 = 0; k0 < 128; k0 += SPD_BK) {
    __syncthreads();   // the previous chunk is consumed
    for (int e = tid; e < 128 * SPD_BK; e += 256) {
      const int row = e / SPD_BK, kk = e % SPD_BK;
      Bt[kk * SPD_LD + row] = bm[row * 128 + k0 + kk];
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < SPD_BK; ++kk) {
      const float4 b0 = *reinterpret_cast<const float4*>(Bt + kk * SPD_LD + ti * 8);
      const float4 b1 = *reinterpret_cast<const float4*>(Bt + kk * SPD_LD + ti * 8 + 4);
      const float4 m0 = *reinterpret_cast<const float4*>(Ms + (k0 + kk) * SPD_LD + tj * 8);
      const float4 m1 = *reinterpret_cast<const float4*>(Ms + (k0 + kk) * SPD_LD + tj * 8 + 4);
      const float bi[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      const float mj[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) m[i][j] = fmaf(bi[i], mj[j], m[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4* dst = reinterpret_cast<float4*>(out + (ti * 8 + i) * 128 + tj * 8);
    dst[0] = make_float4(b_scale * m[i][0], b_scale * m[i][1], b_scale * m[i][2], b_scale * m[i][3]);
    dst[1] = make_float4(b_scale * m[i][4], b_scale * m[i][5], b_scale * m[i][6], b_scale * m[i][7]);
  }
}

void launch_lb_spd_factor(const float* A, const float* B, const float* alpha, float* trans,
                          float* inj, int n_mats, float a_scale, float b_scale,
                          cudaStream_t stream) {
  if (!n_mats) return;
  static std::atomic<uint64_t> attr{0};
  if (attr_needed(attr)) {
    cudaFuncSetAttribute(lb_spd_factor_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SPD_SMEM);
    attr_done(attr);
  }
  lb_spd_factor_kernel<<<n_mats, 256, SPD_SMEM, stream>>>(A, B, alpha, trans, inj, a_scale, b_scale);
}

// ------------------------------------------------------------------------------ scans
constexpr int SC_PITCH = 132;
constexpr int SC_SMEM = 2 * 128 * SC_PITCH * 4;

__global__ void __launch_bounds__(256) lb_scan_kernel(const float* __restrict__ trans,
                                                      const float* __restrict__ inj,
                                                      const float* __restrict__ start, int F,
                                                      int H, float* __restrict__ prefix,
                                                      float* __restrict__ suffix) {
  extern __shared__ float sm[];
  float* St = sm;                       // state [128][SC_PITCH]
  float* Tm = sm + 128 * SC_PITCH;      // transition
  const int h = blockIdx.x, dir = blockIdx.y;
  const int tid = threadIdx.x;
  const int ti = tid >> 4, tj = tid & 15;
  for (int i = tid; i < 16384; i += 256) {
    const int r = i >> 7, c = i & 127;
    St[r * SC_PITCH + c] = start ? start[(int64_t)h * 16384 + i] : 0.f;
  }
  float* bank = dir == 0 ? prefix : suffix;
  for (int step = 0; step < F; ++step) {
    const int f = dir == 0 ? step : F - 1 - step;
    const int64_t base = ((int64_t)f * H + h) * 16384;
    const float4* t4 = reinterpret_cast<const float4*>(trans + base);
    for (int i = tid; i < 4096; i += 256) {
      const int r = i >> 5, c4 = i & 31;
      *reinterpret_cast<float4*>(&Tm[r * SC_PITCH + c4 * 4]) = t4[i];
    }
    __syncthreads();
    float acc[8][8];
    const float* ij = inj + base;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 a0 = *reinterpret_cast<const float4*>(ij + (ti * 8 + i) * 128 + tj * 8);
      const float4 a1 = *reinterpret_cast<const float4*>(ij + (ti * 8 + i) * 128 + tj * 8 + 4);
      acc[i][0] = a0.x; acc[i][1] = a0.y; acc[i][2] = a0.z; acc[i][3] = a0.w;
      acc[i][4] = a1.x; acc[i][5] = a1.y; acc[i][6] = a1.z; acc[i][7] = a1.w;
    }
#pragma unroll 4
    for (int k = 0; k < 128; ++k) {
      float si[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) si[i] = St[(ti * 8 + i) * SC_PITCH + k];
      const float4 m0 = *reinterpret_cast<const float4*>(&Tm[k * SC_PITCH + tj * 8]);
      const float4 m1 = *reinterpret_cast<const float4*>(&Tm[k * SC_PITCH + tj * 8 + 4]);
      const float mj[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] += si[i] * mj[j];
    }
    __syncthreads();
    float* ob = bank + base;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = ti * 8 + i;
      *reinterpret_cast<float4*>(&St[r * SC_PITCH + tj * 8]) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      *reinterpret_cast<float4*>(&St[r * SC_PITCH + tj * 8 + 4]) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
      *reinterpret_cast<float4*>(ob + r * 128 + tj * 8) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      *reinterpret_cast<float4*>(ob + r * 128 + tj * 8 + 4) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
    }
    __syncthreads();
  }
}

// Row-split scan for few heads (one rank's share under sequence parallelism). Each row of
// the state evolves on its own, S_new[r, :] = S[r, :] T + inj[r, :], so the 128 rows of a
// (head, direction) recurrence are split over RS independent CTAs (no communication): a
// CTA keeps its 128/RS state rows in shared memory and streams the full transition of
// each frame through a 2-slot ring filled by one bulk copy per frame (the copy of frame
// t+1 lands while frame t computes; the RS CTAs of a head read the same T from L2). The
// serial step count stays F; the work per step and CTA drops by RS.
template <int RS, int NSLOT>
__global__ void __launch_bounds__(256, NSLOT == 1 ? 2 : 1) lb_scan_rows_kernel(
    const float* __restrict__ trans, const float* __restrict__ inj,
    const float* __restrict__ start, int F, int H, float* __restrict__ prefix,
    float* __restrict__ suffix, int* err) {
  constexpr int NR = 128 / RS;            // state rows of this CTA
  constexpr int RT = NR * 128 / 256 / 4;  // rows per thread (4 columns per thread)
  constexpr int CG = 32;                  // column groups of 4
  static_assert(RT >= 1 && CG * (NR / RT) == 256, "thread tiling");
  extern __shared__ __align__(16) float smf[];
  float* Tb = smf;                              // [NSLOT][128][128] transition ring
  float* St = smf + NSLOT * 16384;              // [NR][SC_PITCH] state rows
  uint64_t* full = reinterpret_cast<uint64_t*>(St + NR * SC_PITCH);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 2);
  const int h = blockIdx.x / RS, part = blockIdx.x % RS, dir = blockIdx.y;
  const int row0 = part * NR;
  const int tid = threadIdx.x;
  const int tj = tid % CG, ti = tid / CG;       // column group, row group
  const int c = tj * 4;
  for (int i = tid; i < NR * 128; i += 256) {
    const int r = i >> 7, cc = i & 127;
    St[r * SC_PITCH + cc] = start ? start[(int64_t)h * 16384 + (row0 + r) * 128 + cc] : 0.f;
  }
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  float* bank = dir == 0 ? prefix : suffix;
  auto base_of = [&](int step) {
    const int f = dir == 0 ? step : F - 1 - step;
    return ((int64_t)f * H + h) * 16384;
  };
  int issued = 0, done = 0;               // copies issued / consumed (thread 0's view)
  auto issue = [&](int step) {            // thread 0: T of frame `step` into slot step % NSLOT
    ++issued;
    uint64_t* bar = &full[step % NSLOT];
    mbar_arrive_expect_tx(bar, 16384 * 4);
    bulk_load(Tb + (step % NSLOT) * 16384, trans + base_of(step), 16384 * 4, bar);
  };
  if (tid == 0) {
    for (int q = 0; q < NSLOT && q < F; ++q) issue(q);
  }
  float4 inx[RT];
#pragma unroll
  for (int i = 0; i < RT; ++i)
    inx[i] = __ldg(reinterpret_cast<const float4*>(inj + base_of(0) + (row0 + ti * RT + i) * 128 + c));
  bool ok = true;
  for (int step = 0; step < F; ++step) {
    ok = mbar_wait(&full[step % NSLOT], (uint32_t)((step / NSLOT) & 1), abort_flag, err,
                   kErrTimeoutProducer);
    if (__syncthreads_or(!ok)) break;
    done = step + 1;
    float4 acc[RT];
#pragma unroll
    for (int i = 0; i < RT; ++i) acc[i] = inx[i];
    if (step + 1 < F) {
#pragma unroll
      for (int i = 0; i < RT; ++i)
        inx[i] = __ldg(reinterpret_cast<const float4*>(inj + base_of(step + 1) +
                                                      (row0 + ti * RT + i) * 128 + c));
    }
    const float* T = Tb + (step % NSLOT) * 16384;
#pragma unroll 4
    for (int k = 0; k < 128; ++k) {
      const float4 m = *reinterpret_cast<const float4*>(&T[k * 128 + c]);
#pragma unroll
      for (int i = 0; i < RT; ++i) {
        const float si = St[(ti * RT + i) * SC_PITCH + k];
        acc[i].x = fmaf(si, m.x, acc[i].x);
        acc[i].y = fmaf(si, m.y, acc[i].y);
        acc[i].z = fmaf(si, m.z, acc[i].z);
        acc[i].w = fmaf(si, m.w, acc[i].w);
      }
    }
    __syncthreads();     // every thread has read the state and this step's slot
    if (tid == 0 && step + NSLOT < F) issue(step + NSLOT);
    float* ob = bank + base_of(step);
#pragma unroll
    for (int i = 0; i < RT; ++i) {
      const int r = ti * RT + i;
      *reinterpret_cast<float4*>(&St[r * SC_PITCH + c]) = acc[i];
      *reinterpret_cast<float4*>(ob + (row0 + r) * 128 + c) = acc[i];
    }
  }
  // an aborted block waits (bounded) for its own copies in flight before exiting
  if (tid == 0 && *abort_flag) {
    const long long t0 = clock64();
    for (int q = done; q < issued; ++q)
      while (!mbar_try_wait(&full[q % NSLOT], (uint32_t)((q / NSLOT) & 1)) &&
             clock64() - t0 < kWaitBudgetCycles) {
      }
  }
}

template <int RS, int NSLOT>
static void launch_scan_rows(const float* trans, const float* inj, const float* start, int F,
                             int H, float* prefix, float* suffix, int* err, int ndir,
                             cudaStream_t stream) {
  constexpr int smem = (NSLOT * 16384 + (128 / RS) * SC_PITCH) * 4 + 64;
  static std::atomic<uint64_t> attr{0};
  if (attr_needed(attr)) {
    cudaFuncSetAttribute(lb_scan_rows_kernel<RS, NSLOT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         smem);
    cudaFuncSetAttribute(lb_scan_rows_kernel<RS, NSLOT>,
                         cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
    attr_done(attr);
  }
  lb_scan_rows_kernel<RS, NSLOT><<<dim3(H * RS, ndir), 256, smem, stream>>>(trans, inj, start, F, H,
                                                                             prefix, suffix, err);
}

// Row split for the scan: the largest of 1, 2, 4, 8 that keeps all nrec*RS CTAs resident
// (one per SM) on the device; nrec = heads x directions.
static int scan_cluster_size(int nrec) {
  const int sms = num_sms();
  int cs = 1;
  while (cs < 8 && nrec * cs * 2 <= sms) cs *= 2;
  return cs;
}

static int g_scan_cluster = 0;   // 0: automatic; else forced: 1 (one CTA per recurrence),
                                 // 2, 4, 8 (row parts, two slots), -2 (two parts, one slot)
void lb_scan_set_cluster(int cs) { g_scan_cluster = cs; }

// ndir = 2: both recurrences (prefix and suffix banks); ndir = 1: the prefix recurrence
// only (grid.y = 1, so every CTA takes direction 0 and `suffix` is never touched).
void launch_lb_scan(const float* trans, const float* inj, const float* start, int F, int H,
                    float* prefix, float* suffix, int* err, cudaStream_t stream, int ndir) {
  if (!F || !H) return;
  const int nrec = H * ndir;
  static std::atomic<uint64_t> attr{0};
  if (attr_needed(attr)) {
    cudaFuncSetAttribute(lb_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SC_SMEM);
    attr_done(attr);
  }
  // many heads: two half-row CTAs per recurrence at two CTAs per SM (one transition slot);
  // few heads: 2, 4 or 8 row parts per recurrence, one CTA per SM, two transition slots
  const int cs = g_scan_cluster ? g_scan_cluster : scan_cluster_size(nrec);
  if (cs == -2 || (cs == 1 && !g_scan_cluster && nrec * 2 <= 2 * num_sms())) {
    launch_scan_rows<2, 1>(trans, inj, start, F, H, prefix, suffix, err, ndir, stream);
    return;
  }
  switch (cs) {
    case 2: launch_scan_rows<2, 2>(trans, inj, start, F, H, prefix, suffix, err, ndir, stream); return;
    case 4: launch_scan_rows<4, 2>(trans, inj, start, F, H, prefix, suffix, err, ndir, stream); return;
    case 8: launch_scan_rows<8, 2>(trans, inj, start, F, H, prefix, suffix, err, ndir, stream); return;
    default: break;
  }
  lb_scan_kernel<<<dim3(H, ndir), 256, SC_SMEM, stream>>>(trans, inj, start, F, H, prefix, suffix);
}

// ----------------------------------------------------------------------------- gather
// out[t,h,v,k] = before(t)[v,k] * ab[t,h,k] + after(t)[v,k] * aa[t,h,k]; a missing side
// reads the scan start (text state) or zero.
__global__ void __launch_bounds__(256) lb_gather_kernel(
    const float* __restrict__ prefix, const float* __restrict__ suffix,
    const int* __restrict__ idx /*[F,4]: bi, ai, has_b, has_a*/, const float* __restrict__ ab,
    const float* __restrict__ aa, const float* __restrict__ start, int F, int H,
    __nv_bfloat16* __restrict__ out) {
  const int64_t i4 = (int64_t)blockIdx.x * 256 + threadIdx.x;   // one float4 per thread
  const int64_t total4 = (int64_t)F * H * 4096;
  if (i4 >= total4) return;
  const int64_t e = i4 * 4;
  const int t = (int)(e / ((int64_t)H * 16384));
  const int h = (int)((e / 16384) % H);
  const int vk = (int)(e % 16384);
  const int kcol = vk & 127;
  const int* ix = idx + 4 * t;
  float4 b, a;
  const int64_t off_b = ((int64_t)ix[0] * H + h) * 16384 + vk;
  const int64_t off_a = ((int64_t)ix[1] * H + h) * 16384 + vk;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 st = start ? *reinterpret_cast<const float4*>(start + (int64_t)h * 16384 + vk) : zero;
  b = ix[2] ? *reinterpret_cast<const float4*>(prefix + off_b) : st;
  a = ix[3] ? *reinterpret_cast<const float4*>(suffix + off_a) : st;
  const float* fb = ab + ((int64_t)t * H + h) * 128 + kcol;
  const float* fa = aa + ((int64_t)t * H + h) * 128 + kcol;
  const float o0 = b.x * fb[0] + a.x * fa[0], o1 = b.y * fb[1] + a.y * fa[1];
  const float o2 = b.z * fb[2] + a.z * fa[2], o3 = b.w * fb[3] + a.w * fa[3];
  *reinterpret_cast<uint2*>(out + e) = make_uint2(pack_bf16(o0, o1), pack_bf16(o2, o3));
}

void launch_lb_gather(const float* prefix, const float* suffix, const int* idx, const float* ab,
                      const float* aa, const float* start, int F, int H, void* out,
                      cudaStream_t stream) {
  const int64_t total4 = (int64_t)F * H * 4096;
  if (!total4) return;
  lb_gather_kernel<<<(unsigned)((total4 + 255) / 256), 256, 0, stream>>>(
      prefix, suffix, idx, ab, aa, start, F, H, reinterpret_cast<__nv_bfloat16*>(out));
}

// ---------------------------------------------------------------------------- readout
// CTA = (frame, head, 128-token tile). R = Q_tile . S^T on tcgen05 (both K-major), then
// thread = token: RMSNorm over the 128 outputs, * w * sigmoid(gate), bf16 store in token
// order into the O-projection input.
constexpr int RO_TILE = 128 * 128 * 2;
constexpr int RO_SMEM = 2 * RO_TILE + 1024 + 64;

__global__ void __launch_bounds__(128) lb_readout_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmS, int S,
    int H, const float* __restrict__ w, const __nv_bfloat16* __restrict__ gate, int64_t ldg,
    int gate_logits, __nv_bfloat16* __restrict__ out, int64_t ldo, float eps, int* err,
    const RowScatter scatter) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * RO_TILE);
  uint64_t* done = full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tiles_per_frame = (S + 127) / 128;
  const int mt = blockIdx.x % tiles_per_frame;
  const int fh = blockIdx.x / tiles_per_frame;
  const int f = fh / H, h = fh % H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(full, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int row0 = f * S + mt * 128;
  if (tid == 0) {
    mbar_arrive_expect_tx(full, 2 * RO_TILE);
    tma_load_2d(smem, &tmQ, full, h * 128, row0);
    tma_load_2d(smem + RO_TILE / 2, &tmQ, full, h * 128 + 64, row0);
    tma_load_2d(smem + RO_TILE, &tmS, full, 0, fh * 128);
    tma_load_2d(smem + RO_TILE + RO_TILE / 2, &tmS, full, 64, fh * 128);
    if (mbar_wait(full, 0, abort_flag, err, kErrTimeoutMma)) {
      tc_fence_after();
      constexpr uint32_t idesc = umma_idesc_bf16(128, 128, false, false);
      const uint32_t aQ = smem_u32(smem), aS = smem_u32(smem + RO_TILE);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t off = (k >> 2) * (RO_TILE / 2) + (k & 3) * 32;
        umma_f16_ss(tmem, umma_desc_kmajor_sw128(aQ + off), umma_desc_kmajor_sw128(aS + off),
                    idesc, k != 0);
      }
    }
    umma_commit(done);
  }
  const bool ok = mbar_wait(done, 0, abort_flag, err, kErrTimeoutEpilogue) && !*abort_flag;
  if (ok) {
    tc_fence_after();
    const int r = warp * 32 + lane;
    const int tok = mt * 128 + r;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float v[128];
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      uint32_t u[32];
      tmem_ld32(tmem + lane_off + c, u);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) v[c + i] = __uint_as_float(u[i]);
    }
    if (tok < S) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) ss += v[i] * v[i];
      const float rstd = rsqrtf(ss / 128.f + eps);
      const int64_t row = (int64_t)f * S + tok;
      const __nv_bfloat16* g = gate + row * ldg + h * 128;
      __nv_bfloat16* o = scatter.row_ptr(out, ldo, row) + h * 128;
#pragma unroll
      for (int c = 0; c < 128; c += 8) {
        const uint4 gv = *reinterpret_cast<const uint4*>(g + c);
        const uint32_t* gu = reinterpret_cast<const uint32_t*>(&gv);
        uint32_t pk[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float g0 = bf16_lo(gu[j]), g1 = bf16_hi(gu[j]);
          if (gate_logits) {
            g0 = sigmoidf_(g0);
            g1 = sigmoidf_(g1);
          }
          pk[j] = pack_bf16(v[c + 2 * j] * rstd * w[c + 2 * j] * g0,
                            v[c + 2 * j + 1] * rstd * w[c + 2 * j + 1] * g1);
        }
        *reinterpret_cast<uint4*>(o + c) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

void launch_lb_readout(const void* q, int64_t ldq, const void* state, int F, int S, int H,
                       const float* w, const void* gate, int64_t ldg, int gate_logits, void* out,
                       int64_t ldo, float eps, int* err, cudaStream_t stream,
                       const RowScatter* scatter) {
  if (!F || !S || !H) return;
  static std::atomic<uint64_t> attr{0};
  if (attr_needed(attr)) {
    cudaFuncSetAttribute(lb_readout_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RO_SMEM);
    attr_done(attr);
  }
  CUtensorMap tq = make_tmap_2d(q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)H * 128,
                                (uint64_t)F * S, ldq * 2, 64, 128);
  CUtensorMap ts = make_tmap_2d(state, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128,
                                (uint64_t)F * H * 128, 256, 64, 128);
  const int tiles = F * H * ((S + 127) / 128);
  lb_readout_kernel<<<tiles, 128, RO_SMEM, stream>>>(
      tq, ts, S, H, w, reinterpret_cast<const __nv_bfloat16*>(gate), ldg, gate_logits,
      reinterpret_cast<__nv_bfloat16*>(out), ldo, eps, err, scatter ? *scatter : RowScatter{});
}

}  // namespace vdn
