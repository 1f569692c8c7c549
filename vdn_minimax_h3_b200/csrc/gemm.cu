// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[M, N] = A[M, K] @ B[N, K]^T      (both operands K-major, i.e. nn.Linear layout)
//
// or, for the two products of a Linear's backward, with either operand stored MN-major
// (template LAYOUT: bit 0 = A held as [K, M], bit 1 = B held as [K, N], rows contiguous):
//   dgrad  dX = dY W        A = dY [T, out] K-major, B = W [out, in] read as [K, N]
//   wgrad  dW = dY^T X      A = dY read as [K=T, M=out], B = X [T, in] read as [K, N]
// An MN-major operand arrives as 64-column boxes (64 K-rows x 128 B each, 128-byte swizzle)
// and is described to tcgen05.mma as MN-major with the box size as the stride between the
// 64-wide MN atoms, so neither backward product needs a transposed copy.
//
// One CTA per SM, 128x256 output tiles, 64-deep K blocks:
//   warp 0      TMA producer: A and B tiles into a 4-stage shared-memory ring
//               (128-byte swizzle), completion counted by mbarrier transaction bytes.
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma (M=128, N=256, K=16)
//               into a TMEM accumulator; tcgen05.commit frees each smem stage and
//               signals a finished accumulator. Two accumulators (2 x 256 TMEM columns)
//               so the epilogue of tile i overlaps the main loop of tile i+1.
//   warps 2-5   epilogue: tcgen05.ld 32x32b.x32 (thread = output row), fused math, store.
//
// Fused epilogues (the elementwise work that follows each DiT GEMM in the reference's
// block forward, src/models/ops/fused_block.py:41-90):
//   EPI_STORE      C = acc (+ bias)
//   EPI_RESIDUAL   X += gate[adaln_idx[row]] * (acc + bias)       (the gated residual)
//   EPI_SWIGLU     H = (acc_v + b_v) * silu(acc_g + b_g); the weight rows are interleaved
//                  per 256-row tile as [128 value rows | 128 gate rows]
//   EPI_ADD        C += acc (+ bias)                               (accumulate into C)
//   EPI_STORE_F32  C without bias as bf16, each row stored to its owner's buffer (the
//                  reduce-scatter of a row-parallel GEMM: partial sums cross NVLink once)
//   EPI_ROUTE      every 8-column group of a row goes to its own destination (a route
//                  table of addresses), and the 128-column q/k heads additionally get the
//                  per-head RMSNorm + rotate-half RoPE of the attention input
//                  (softmax_attention/kernels.py:27-30) written to a second route. One
//                  GEMM thus emits raw q/k/v/gates, normalised+rotated q/k, and places
//                  each head where its consumer reads it: the attention's q/k buffers on
//                  one GPU, or the Ulysses receive slabs (local or a peer's, through an
//                  IPC mapping) under sequence parallelism.
//
// Every wait is bounded (common.cuh): a protocol failure records an error code, unwinds
// the CTA, drains its own copies and MMAs and frees its TMEM instead of hanging the GPU.
#include "common.cuh"
#include "tma.cuh"
#include "launchers.h"

namespace vdn {

constexpr int GM_BM = 128;
constexpr int GM_BN = 256;
constexpr int GM_BK = 64;
constexpr int GM_STAGES = 4;
constexpr int GM_A_BYTES = GM_BM * GM_BK * 2;  // 16 KB
constexpr int GM_B_BYTES = GM_BN * GM_BK * 2;  // 32 KB
constexpr int GM_STAGE_BYTES = GM_A_BYTES + GM_B_BYTES;
constexpr int GM_THREADS = 192;
constexpr int GM_GROUP_N = 16;  // n-blocks per raster band (weights of one band stay in L2)
constexpr int GM_ROUTE_STAGE = 4 * 32 * 5 * 16;  // epilogue warps' route staging (10 KB)
constexpr int GM_SMEM = GM_STAGES * GM_STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + GM_ROUTE_STAGE;
constexpr int kMaxRoutePlanes = 8;

enum EpiMode : int { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ADD = 3, EPI_ROUTE = 4,
                    EPI_STORE_F32 = 5 };

struct EpiParams {
  __nv_bfloat16* out;        // C / X / H
  int64_t ldo;               // row stride of `out` (elements)
  const float* bias;         // [N] fp32 or null
  const __nv_bfloat16* gate; // EPI_RESIDUAL: gate table [rows, ldg]
  int64_t ldg;
  const int* gate_idx;       // EPI_RESIDUAL: per-row table index
  int* err;                  // device error word
  RowScatter scatter;           // EPI_STORE_F32: rows to their tensor-parallel owners
  // EPI_ROUTE
  const long long* route;       // [planes][N/8] address of (row 0, column 8g), 0 = no store
  int64_t route_ld[kMaxRoutePlanes];  // row stride (elements) of each plane's destinations
  int planes;
  int q0, q1, k0, k1;           // GEMM column ranges of the q heads and the k heads
  const float* norm_q;          // [128] per-head RMSNorm weights
  const float* norm_k;
  float qk_eps;
  const float* rope_cos;        // [M, ld_rope] fp32, rotate-half layout (cos[j] == cos[j+64])
  const float* rope_sin;
  int64_t ld_rope;
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  // n-band major raster: a band of GM_GROUP_N n-blocks sweeps all of M.
  int band_size = GM_GROUP_N * num_m;
  int band = tile / band_size;
  int in_band = tile - band * band_size;
  int n0 = band * GM_GROUP_N;
  int gn = min(GM_GROUP_N, num_n - n0);
  mb = in_band / gn;
  nb = n0 + (in_band - mb * gn);
}

// EPI_ROUTE helpers ------------------------------------------------------------------------
// Warp-cooperative store of one 32-column chunk of 32 rows (lane = row, 16 packed bf16
// pairs per lane) through the route: the chunk is transposed through a 2.5 KB shared
// staging area so that each store instruction writes 8 rows x 64 contiguous bytes instead
// of 32 rows x 16 bytes -- the destinations are often a peer GPU's memory, where small
// scattered writes waste NVLink bandwidth. Every lane of the warp must call it.
constexpr int kRouteStageWords = 32 * 5;   // uint4 per warp: 32 rows x (4 + 1 pad)

__device__ __forceinline__ void route_store_chunk(const long long* route, int64_t ld, int col,
                                                  int ngroups, int row_base, int M,
                                                  uint4* stage, const uint32_t* packed) {
  const int lane = lane_id();
#pragma unroll
  for (int g = 0; g < 4; ++g)
    stage[lane * 5 + g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
  __syncwarp();
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int r = step * 8 + (lane >> 2), g = lane & 3;
    const int row = row_base + r;
    if (g < ngroups && row < M) {
      const long long dst = __ldg(route + (col >> 3) + g);
      if (dst)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst) + (int64_t)row * ld) =
            stage[r * 5 + g];
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void epilogue_route(const EpiParams& p, uint32_t lane_base, int row,
                                               bool row_ok, int n0, int N, int M, uint4* stage) {
  const int row_base = row - lane_id();
#pragma unroll 1
  for (int h2 = 0; h2 < GM_BN; h2 += 128) {
    const int hc = n0 + h2;
    if (hc >= N) break;
    const bool isq = hc >= p.q0 && hc < p.q1;
    const bool isk = hc >= p.k0 && hc < p.k1;
    if (isq || isk) {
      // One q/k head per thread-row: raw values rounded to bf16 (the projection's output
      // dtype), RMS over the head, then rotate-half RoPE on the normalised values.
      uint32_t hv[64];
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < 128; c += 32) {
        uint32_t v[32];
        tmem_ld32(lane_base + h2 + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float a0 = __uint_as_float(v[j]), a1 = __uint_as_float(v[j + 1]);
          if (p.bias) {
            a0 += __ldg(p.bias + hc + c + j);
            a1 += __ldg(p.bias + hc + c + j + 1);
          }
          const uint32_t pk = pack_bf16(a0, a1);
          hv[(c + j) >> 1] = pk;
          const float r0 = bf16_lo(pk), r1 = bf16_hi(pk);
          ss = fmaf(r0, r0, fmaf(r1, r1, ss));
        }
        route_store_chunk(p.route, p.route_ld[0], hc + c, 4, row_base, M, stage, hv + (c >> 1));
      }
      const float rstd = rsqrtf(ss * (1.f / 128.f) + p.qk_eps);
      const float* w = isq ? p.norm_q : p.norm_k;
      // rows past M have no rope table row: they compute on row 0 and are not stored
      const int64_t rrow = row_ok ? row : 0;
      const float4* cr = reinterpret_cast<const float4*>(p.rope_cos + rrow * p.ld_rope);
      const float4* sr = reinterpret_cast<const float4*>(p.rope_sin + rrow * p.ld_rope);
      const long long* proc = p.route + (N >> 3);  // plane 1: processed q/k
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 c4 = __ldg(cr + ((c + j) >> 2));
          const float4 s4 = __ldg(sr + ((c + j) >> 2));
          const float cs[4] = {c4.x, c4.y, c4.z, c4.w};
          const float sn[4] = {s4.x, s4.y, s4.z, s4.w};
          float o1[4], o2[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i1 = c + j + e, i2 = i1 + 64;
            const uint32_t u1 = hv[i1 >> 1], u2 = hv[i2 >> 1];
            const float x1 = ((i1 & 1) ? bf16_hi(u1) : bf16_lo(u1)) * rstd * __ldg(w + i1);
            const float x2 = ((i2 & 1) ? bf16_hi(u2) : bf16_lo(u2)) * rstd * __ldg(w + i2);
            // cos/sin repeat with period 64 in the rotate-half layout
            o1[e] = x1 * cs[e] - x2 * sn[e];
            o2[e] = x2 * cs[e] + x1 * sn[e];
          }
          lo[j >> 1] = pack_bf16(o1[0], o1[1]);
          lo[(j >> 1) + 1] = pack_bf16(o1[2], o1[3]);
          hi[j >> 1] = pack_bf16(o2[0], o2[1]);
          hi[(j >> 1) + 1] = pack_bf16(o2[2], o2[3]);
        }
        route_store_chunk(proc, p.route_ld[1], hc + c, 4, row_base, M, stage, lo);
        route_store_chunk(proc, p.route_ld[1], hc + c + 64, 4, row_base, M, stage, hi);
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t v[32];
        tmem_ld32(lane_base + h2 + c, v);
        tmem_wait_ld();
        const int col0 = hc + c;
        if (col0 >= N) continue;   // warp-uniform
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float a0 = __uint_as_float(v[j]), a1 = __uint_as_float(v[j + 1]);
          if (p.bias && col0 + j < N) {
            a0 += __ldg(p.bias + col0 + j);
            a1 += __ldg(p.bias + col0 + j + 1);
          }
          packed[j >> 1] = pack_bf16(a0, a1);
        }
        // N is a multiple of 8, so a partial chunk ends on a whole 8-column group. Every
        // plane with an address receives a copy (e.g. a field replicated to all ranks).
        const int ngroups = min(4, (N - col0) >> 3);
#pragma unroll 1
        for (int pl = 0; pl < p.planes; ++pl)
          route_store_chunk(p.route + (int64_t)pl * (N >> 3), p.route_ld[pl], col0, ngroups,
                            row_base, M, stage, packed);
      }
    }
  }
}

template <int EPI>
__device__ __forceinline__ void epilogue_tile(const EpiParams& p, uint32_t tacc, int quarter,
                                              int m0, int n0, int M, int N, uint4* stage) {
  const int lane = lane_id();
  const int row = m0 + quarter * 32 + lane;
  const uint32_t lane_base = tacc + ((uint32_t)(quarter * 32) << 16);
  const bool row_ok = row < M;
  if constexpr (EPI == EPI_ROUTE) {
    epilogue_route(p, lane_base, row, row_ok, n0, N, M, stage);
    return;
  }
  if constexpr (EPI == EPI_STORE_F32) {
    // bf16 partial products without bias, each row to its owner's buffer, staged so each
    // store writes 8 rows x 64 contiguous bytes
    const int row_base = m0 + quarter * 32;
#pragma unroll 1
    for (int c = 0; c < GM_BN; c += 32) {
      uint32_t v[32];
      tmem_ld32(lane_base + c, v);
      tmem_wait_ld();
      const int col0 = n0 + c;
      if (col0 >= N) continue;   // warp-uniform
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) packed[j] = pack_bf16(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
#pragma unroll
      for (int g = 0; g < 4; ++g)
        stage[lane * 5 + g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
      __syncwarp();
#pragma unroll
      for (int step = 0; step < 4; ++step) {
        const int rr = step * 8 + (lane >> 2), g = lane & 3;
        const int srow = row_base + rr;
        if (srow < M) {
          __nv_bfloat16* d = (p.scatter.n == 0 ? p.out + (int64_t)srow * p.ldo
                                               : p.scatter.row_ptr(p.out, p.ldo, srow)) + col0 + 8 * g;
          *reinterpret_cast<uint4*>(d) = stage[rr * 5 + g];
        }
      }
      __syncwarp();
    }
    return;
  }
  if constexpr (EPI == EPI_SWIGLU) {
    // columns [0,128) value, [128,256) gate -> 128 outputs at n0/2.
    const int out_c0 = n0 >> 1;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      uint32_t v[32], g[32];
      tmem_ld32(lane_base + c, v);
      tmem_ld32(lane_base + 128 + c, g);
      tmem_wait_ld();
      if (!row_ok) continue;
      const int oc = out_c0 + c;
      if (oc >= (N >> 1)) continue;
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float a0 = __uint_as_float(v[j]), a1 = __uint_as_float(v[j + 1]);
        float g0 = __uint_as_float(g[j]), g1 = __uint_as_float(g[j + 1]);
        if (p.bias) {
          a0 += p.bias[n0 + c + j];
          a1 += p.bias[n0 + c + j + 1];
          g0 += p.bias[n0 + 128 + c + j];
          g1 += p.bias[n0 + 128 + c + j + 1];
        }
        packed[j >> 1] = pack_bf16(a0 * siluf_(g0), a1 * siluf_(g1));
      }
      uint4* dst = reinterpret_cast<uint4*>(p.out + (int64_t)row * p.ldo + oc);
      if (oc + 32 <= (N >> 1)) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
      } else {
        __nv_bfloat16* d = p.out + (int64_t)row * p.ldo + oc;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (oc + j < (N >> 1)) {
            uint32_t w = packed[j >> 1];
            d[j] = __ushort_as_bfloat16((unsigned short)((j & 1) ? (w >> 16) : (w & 0xFFFF)));
          }
        }
      }
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < GM_BN; c += 32) {
    uint32_t v[32];
    tmem_ld32(lane_base + c, v);
    tmem_wait_ld();
    const int col0 = n0 + c;
    if (!row_ok || col0 >= N) continue;
    const bool full = col0 + 32 <= N;
    float f[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
    if (p.bias) {
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] += p.bias[col0 + j];
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) f[j] += p.bias[col0 + j];
      }
    }
    __nv_bfloat16* orow = p.out + (int64_t)row * p.ldo + col0;
    if constexpr (EPI == EPI_RESIDUAL || EPI == EPI_ADD) {
      const __nv_bfloat16* grow =
          EPI == EPI_RESIDUAL ? p.gate + (int64_t)p.gate_idx[row] * p.ldg + col0 : nullptr;
      if (full) {
        uint4 xr[4], gr[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) xr[q] = reinterpret_cast<const uint4*>(orow)[q];
        if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
          for (int q = 0; q < 4; ++q) gr[q] = reinterpret_cast<const uint4*>(grow)[q];
        }
        const uint32_t* xw = reinterpret_cast<const uint32_t*>(xr);
        const uint32_t* gw = reinterpret_cast<const uint32_t*>(gr);
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y0 = f[2 * j], y1 = f[2 * j + 1];
          if constexpr (EPI == EPI_RESIDUAL) {
            y0 *= bf16_lo(gw[j]);
            y1 *= bf16_hi(gw[j]);
          }
          packed[j] = pack_bf16(bf16_lo(xw[j]) + y0, bf16_hi(xw[j]) + y1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<uint4*>(orow)[q] =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (col0 + j < N) {
            float y = f[j];
            if constexpr (EPI == EPI_RESIDUAL) y *= __bfloat162float(grow[j]);
            orow[j] = __float2bfloat16(__bfloat162float(orow[j]) + y);
          }
        }
      }
    } else {  // EPI_STORE
      if (full) {
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) packed[j] = pack_bf16(f[2 * j], f[2 * j + 1]);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<uint4*>(orow)[q] =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) orow[j] = __float2bfloat16(f[j]);
      }
    }
  }
}

template <int EPI, int LAYOUT>
__global__ void __launch_bounds__(GM_THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, EpiParams p, int M, int N,
                     int K) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GM_STAGES * GM_STAGE_BYTES);
  uint64_t* empty = full + GM_STAGES;
  uint64_t* tfull = empty + GM_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint4* route_stage = reinterpret_cast<uint4*>(smem + GM_STAGES * GM_STAGE_BYTES + 256);

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (M + GM_BM - 1) / GM_BM;
  const int num_n = (N + GM_BN - 1) / GM_BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + GM_BK - 1) / GM_BK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < GM_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, issued_par = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_sleep(&empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * GM_STAGE_BYTES;
          uint8_t* sB = sA + GM_A_BYTES;
          if constexpr (LAYOUT == 0) {
            mbar_arrive_expect_tx(&full[stage], GM_STAGE_BYTES);
            tma_load_2d(sA, &tmA, &full[stage], kb * GM_BK, mb * GM_BM);
            tma_load_2d(sB, &tmB, &full[stage], kb * GM_BK, nb * GM_BN);
          } else {
            // MN-major boxes that start past the edge are not loaded: they would only
            // feed accumulator rows / columns the epilogue never stores.
            const int na = (LAYOUT & 1) ? min(GM_BM / 64, (M - mb * GM_BM + 63) / 64) : 1;
            const int nbx = (LAYOUT & 2) ? min(GM_BN / 64, (N - nb * GM_BN + 63) / 64) : 1;
            const uint32_t bytes = ((LAYOUT & 1) ? na * (GM_A_BYTES / 2) : GM_A_BYTES) +
                                   ((LAYOUT & 2) ? nbx * (GM_B_BYTES / 4) : GM_B_BYTES);
            mbar_arrive_expect_tx(&full[stage], bytes);
            if constexpr ((LAYOUT & 1) != 0) {
              for (int i = 0; i < na; ++i)
                tma_load_2d(sA + i * (GM_A_BYTES / 2), &tmA, &full[stage], mb * GM_BM + 64 * i, kb * GM_BK);
            } else {
              tma_load_2d(sA, &tmA, &full[stage], kb * GM_BK, mb * GM_BM);
            }
            if constexpr ((LAYOUT & 2) != 0) {
              for (int i = 0; i < nbx; ++i)
                tma_load_2d(sB + i * (GM_B_BYTES / 4), &tmB, &full[stage], nb * GM_BN + 64 * i, kb * GM_BK);
            } else {
              tma_load_2d(sB, &tmB, &full[stage], kb * GM_BK, nb * GM_BN);
            }
          }
          issued_mask |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == GM_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain: every load this thread issued must land before the CTA exits.
        for (int s = 0; s < GM_STAGES; ++s) {
          if (!(issued_mask >> s & 1)) continue;
          uint32_t par = (issued_par >> s) & 1;
          long long t0 = clock64();
          while (!mbar_try_wait(&full[s], par) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(GM_BM, GM_BN, (LAYOUT & 1) != 0, (LAYOUT & 2) != 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait_sleep(&tempty[buf], (use & 1) ^ 1, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tacc = tmem_base + buf * GM_BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_sleep(&full[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aaddr = smem_u32(smem + stage * GM_STAGE_BYTES);
          const uint32_t baddr = aaddr + GM_A_BYTES;
#pragma unroll
          for (int k = 0; k < GM_BK / 16; ++k) {
            // K-major: 16 K-elements = 32 B into the swizzled row; MN-major: 16 K-rows of
            // 128 B = 2048 B down the box, 64-wide MN atoms one box apart.
            const uint64_t da = (LAYOUT & 1) ? umma_desc_mnmajor_sw128(aaddr + k * 2048, GM_A_BYTES / 2)
                                             : umma_desc_kmajor_sw128(aaddr + k * 32);
            const uint64_t db = (LAYOUT & 2) ? umma_desc_mnmajor_sw128(baddr + k * 2048, GM_B_BYTES / 4)
                                             : umma_desc_kmajor_sw128(baddr + k * 32);
            umma_f16_ss(tacc, da, db, idesc, (kb | k) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == GM_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&tfull[buf]);
      }
      // All MMAs issued by this thread complete before TMEM is released.
      umma_commit(mma_done);
      long long t0 = clock64();
      while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else {
    const int quarter = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      if (!mbar_wait_sleep(&tfull[buf], use & 1, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      epilogue_tile<EPI>(p, tmem_base + buf * GM_BN, quarter, mb * GM_BM, nb * GM_BN, M, N,
                         route_stage + quarter * kRouteStageWords);
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------------------- host
template <int EPI, int LAYOUT = 0>
static void launch_gemm(const GemmArgs& a, EpiParams p, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_set{0};
  if (attr_needed(attr_set)) {
    cudaFuncSetAttribute(gemm_bf16_kernel<EPI, LAYOUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         GM_SMEM);
    attr_done(attr_set);
  }
  constexpr auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta = (LAYOUT & 1) ? make_tmap_2d(a.A, BF16, 2, a.M, a.K, a.lda * 2, 64, GM_BK)
                                : make_tmap_2d(a.A, BF16, 2, a.K, a.M, a.lda * 2, GM_BK, GM_BM);
  CUtensorMap tb = (LAYOUT & 2) ? make_tmap_2d(a.B, BF16, 2, a.N, a.K, a.ldb * 2, 64, GM_BK)
                                : make_tmap_2d(a.B, BF16, 2, a.K, a.N, a.ldb * 2, GM_BK, GM_BN);
  const int tiles = ((a.M + GM_BM - 1) / GM_BM) * ((a.N + GM_BN - 1) / GM_BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  gemm_bf16_kernel<EPI, LAYOUT><<<grid, GM_THREADS, GM_SMEM, stream>>>(ta, tb, p, a.M, a.N, a.K);
}

void launch_gemm_bf16_routed(const GemmArgs& a, const GemmRoute& r, const float* bias, int* err,
                             cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return;
  EpiParams p{};
  p.bias = bias;
  p.err = err;
  if (r.planes < 1 || r.planes > kMaxRoutePlanes)
    throw std::runtime_error("routed GEMM: 1..8 route planes");
  p.route = r.route;
  p.planes = r.planes;
  for (int i = 0; i < r.planes; ++i) p.route_ld[i] = r.route_ld[i];
  p.q0 = r.q0;
  p.q1 = r.q1;
  p.k0 = r.k0;
  p.k1 = r.k1;
  p.norm_q = r.norm_q;
  p.norm_k = r.norm_k;
  p.qk_eps = r.qk_eps;
  p.rope_cos = r.rope_cos;
  p.rope_sin = r.rope_sin;
  p.ld_rope = r.ld_rope;
  launch_gemm<EPI_ROUTE>(a, p, stream);
}

void launch_gemm_bf16_f32_scatter(const GemmArgs& a, void* out, int64_t ldo, const RowScatter& sc,
                                  int* err, cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return;
  EpiParams p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.scatter = sc;
  p.err = err;
  launch_gemm<EPI_STORE_F32>(a, p, stream);
}

void launch_gemm_bf16(const GemmArgs& a, int mode, void* out, int64_t ldo, const float* bias,
                      const void* gate, int64_t ldg, const int* gate_idx, int* err,
                      cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return;
  EpiParams p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.bias = bias;
  p.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  p.ldg = ldg;
  p.gate_idx = gate_idx;
  p.err = err;
  switch (mode) {
    case EPI_STORE: launch_gemm<EPI_STORE>(a, p, stream); break;
    case EPI_RESIDUAL: launch_gemm<EPI_RESIDUAL>(a, p, stream); break;
    case EPI_SWIGLU: launch_gemm<EPI_SWIGLU>(a, p, stream); break;
    case EPI_ADD: launch_gemm<EPI_ADD>(a, p, stream); break;
    default: throw std::runtime_error("unknown GEMM epilogue mode");
  }
}

void launch_gemm_bf16_layout(const GemmArgs& a, bool a_mn, bool b_mn, bool accumulate, void* out,
                             int64_t ldo, int* err, cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return;
  EpiParams p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.err = err;
  const int layout = (a_mn ? 1 : 0) | (b_mn ? 2 : 0);
  switch (layout * 2 + (accumulate ? 1 : 0)) {
    case 0: launch_gemm<EPI_STORE, 0>(a, p, stream); break;
    case 1: launch_gemm<EPI_ADD, 0>(a, p, stream); break;
    case 2: launch_gemm<EPI_STORE, 1>(a, p, stream); break;
    case 3: launch_gemm<EPI_ADD, 1>(a, p, stream); break;
    case 4: launch_gemm<EPI_STORE, 2>(a, p, stream); break;
    case 5: launch_gemm<EPI_ADD, 2>(a, p, stream); break;
    case 6: launch_gemm<EPI_STORE, 3>(a, p, stream); break;
    default: launch_gemm<EPI_ADD, 3>(a, p, stream); break;
  }
}

}  // namespace vdn
