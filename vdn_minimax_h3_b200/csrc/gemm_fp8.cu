// Block-scaled fp8 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[M, N] = (A[M, K] * sA) @ (B[N, K] * sB)^T
//
// A and B are E4M3 (K-major); sA, sB are power-of-two (UE8M0) scales, one per row and
// 32-element K block, in the blocked layout of common.cuh:sf_offset. The activation
// quantisers write one scale per 1x128 block (replicated over its four 32-blocks), the
// weight quantiser one per 128x128 block: the reference's block-scaled fp8 recipe
// (src/models/ops/fp8_linear.py; 1x128 activation / 128x128 weight scales), applied by the
// tensor core itself (tcgen05.mma kind::mxf8f6f4.block_scale) rather than in the epilogue.
//
// One CTA per SM, 128x256 tiles, 128-deep K blocks in a 4-stage ring, 384 threads:
//   warp 0      TMA: A (128 x 128 B) and B (256 x 128 B) tiles, 128-byte swizzle, plus the
//               stage's scale factors by untiled bulk copies (512 B for A, 1 KB for B).
//   warp 1      MMA issuer: per stage, tcgen05.cp of the scale factors into TMEM
//               (32x128b.warpx4), then four M=128 N=256 K=32 block-scaled MMAs.
//   warps 2-3   idle (they complete warpgroup 0, whose registers go to the epilogue).
//   warps 4-11  epilogue, two warpgroups of 128 columns each. Each thread copies its
//               row's 128 accumulators to registers and frees the accumulator at once, so
//               the next tile's MMAs overlap the epilogue math and stores although TMEM
//               (512 columns: accumulator 0-255, scale factors 256-319) holds only one
//               accumulator.
// Epilogues: STORE (bf16 C + bias), RESIDUAL (X += gate[idx] * (C + bias)), SWIGLU_Q
// (weight rows interleaved per 128 as [64 value | 64 gate]; h = v * silu(g) quantised to
// E4M3 with one scale per 1x64 output block -- each epilogue thread owns 64 outputs of
// its row -- the A operand of the next fp8 GEMM).
//
// Every wait is bounded (common.cuh) and unwinds instead of hanging.
#include "common.cuh"
#include "launchers.h"
#include "tma.cuh"

#include <stdexcept>

namespace vdn {

constexpr int F8_BM = 128;
constexpr int F8_BN = 256;
constexpr int F8_BK = 128;                       // elements = bytes
constexpr int F8_STAGES = 4;
constexpr int F8_A_BYTES = F8_BM * F8_BK;        // 16 KB
constexpr int F8_B_BYTES = F8_BN * F8_BK;        // 32 KB
constexpr int F8_SFA_BYTES = 512;                // 128 rows x 4 K-blocks
constexpr int F8_SFB_BYTES = 1024;               // 256 rows x 4 K-blocks
constexpr int F8_STAGE_BYTES = 51200;            // A | B | SFA | SFB, padded to 1 KB
constexpr int F8_THREADS = 384;
constexpr int F8_ROUTE_STAGE = 8 * 32 * 5 * 16;   // epilogue warps' route staging (20 KB)
constexpr int F8_SMEM = F8_STAGES * F8_STAGE_BYTES + 1024 /*align*/ + 2048 /*barriers*/ + F8_ROUTE_STAGE;
constexpr int F8_SF_COL = 256;                   // TMEM column of the first scale factors
constexpr int F8_SF_STAGE_COLS = 16;             // SFA 4 columns, SFB 8
constexpr int F8_REGS_LOW = 72;
constexpr int F8_REGS_HIGH = 216;
static_assert(F8_A_BYTES + F8_B_BYTES + F8_SFA_BYTES + F8_SFB_BYTES <= F8_STAGE_BYTES, "stage");
static_assert(128 * F8_REGS_LOW + 256 * F8_REGS_HIGH <= F8_THREADS * 168, "register split");

enum Fp8Epi : int { F8_STORE = 0, F8_RESIDUAL = 1, F8_SWIGLU_Q = 2, F8_ROUTE = 3, F8_STORE_F32 = 4 };

struct Fp8Params {
  const uint8_t* sfa;          // blocked scale factors of A
  const uint8_t* sfb;          // blocked scale factors of B (per 256-row tile)
  __nv_bfloat16* out;          // STORE: C, RESIDUAL: X
  int64_t ldo;
  const float* bias;           // [N] or null
  const __nv_bfloat16* gate;   // RESIDUAL
  int64_t ldg;
  const int* gate_idx;
  uint8_t* q_out;              // SWIGLU_Q: E4M3 [M, N/2], row stride ldq
  int64_t ldq;
  uint8_t* q_sf;               // SWIGLU_Q: blocked scale factors of q_out
  GemmRoute route;             // ROUTE: destinations and the q/k head processing
  RowScatter scatter;          // STORE_F32: rows to their tensor-parallel owners
  int* err;
  long long* trace;            // optional: per-CTA cycle counts of the producer / MMA waits
};

// Diagnostics (off unless set): per CTA [0] MMA-thread cycles, [1] of them waiting for
// staged operands, [2] waiting for the accumulator, [3] producer cycles waiting for a free
// stage, [4] tiles.
static long long* g_fp8_trace = nullptr;
void gemm_fp8_set_trace(long long* t) { g_fp8_trace = t; }

// ROUTE epilogue on one 128-column group held in registers: q/k heads get raw stores to
// plane 0 and RMSNorm + rotate-half RoPE stores to plane 1; other columns are stored to
// every plane with an address (the routed epilogue of gemm.cu, here after the accumulator
// has been copied out of TMEM).
// Warp-cooperative store of one 32-column chunk of 32 rows through the route, transposed
// through shared memory so each store instruction writes 8 rows x 64 contiguous bytes (the
// destinations are often a peer GPU's memory). Every lane of the warp must call it.
constexpr int kF8StageWords = 32 * 5;

__device__ __forceinline__ void f8_route_store(const GemmRoute& r, int plane, int N, int col,
                                               int row_base, int M, uint4* stage,
                                               const uint32_t* packed, int ngroups) {
  const long long* tab = r.route + (int64_t)plane * (N >> 3);
  const int lane = lane_id();
#pragma unroll
  for (int g = 0; g < 4; ++g)
    stage[lane * 5 + g] = make_uint4(packed[4 * g], packed[4 * g + 1], packed[4 * g + 2], packed[4 * g + 3]);
  __syncwarp();
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int rr = step * 8 + (lane >> 2), g = lane & 3;
    const int row = row_base + rr;
    if (g < ngroups && row < M) {
      const long long dst = __ldg(tab + (col >> 3) + g);
      if (dst)
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst) + (int64_t)row * r.route_ld[plane]) =
            stage[rr * 5 + g];
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void f8_route_epilogue(const Fp8Params& p, const uint32_t* v, int hc,
                                                  int row, int N, int M, uint4* stage) {
  const int row_base = row - lane_id();
  const bool row_ok = row < M;
  const GemmRoute& r = p.route;
  const bool isq = hc >= r.q0 && hc < r.q1;
  const bool isk = hc >= r.k0 && hc < r.k1;
  if (isq || isk) {
    uint32_t hv[64];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 128; j += 2) {
      float a0 = __uint_as_float(v[j]), a1 = __uint_as_float(v[j + 1]);
      if (p.bias) {
        a0 += __ldg(p.bias + hc + j);
        a1 += __ldg(p.bias + hc + j + 1);
      }
      const uint32_t pk = pack_bf16(a0, a1);
      hv[j >> 1] = pk;
      const float r0 = bf16_lo(pk), r1 = bf16_hi(pk);
      ss = fmaf(r0, r0, fmaf(r1, r1, ss));
    }
#pragma unroll
    for (int c = 0; c < 128; c += 32)
      f8_route_store(r, 0, N, hc + c, row_base, M, stage, hv + (c >> 1), 4);
    const float rstd = rsqrtf(ss * (1.f / 128.f) + r.qk_eps);
    const float* w = isq ? r.norm_q : r.norm_k;
    // rows past M have no rope table row: they compute on row 0 and are not stored
    const int64_t rrow = row_ok ? row : 0;
    const float4* cr = reinterpret_cast<const float4*>(r.rope_cos + rrow * r.ld_rope);
    const float4* sr = reinterpret_cast<const float4*>(r.rope_sin + rrow * r.ld_rope);
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
          o1[e] = x1 * cs[e] - x2 * sn[e];
          o2[e] = x2 * cs[e] + x1 * sn[e];
        }
        lo[j >> 1] = pack_bf16(o1[0], o1[1]);
        lo[(j >> 1) + 1] = pack_bf16(o1[2], o1[3]);
        hi[j >> 1] = pack_bf16(o2[0], o2[1]);
        hi[(j >> 1) + 1] = pack_bf16(o2[2], o2[3]);
      }
      f8_route_store(r, 1, N, hc + c, row_base, M, stage, lo, 4);
      f8_route_store(r, 1, N, hc + c + 64, row_base, M, stage, hi, 4);
    }
    return;
  }
#pragma unroll
  for (int c = 0; c < 128; c += 32) {
    const int col0 = hc + c;
    if (col0 >= N) break;
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      float a0 = __uint_as_float(v[c + j]), a1 = __uint_as_float(v[c + j + 1]);
      if (p.bias) {
        a0 += __ldg(p.bias + col0 + j);
        a1 += __ldg(p.bias + col0 + j + 1);
      }
      packed[j >> 1] = pack_bf16(a0, a1);
    }
    const int ngroups = min(4, (N - col0) >> 3);
#pragma unroll 1
    for (int pl = 0; pl < r.planes; ++pl)
      f8_route_store(r, pl, N, col0, row_base, M, stage, packed, ngroups);
  }
}

__device__ __forceinline__ void f8_tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  constexpr int group = 16;  // n-blocks per raster band: one band's weights stay in L2
  const int band_size = group * num_m;
  const int band = tile / band_size;
  const int in_band = tile - band * band_size;
  const int n0 = band * group;
  const int gn = min(group, num_n - n0);
  mb = in_band / gn;
  nb = n0 + (in_band - mb * gn);
}

template <int EPI>
__device__ __forceinline__ void f8_epilogue(const Fp8Params& p, const uint32_t* v, int ew, int row,
                                            bool row_ok, int nb, int M, int N, uint4* stage) {
  const int col0 = nb * F8_BN + ew * 128;
  if constexpr (EPI == F8_ROUTE) {
    if (col0 < N) f8_route_epilogue(p, v, col0, row, N, M, stage);   // col0: warp-uniform
    return;
  }
  if constexpr (EPI == F8_STORE_F32) {
    // bf16 partial products, no bias, each row to its owner (the reduce-scatter of a
    // row-parallel GEMM), staged so each store writes 8 rows x 64 contiguous bytes
    const int lane = lane_id();
    const int row_base = row - lane;
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      if (col0 + c >= N) break;   // warp-uniform
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        packed[j] = pack_bf16(__uint_as_float(v[c + 2 * j]), __uint_as_float(v[c + 2 * j + 1]));
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
                                               : p.scatter.row_ptr(p.out, p.ldo, srow)) + col0 + c + 8 * g;
          *reinterpret_cast<uint4*>(d) = stage[rr * 5 + g];
        }
      }
      __syncwarp();
    }
    return;
  }
  if constexpr (EPI == F8_SWIGLU_Q) {
    // this warpgroup's 128 columns: [64 value | 64 gate] -> 64 outputs, one scale per 1x64
    // block (two 32-element scale-factor bytes, written as one 16-bit half of the word)
    if (!row_ok) return;
    float h[64];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      float a = __uint_as_float(v[j]), g = __uint_as_float(v[64 + j]);
      if (p.bias) {
        a += __ldg(p.bias + col0 + j);
        g += __ldg(p.bias + col0 + 64 + j);
      }
      h[j] = a * siluf_(g);
      amax = fmaxf(amax, fabsf(h[j]));
    }
    const int e = e8_exponent(amax);
    const float inv = exp2_int(-e < -126 ? -126 : (-e > 127 ? 127 : -e));
    const int oc = nb * 128 + ew * 64;               // output column of h[0]
    uint8_t* dst = p.q_out + (int64_t)row * p.ldq + oc;
#pragma unroll
    for (int j = 0; j < 64; j += 16) {
      uint32_t w[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint16_t lo = pack_e4m3x2(h[j + 4 * t] * inv, h[j + 4 * t + 1] * inv);
        const uint16_t hi = pack_e4m3x2(h[j + 4 * t + 2] * inv, h[j + 4 * t + 3] * inv);
        w[t] = (uint32_t)lo | ((uint32_t)hi << 16);
      }
      *reinterpret_cast<uint4*>(dst + j) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    const uint16_t b = (uint16_t)((e + 127) & 0xFF);
    const int kb_total = (N / 2) / 32;
    *reinterpret_cast<uint16_t*>(p.q_sf + sf_offset(row, (int64_t)nb * 4 + ew * 2, kb_total)) =
        (uint16_t)(b | (b << 8));
    return;
  }
  if (!row_ok || col0 >= N) return;
#pragma unroll
  for (int c = 0; c < 128; c += 32) {
    if (col0 + c >= N) break;
    float f[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      f[j] = __uint_as_float(v[c + j]);
      if (p.bias) f[j] += __ldg(p.bias + col0 + c + j);
    }
    __nv_bfloat16* orow = p.out + (int64_t)row * p.ldo + col0 + c;
    uint32_t packed[16];
    if constexpr (EPI == F8_RESIDUAL) {
      const __nv_bfloat16* grow = p.gate + (int64_t)p.gate_idx[row] * p.ldg + col0 + c;
      uint4 xr[4], gr[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        xr[q] = reinterpret_cast<const uint4*>(orow)[q];
        gr[q] = reinterpret_cast<const uint4*>(grow)[q];
      }
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(xr);
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(gr);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        packed[j] = pack_bf16(bf16_lo(xw[j]) + f[2 * j] * bf16_lo(gw[j]),
                              bf16_hi(xw[j]) + f[2 * j + 1] * bf16_hi(gw[j]));
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) packed[j] = pack_bf16(f[2 * j], f[2 * j + 1]);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      reinterpret_cast<uint4*>(orow)[q] =
          make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
  }
}

template <int EPI>
__global__ void __launch_bounds__(F8_THREADS, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    Fp8Params p, int M, int N, int K) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + F8_STAGES * F8_STAGE_BYTES);
  uint64_t* empty = full + F8_STAGES;
  uint64_t* tfull = empty + F8_STAGES;
  uint64_t* tempty = tfull + 1;
  uint64_t* mma_done = tempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint4* route_stage = reinterpret_cast<uint4*>(smem + F8_STAGES * F8_STAGE_BYTES + 2048);

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (M + F8_BM - 1) / F8_BM;
  const int num_n = (N + F8_BN - 1) / F8_BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = K / F8_BK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < F8_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 256);
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
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    setmaxnreg_dec<F8_REGS_LOW>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------------ producer
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, issued_par = 0;
      long long t_empty = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        f8_tile_coords(tile, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          const long long tw = p.trace ? clock64() : 0;
          if (!mbar_wait_sleep(&empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          if (p.trace) t_empty += clock64() - tw;
          uint8_t* sA = smem + stage * F8_STAGE_BYTES;
          uint8_t* sB = sA + F8_A_BYTES;
          uint8_t* sSFA = sB + F8_B_BYTES;
          uint8_t* sSFB = sSFA + F8_SFA_BYTES;
          mbar_arrive_expect_tx(&full[stage], F8_A_BYTES + F8_B_BYTES + F8_SFA_BYTES + F8_SFB_BYTES);
          tma_load_2d(sA, &tmA, &full[stage], kb * F8_BK, mb * F8_BM);
          tma_load_2d(sB, &tmB, &full[stage], kb * F8_BK, nb * F8_BN);
          bulk_load(sSFA, p.sfa + ((int64_t)mb * num_kb + kb) * F8_SFA_BYTES, F8_SFA_BYTES, &full[stage]);
          bulk_load(sSFB, p.sfb + ((int64_t)nb * num_kb + kb) * F8_SFB_BYTES, F8_SFB_BYTES, &full[stage]);
          issued_mask |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == F8_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (p.trace) p.trace[blockIdx.x * 8 + 3] = t_empty;
      if (!ok) {
        for (int s = 0; s < F8_STAGES; ++s) {
          if (!(issued_mask >> s & 1)) continue;
          const uint32_t par = (issued_par >> s) & 1;
          long long t0 = clock64();
          while (!mbar_try_wait(&full[s], par) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      const long long t_start = p.trace ? clock64() : 0;
      long long t_full = 0, t_acc = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const long long ta = p.trace ? clock64() : 0;
        if (!mbar_wait_sleep(tempty, (local & 1) ^ 1, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        if (p.trace) t_acc += clock64() - ta;
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          const long long tf = p.trace ? clock64() : 0;
          if (!mbar_wait_sleep(&full[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          if (p.trace) t_full += clock64() - tf;
          tc_fence_after();
          const uint32_t aA = smem_u32(smem + stage * F8_STAGE_BYTES);
          const uint32_t aB = aA + F8_A_BYTES;
          const uint32_t aSFA = aB + F8_B_BYTES;
          const uint32_t aSFB = aSFA + F8_SFA_BYTES;
          const uint32_t sfa_col = tmem + F8_SF_COL + stage * F8_SF_STAGE_COLS;
          const uint32_t sfb_col = sfa_col + 4;
          tmem_cp_32x128b_warpx4(sfa_col, umma_desc_interleave_rows16(aSFA));
          tmem_cp_32x128b_warpx4(sfb_col, umma_desc_interleave_rows16(aSFB));
          tmem_cp_32x128b_warpx4(sfb_col + 4, umma_desc_interleave_rows16(aSFB + 512));
#pragma unroll
          for (int k = 0; k < F8_BK / 32; ++k) {
            umma_mxf8_ss(tmem, umma_desc_kmajor_sw128(aA + k * 32), umma_desc_kmajor_sw128(aB + k * 32),
                         umma_idesc_mxf8(F8_BM, F8_BN, k), sfa_col | ((uint32_t)k << 30),
                         sfb_col | ((uint32_t)k << 30), (kb | k) != 0);
          }
          umma_commit(&empty[stage]);
          if (++stage == F8_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(tfull);
      }
      if (p.trace) {
        p.trace[blockIdx.x * 8 + 0] = clock64() - t_start;
        p.trace[blockIdx.x * 8 + 1] = t_full;
        p.trace[blockIdx.x * 8 + 2] = t_acc;
        p.trace[blockIdx.x * 8 + 4] = local;
      }
      umma_commit(mma_done);
      long long t0 = clock64();
      while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else {
    // ------------------------------------------------------------------- epilogue
    setmaxnreg_inc<F8_REGS_HIGH>();
    const int ew = (warp - 4) >> 2;          // which 128-column half
    const int quarter = warp & 3;
    const int r_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + ew * 128;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int mb, nb;
      f8_tile_coords(tile, num_m, num_n, mb, nb);
      if (!mbar_wait_sleep(tfull, local & 1, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      uint32_t v[128];
#pragma unroll
      for (int c = 0; c < 128; c += 32)
        tmem_ld32(lane_base + c, *reinterpret_cast<uint32_t(*)[32]>(v + c));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(tempty);   // the accumulator is free for the next tile's MMAs
      const int row = mb * F8_BM + r_in_tile;
      f8_epilogue<EPI>(p, v, ew, row, row < M, nb, M, N, route_stage + (warp - 4) * kF8StageWords);
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int EPI>
static void launch_fp8(const GemmFp8Args& a, Fp8Params p, cudaStream_t stream) {
  p.trace = g_fp8_trace;
  static std::atomic<uint64_t> attr_set{0};
  if (attr_needed(attr_set)) {
    cudaFuncSetAttribute(gemm_fp8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, F8_SMEM);
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, gemm_fp8_kernel<EPI>) != cudaSuccess ||
        fa.numRegs * F8_THREADS < 128 * F8_REGS_LOW + 256 * F8_REGS_HIGH)
      throw std::runtime_error("fp8 GEMM: launch registers cannot fund the register split");
    attr_done(attr_set);
  }
  CUtensorMap ta = make_tmap_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.M, a.lda, F8_BK, F8_BM);
  CUtensorMap tb = make_tmap_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.N, a.ldb, F8_BK, F8_BN);
  const int tiles = ((a.M + F8_BM - 1) / F8_BM) * ((a.N + F8_BN - 1) / F8_BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  gemm_fp8_kernel<EPI><<<grid, F8_THREADS, F8_SMEM, stream>>>(ta, tb, p, a.M, a.N, a.K);
}

void launch_gemm_fp8(const GemmFp8Args& a, int mode, void* out, int64_t ldo, const float* bias,
                     const void* gate, int64_t ldg, const int* gate_idx, void* q_out, int64_t ldq,
                     void* q_sf, int* err, cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return;
  if (a.K % F8_BK) throw std::runtime_error("fp8 GEMM: K must be a multiple of 128");
  Fp8Params p{};
  p.sfa = reinterpret_cast<const uint8_t*>(a.sfa);
  p.sfb = reinterpret_cast<const uint8_t*>(a.sfb);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.bias = bias;
  p.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  p.ldg = ldg;
  p.gate_idx = gate_idx;
  p.q_out = reinterpret_cast<uint8_t*>(q_out);
  p.ldq = ldq;
  p.q_sf = reinterpret_cast<uint8_t*>(q_sf);
  p.err = err;
  switch (mode) {
    case F8_STORE: launch_fp8<F8_STORE>(a, p, stream); break;
    case F8_RESIDUAL: launch_fp8<F8_RESIDUAL>(a, p, stream); break;
    case F8_SWIGLU_Q: launch_fp8<F8_SWIGLU_Q>(a, p, stream); break;
    default: throw std::runtime_error("unknown fp8 GEMM epilogue mode");
  }
}

void launch_gemm_fp8_f32_scatter(const GemmFp8Args& a, void* out, int64_t ldo, const RowScatter& sc,
                                 int* err, cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return;
  if (a.K % F8_BK) throw std::runtime_error("fp8 GEMM: K must be a multiple of 128");
  Fp8Params p{};
  p.sfa = reinterpret_cast<const uint8_t*>(a.sfa);
  p.sfb = reinterpret_cast<const uint8_t*>(a.sfb);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.scatter = sc;
  p.err = err;
  launch_fp8<F8_STORE_F32>(a, p, stream);
}

void launch_gemm_fp8_routed(const GemmFp8Args& a, const GemmRoute& r, const float* bias, int* err,
                            cudaStream_t stream) {
  if (a.M == 0 || a.N == 0) return;
  if (a.K % F8_BK) throw std::runtime_error("fp8 GEMM: K must be a multiple of 128");
  if (r.planes < 1 || r.planes > 8) throw std::runtime_error("routed GEMM: 1..8 route planes");
  Fp8Params p{};
  p.sfa = reinterpret_cast<const uint8_t*>(a.sfa);
  p.sfb = reinterpret_cast<const uint8_t*>(a.sfb);
  p.bias = bias;
  p.route = r;
  p.err = err;
  launch_fp8<F8_ROUTE>(a, p, stream);
}

// ------------------------------------------------------------------ activation quantiser
// One warp per row; each half-warp owns a 1x128 block (16 lanes x 8 elements): block
// amax by shuffles, one power-of-two scale, E4M3 bytes and the scale-factor word.
__global__ void __launch_bounds__(256) quant_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                         int64_t ldx, int M, int K,
                                                         uint8_t* __restrict__ q, int64_t ldq,
                                                         uint8_t* __restrict__ sf) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int kb32_total = K / 32;
  const int nvec = K / 8;
  for (int base = 0; base < nvec; base += 32) {   // K % 128 == 0: half-warps are whole blocks
    const int c = base + lane;
    const bool valid = c < nvec;
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (valid) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + (int64_t)row * ldx + c * 8);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f[2 * j] = bf16_lo(w[j]);
        f[2 * j + 1] = bf16_hi(w[j]);
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (!valid) continue;
    const int e = e8_exponent(amax);
    const float inv = exp2_int(-e < -126 ? -126 : (-e > 127 ? 127 : -e));
    uint32_t lo = (uint32_t)pack_e4m3x2(f[0] * inv, f[1] * inv) |
                  ((uint32_t)pack_e4m3x2(f[2] * inv, f[3] * inv) << 16);
    uint32_t hi = (uint32_t)pack_e4m3x2(f[4] * inv, f[5] * inv) |
                  ((uint32_t)pack_e4m3x2(f[6] * inv, f[7] * inv) << 16);
    *reinterpret_cast<uint2*>(q + (int64_t)row * ldq + c * 8) = make_uint2(lo, hi);
    if ((lane & 15) == 0) {
      const uint32_t b = (uint32_t)(e + 127) & 0xFF;
      *reinterpret_cast<uint32_t*>(sf + sf_offset(row, (int64_t)(c / 16) * 4, kb32_total)) =
          b | (b << 8) | (b << 16) | (b << 24);
    }
  }
}

void launch_quant_rows(const void* x, int64_t ldx, int M, int K, void* q, int64_t ldq, void* sf,
                       cudaStream_t stream) {
  if (M == 0) return;
  if (K % 128) throw std::runtime_error("fp8 quantiser: K must be a multiple of 128");
  quant_rows_kernel<<<(M + 7) / 8, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, K, reinterpret_cast<uint8_t*>(q), ldq,
      reinterpret_cast<uint8_t*>(sf));
}

}  // namespace vdn
