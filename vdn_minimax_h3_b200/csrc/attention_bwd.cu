// Window softmax attention, training backward, on the 5th-generation tensor cores (sm_100a).
//
// Two kernels over the same analytic plans as the forward (no mask tensor, no gather):
//
//   attn_bwd_dq_kernel   one CTA per (head, 128 query rows); walks the forward plan's K/V
//                        ranges. Per 128-key block: S = Q K^T and dP = dO V^T (tcgen05,
//                        both into TMEM), P = 2^(S*c - lse) and dS = P (dP - delta) in
//                        registers (thread = query row), dS written back over S in TMEM as
//                        bf16 and dQ += dS K accumulated in TMEM (A operand from TMEM).
//                        delta = rowsum(dO * O) is computed here and stored for the other
//                        kernel.
//   attn_bwd_dkv_kernel  one CTA per (head, 128 key rows); walks the TRANSPOSED plan (for a
//                        K/V tile, the <= 4 contiguous query ranges that attend to it). Per
//                        128-query block: S^T = K Q^T, dP^T = V dO^T, P^T and dS^T in
//                        registers (thread = key row), then dV += P^T dO and dK += dS^T Q,
//                        both accumulated in TMEM (P^T / dS^T as the TMEM A operand).
//
// Scores are the forward's: S = q.k, p = 2^(S * scale * log2 e - lse2) with lse2 the
// forward's per-row log2-sum-exp; dS is the gradient of the raw score, so dQ and dK carry
// the softmax scale once, at the end. Q, K, V, dO tiles arrive by TMA (128-byte swizzle,
// no multicast); every wait is bounded and a protocol failure unwinds, records an error
// code, drains its copies and frees TMEM (common.cuh).
//
// Reference parity: the training backward of the window softmax, which the reference takes
// from autograd of flex_attention (src/models/softmax_attention/flex_attention.py:86-90,
// compiled backward) and of SDPA for the dense teacher.
#include "common.cuh"
#include "launchers.h"
#include "tma.cuh"

#include <stdexcept>

namespace vdn {

namespace {

constexpr int BW_ROWS = 128;                       // query rows (dq) / key rows (dkv) per CTA
constexpr int BW_BLK = 128;                        // walked block (keys for dq, queries for dkv)
constexpr int BW_D = 128;
constexpr int BW_TILE_BYTES = BW_ROWS * BW_D * 2;  // 32 KB: two 64-column swizzled atoms
constexpr int BW_STAGES = 2;
constexpr int BW_THREADS = 256;                    // warp 0 TMA, warp 1 MMA, warps 4-7 compute
constexpr int BW_RANGES = 4;
constexpr int BW_SMEM = 2 * BW_TILE_BYTES + BW_STAGES * 2 * BW_TILE_BYTES +
                        BW_STAGES * 2 * BW_BLK * 4 + 1024 + 256;

struct RangeWalk {
  int a[BW_RANGES], b[BW_RANGES];
  int range, pos, end;
  __device__ void init(const int* row) {
#pragma unroll
    for (int i = 0; i < BW_RANGES; ++i) {
      a[i] = row[2 * i];
      b[i] = row[2 * i + 1];
    }
    range = 0;
    pos = a[0];
    end = b[0];
    skip();
  }
  __device__ void select(int rg) {
#pragma unroll
    for (int i = 0; i < BW_RANGES; ++i)
      if (i == rg) {
        pos = a[i];
        end = b[i];
      }
  }
  __device__ void skip() {
    while (range < BW_RANGES && pos >= end) {
      ++range;
      if (range < BW_RANGES) select(range);
    }
  }
  __device__ bool done() const { return range >= BW_RANGES; }
  __device__ int valid() const { return min(BW_BLK, end - pos); }
  __device__ void next() {
    pos += BW_BLK;
    skip();
  }
};

__device__ __forceinline__ int count_blocks(const int* row) {
  int n = 0;
#pragma unroll
  for (int i = 0; i < BW_RANGES; ++i) {
    const int len = row[2 * i + 1] - row[2 * i];
    n += len > 0 ? (len + BW_BLK - 1) / BW_BLK : 0;
  }
  return n;
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* tm, uint64_t* bar,
                                          int head, int row) {
  tma_load_2d(dst, tm, bar, head * BW_D, row);
  tma_load_2d(dst + BW_TILE_BYTES / 2, tm, bar, head * BW_D + 64, row);
}

struct BwdParams {
  const int* tiles;        // [n, 4] (start, end, segment, -) of the CTA's own rows
  const int* ranges;       // [n_seg, 8] walked (start, end) ranges
  int H, T;
  const float* lse;        // [H, T] log2-domain log-sum-exp of the forward rows
  float* delta;            // [H, T] rowsum(dO * O): written by dq, read by dkv
  const __nv_bfloat16* o;  // forward output (ungated), row stride ldo
  int64_t ldo;
  const __nv_bfloat16* dout;
  int64_t lddo;
  __nv_bfloat16* dq;       // dq kernel output, row stride ldq
  int64_t ldq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t ldk, ldv;
  float scale_log2, scale;
  int* err;
};

// Bounded drain of the TMA copies a producer may still have in flight (abort path).
__device__ __forceinline__ void drain(uint64_t* bar, int phase) {
  if (phase < 0) return;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, (uint32_t)phase) && clock64() - t0 < kWaitBudgetCycles) {
  }
}

}  // namespace

// ---------------------------------------------------------------------------------- dq
__global__ void __launch_bounds__(BW_THREADS, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + BW_TILE_BYTES;
  uint8_t* sK = sDO + BW_TILE_BYTES;                    // [stage][32 KB]
  uint8_t* sV = sK + BW_STAGES * BW_TILE_BYTES;         // [stage][32 KB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + BW_STAGES * BW_TILE_BYTES + BW_STAGES * 2 * BW_BLK * 4);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                // [stage]
  uint64_t* kv_empty = kv_full + BW_STAGES;    // [stage]
  uint64_t* sd_full = kv_empty + BW_STAGES;    // S and dP of the block are in TMEM
  uint64_t* ds_full = sd_full + 1;             // dS (bf16) is in TMEM
  uint64_t* dq_done = ds_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dq_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int head = blockIdx.x % p.H;
  const int* t = p.tiles + 4 * (blockIdx.x / p.H);
  const int* rg = p.ranges + 8 * t[2];
  const int q0 = t[0];

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < BW_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(sd_full, 1);
    mbar_init(ds_full, 128);
    mbar_init(dq_done, 1);
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
  const uint32_t tmem = *tmem_slot;     // S at 0, dP at 128, dQ at 256
  const int nblk = count_blocks(rg);

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int last[BW_STAGES] = {-1, -1};
      mbar_arrive_expect_tx(q_full, 2 * BW_TILE_BYTES);
      load_tile(sQ, &tmQ, q_full, head, q0);
      load_tile(sDO, &tmDO, q_full, head, q0);
      RangeWalk w;
      w.init(rg);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (; !w.done(); w.next()) {
        if (!mbar_wait(&kv_empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        last[stage] = (int)phase;
        mbar_arrive_expect_tx(&kv_full[stage], 2 * BW_TILE_BYTES);
        load_tile(sK + stage * BW_TILE_BYTES, &tmK, &kv_full[stage], head, w.pos);
        load_tile(sV + stage * BW_TILE_BYTES, &tmV, &kv_full[stage], head, w.pos);
        if (++stage == BW_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok || *abort_flag) {
        drain(q_full, 0);
        for (int s = 0; s < BW_STAGES; ++s) drain(&kv_full[s], last[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(BW_ROWS, BW_BLK, false, false);
      constexpr uint32_t idesc_q = umma_idesc_bf16(BW_ROWS, BW_D, false, true);
      auto kdesc = [](const uint8_t* base, int k) {
        return umma_desc_kmajor_sw128(smem_u32(base) + (k >> 2) * (BW_TILE_BYTES / 2) + (k & 3) * 32);
      };
      auto mndesc = [](const uint8_t* base, int k) {
        return umma_desc_mnmajor_sw128(smem_u32(base) + k * 2048, BW_TILE_BYTES / 2);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err, kErrTimeoutMma);
      if (ok) tc_fence_after();
      int stage = 0;
      uint32_t phase = 0;
      for (int j = 0; j < nblk && ok; ++j) {
        if (!mbar_wait(&kv_full[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* k = sK + stage * BW_TILE_BYTES;
        const uint8_t* v = sV + stage * BW_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BW_D / 16; ++kk)
          umma_f16_ss(tmem, kdesc(sQ, kk), kdesc(k, kk), idesc_s, kk != 0);
#pragma unroll
        for (int kk = 0; kk < BW_D / 16; ++kk)
          umma_f16_ss(tmem + 128, kdesc(sDO, kk), kdesc(v, kk), idesc_s, kk != 0);
        umma_commit(sd_full);
        if (!mbar_wait(ds_full, j & 1, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // dQ += dS K: A = dS (bf16 pairs over TMEM columns 0-63), B = K as [keys, d] (MN-major)
#pragma unroll
        for (int kk = 0; kk < BW_BLK / 16; ++kk)
          umma_f16_ts(tmem + 256, tmem + kk * 8, mndesc(k, kk), idesc_q, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kv_empty[stage]);
        if (++stage == BW_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      umma_commit(dq_done);
      drain(dq_done, 0);
    }
  } else if (warp >= 4) {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int row = q0 + r;
    const bool row_ok = row < t[1];
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off, tP = tmem + lane_off + 128, tQ = tmem + lane_off + 256;
    // delta = rowsum(dO * O) and the forward's log2-sum-exp for this row
    float delta = 0.f, lse2 = 0.f;
    if (row < p.T) {
      const uint4* o4 = reinterpret_cast<const uint4*>(p.o + (int64_t)row * p.ldo + head * BW_D);
      const uint4* g4 = reinterpret_cast<const uint4*>(p.dout + (int64_t)row * p.lddo + head * BW_D);
#pragma unroll 4
      for (int c = 0; c < BW_D / 8; ++c) {
        const uint4 a = o4[c], b = g4[c];
        const uint32_t* ua = reinterpret_cast<const uint32_t*>(&a);
        const uint32_t* ub = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
        for (int i = 0; i < 4; ++i) delta += bf16_lo(ua[i]) * bf16_lo(ub[i]) + bf16_hi(ua[i]) * bf16_hi(ub[i]);
      }
      lse2 = p.lse[(int64_t)head * p.T + row];
      if (row_ok) p.delta[(int64_t)head * p.T + row] = delta;
    }
    RangeWalk w;
    w.init(rg);
    bool ok = true;
    for (int j = 0; j < nblk; ++j, w.next()) {
      if (!mbar_wait(sd_full, j & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int valid = w.valid();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t s[64], dp[64];
        tmem_ld32(tS + h * 64, *reinterpret_cast<uint32_t(*)[32]>(s));
        tmem_ld32(tS + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
        tmem_ld32(tP + h * 64, *reinterpret_cast<uint32_t(*)[32]>(dp));
        tmem_ld32(tP + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(dp + 32));
        tmem_wait_ld();
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float d2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 2 * i + e;
            const float pr = (h * 64 + c < valid)
                                 ? ex2f(fmaf(__uint_as_float(s[c]), p.scale_log2, -lse2))
                                 : 0.f;
            d2[e] = pr * (__uint_as_float(dp[c]) - delta);
          }
          pk[i] = pack_bf16(d2[0], d2[1]);
        }
        tmem_st32(tS + h * 32, pk);     // dS over S columns already read
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_full);
    }
    if (ok && mbar_wait(dq_done, 0, abort_flag, p.err, kErrTimeoutSoftmax)) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BW_D; c += 32) {
        uint32_t u[32];
        tmem_ld32(tQ + c, u);
        tmem_wait_ld();
        if (row_ok) {
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            o[i] = pack_bf16(__uint_as_float(u[2 * i]) * p.scale, __uint_as_float(u[2 * i + 1]) * p.scale);
          uint4* dst = reinterpret_cast<uint4*>(p.dq + (int64_t)row * p.ldq + head * BW_D + c);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// --------------------------------------------------------------------------------- dkv
__global__ void __launch_bounds__(BW_THREADS, 1)
    attn_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + BW_TILE_BYTES;
  uint8_t* sQ = sV + BW_TILE_BYTES;                     // [stage][32 KB]
  uint8_t* sDO = sQ + BW_STAGES * BW_TILE_BYTES;        // [stage][32 KB]
  float* sStat = reinterpret_cast<float*>(sDO + BW_STAGES * BW_TILE_BYTES);   // [stage][lse 128 | delta 128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStat + BW_STAGES * 2 * BW_BLK);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;                 // [stage]
  uint64_t* q_empty = q_full + BW_STAGES;      // [stage]
  uint64_t* sd_full = q_empty + BW_STAGES;     // S^T and dP^T in TMEM
  uint64_t* pds_full = sd_full + 1;            // P^T and dS^T (bf16) in TMEM
  uint64_t* kv_done = pds_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int head = blockIdx.x % p.H;
  const int* t = p.tiles + 4 * (blockIdx.x / p.H);
  const int* rg = p.ranges + 8 * t[2];
  const int k0 = t[0];

  if (warp == 0 && lane == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < BW_STAGES; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(sd_full, 1);
    mbar_init(pds_full, 128);
    mbar_init(kv_done, 1);
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
  const uint32_t tmem = *tmem_slot;     // S^T at 0, dP^T at 128, dV at 256, dK at 384
  const int nblk = count_blocks(rg);

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      int last[BW_STAGES] = {-1, -1};
      mbar_arrive_expect_tx(kv_full, 2 * BW_TILE_BYTES);
      load_tile(sK, &tmK, kv_full, head, k0);
      load_tile(sV, &tmV, kv_full, head, k0);
      RangeWalk w;
      w.init(rg);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (; !w.done(); w.next()) {
        if (!mbar_wait(&q_empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        last[stage] = (int)phase;
        mbar_arrive_expect_tx(&q_full[stage], 2 * BW_TILE_BYTES);
        load_tile(sQ + stage * BW_TILE_BYTES, &tmQ, &q_full[stage], head, w.pos);
        load_tile(sDO + stage * BW_TILE_BYTES, &tmDO, &q_full[stage], head, w.pos);
        if (++stage == BW_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok || *abort_flag) {
        drain(kv_full, 0);
        for (int s = 0; s < BW_STAGES; ++s) drain(&q_full[s], last[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(BW_ROWS, BW_BLK, false, false);
      constexpr uint32_t idesc_g = umma_idesc_bf16(BW_ROWS, BW_D, false, true);
      auto kdesc = [](const uint8_t* base, int k) {
        return umma_desc_kmajor_sw128(smem_u32(base) + (k >> 2) * (BW_TILE_BYTES / 2) + (k & 3) * 32);
      };
      auto mndesc = [](const uint8_t* base, int k) {
        return umma_desc_mnmajor_sw128(smem_u32(base) + k * 2048, BW_TILE_BYTES / 2);
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, p.err, kErrTimeoutMma);
      if (ok) tc_fence_after();
      int stage = 0;
      uint32_t phase = 0;
      for (int j = 0; j < nblk && ok; ++j) {
        if (!mbar_wait(&q_full[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* q = sQ + stage * BW_TILE_BYTES;
        const uint8_t* g = sDO + stage * BW_TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BW_D / 16; ++kk)
          umma_f16_ss(tmem, kdesc(sK, kk), kdesc(q, kk), idesc_s, kk != 0);
#pragma unroll
        for (int kk = 0; kk < BW_D / 16; ++kk)
          umma_f16_ss(tmem + 128, kdesc(sV, kk), kdesc(g, kk), idesc_s, kk != 0);
        umma_commit(sd_full);
        if (!mbar_wait(pds_full, j & 1, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // dV += P^T dO and dK += dS^T Q: A from TMEM (P^T at 0, dS^T at 128), B = dO / Q as
        // [queries, d] (MN-major)
#pragma unroll
        for (int kk = 0; kk < BW_BLK / 16; ++kk)
          umma_f16_ts(tmem + 256, tmem + kk * 8, mndesc(g, kk), idesc_g, (j > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < BW_BLK / 16; ++kk)
          umma_f16_ts(tmem + 384, tmem + 128 + kk * 8, mndesc(q, kk), idesc_g, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&q_empty[stage]);
        if (++stage == BW_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      umma_commit(kv_done);
      drain(kv_done, 0);
    }
  } else if (warp >= 4) {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;          // key row within the tile
    const int krow = k0 + r;
    const bool row_ok = krow < t[1];
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off, tP = tmem + lane_off + 128;
    RangeWalk w;
    w.init(rg);
    bool ok = true;
    for (int j = 0; j < nblk; ++j, w.next()) {
      // this block's per-query statistics into shared memory (thread r loads query r)
      float* st = sStat + (j & 1) * 2 * BW_BLK;
      const int valid = w.valid();
      const int qr = w.pos + r;
      st[r] = r < valid ? p.lse[(int64_t)head * p.T + qr] : 0.f;
      st[BW_BLK + r] = r < valid ? p.delta[(int64_t)head * p.T + qr] : 0.f;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (!mbar_wait(sd_full, j & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t s[64], dp[64];
        tmem_ld32(tS + h * 64, *reinterpret_cast<uint32_t(*)[32]>(s));
        tmem_ld32(tS + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
        tmem_ld32(tP + h * 64, *reinterpret_cast<uint32_t(*)[32]>(dp));
        tmem_ld32(tP + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(dp + 32));
        tmem_wait_ld();
        uint32_t pp[32], pd[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float pr[2], d2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = h * 64 + 2 * i + e;
            pr[e] = c < valid ? ex2f(fmaf(__uint_as_float(s[2 * i + e]), p.scale_log2, -st[c])) : 0.f;
            d2[e] = pr[e] * (__uint_as_float(dp[2 * i + e]) - st[BW_BLK + c]);
          }
          pp[i] = pack_bf16(pr[0], pr[1]);
          pd[i] = pack_bf16(d2[0], d2[1]);
        }
        tmem_st32(tS + h * 32, pp);     // P^T over S^T columns already read
        tmem_st32(tP + h * 32, pd);     // dS^T over dP^T columns already read
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(pds_full);
    }
    if (ok && mbar_wait(kv_done, 0, abort_flag, p.err, kErrTimeoutSoftmax)) {
      tc_fence_after();
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const uint32_t src = tmem + lane_off + 256 + which * 128;
        __nv_bfloat16* base = which == 0 ? p.dv : p.dk;
        const int64_t ld = which == 0 ? p.ldv : p.ldk;
        const float mul = which == 0 ? 1.f : p.scale;
#pragma unroll 1
        for (int c = 0; c < BW_D; c += 32) {
          uint32_t u[32];
          tmem_ld32(src + c, u);
          tmem_wait_ld();
          if (row_ok) {
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              o[i] = pack_bf16(__uint_as_float(u[2 * i]) * mul, __uint_as_float(u[2 * i + 1]) * mul);
            uint4* dst = reinterpret_cast<uint4*>(base + (int64_t)krow * ld + head * BW_D + c);
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

void launch_attention_bwd(const AttnBwdArgs& a, cudaStream_t stream) {
  static std::atomic<uint64_t> attr{0};
  if (attr_needed(attr)) {
    cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM);
    cudaFuncSetAttribute(attn_bwd_dkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM);
    attr_done(attr);
  }
  const uint64_t cols = (uint64_t)a.H * BW_D;
  auto tmap = [&](const void* ptr, int64_t ld) {
    return make_tmap_2d(ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, a.T, ld * 2, 64, BW_ROWS);
  };
  const CUtensorMap tq = tmap(a.q, a.ldq), tk = tmap(a.k, a.ldk), tv = tmap(a.v, a.ldv),
                    tdo = tmap(a.dout, a.lddo);
  BwdParams p{};
  p.H = a.H;
  p.T = a.T;
  p.lse = a.lse;
  p.delta = a.delta;
  p.o = reinterpret_cast<const __nv_bfloat16*>(a.o);
  p.ldo = a.ldo;
  p.dout = reinterpret_cast<const __nv_bfloat16*>(a.dout);
  p.lddo = a.lddo;
  p.dq = reinterpret_cast<__nv_bfloat16*>(a.dq);
  p.ldq = a.lddq;
  p.dk = reinterpret_cast<__nv_bfloat16*>(a.dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(a.dv);
  p.ldk = a.lddk;
  p.ldv = a.lddv;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.scale = a.scale;
  p.err = a.err;
  if (a.n_q_tiles > 0) {
    p.tiles = a.q_tiles;
    p.ranges = a.kv_ranges;
    attn_bwd_dq_kernel<<<a.n_q_tiles * a.H, BW_THREADS, BW_SMEM, stream>>>(tq, tk, tv, tdo, p);
  }
  if (a.n_k_tiles > 0) {
    p.tiles = a.k_tiles;
    p.ranges = a.q_ranges;
    attn_bwd_dkv_kernel<<<a.n_k_tiles * a.H, BW_THREADS, BW_SMEM, stream>>>(tq, tk, tv, tdo, p);
  }
}

}  // namespace vdn
