// Window softmax attention on the 5th-generation tensor cores (sm_100a).
//
// One work item = (head, 256 query rows) of one plan segment, processed as TWO 128-row
// tiles that share every K/V block. The segment's kept K/V rows are at most four CONTIGUOUS
// row ranges of the packed sequence (globals, the window frames, the anchor frames;
// models/window.py: AttentionPlan); the kernel walks them in 128-key blocks straight out of
// the [T, H, d] projections -- no gather, no mask tensor; only the ragged tail of a range
// is masked.
//
// Roles (384 threads = 3 warpgroups, one CTA per SM, persistent over head-major work items
// so the CTAs in flight share one head's K/V in L2):
//   warp 0      TMA producer: both Q tiles once per item and K blocks into a 3-stage ring
//   warp 2      TMA producer: V blocks into a 2-stage ring (a warp of its own: two
//               producers in one warp serialise their barrier waits)
//   warp 1      MMA issuer (one thread): per block j and tile t, first O_t += P_t V for
//               block j-1 with P read from TMEM (tcgen05.mma with the A operand in TMEM),
//               then S_t = Q_t K_j^T (kind::f16, M=128, N=128) into the same TMEM columns;
//               MMAs execute in issue order, so the S write follows the P read.
//   warp 3      idle (completes warpgroup 0, whose registers go to the softmax)
//   warps 4-7   softmax of tile 0, warps 8-11 softmax of tile 1 (thread = query row): S row
//               from TMEM into registers, online softmax in the exp2 domain with a lazy
//               rescale (O in TMEM is rescaled only when the running max grows by more
//               than 2^8), P written back as packed bf16 over S in TMEM, epilogue
//               O / l * sigmoid(gate). While one tile's softmax runs, the tensor core works
//               on the other tile. Keeping P out of shared memory leaves the shared-memory
//               bandwidth to the Q, K and V operand reads. Optionally a fraction of the
//               exponentials run as a cubic polynomial on the FMA pipe (2^x = 2^n * p(f),
//               Cody-Waite split, p fitted for minimax relative error 8.6e-5 on [0,1)).
// TMEM (512 columns): S[tile] (and P over its first 64 columns) at 128 * tile, O[tile] at
// 256 + 128 * tile.
//
// Every wait is bounded; a protocol failure unwinds, drains and frees TMEM (common.cuh).
// Reference parity: the window softmax of src/models/softmax_attention/ (decomposed.py's
// dense leg + varlen leg, flex_attention.py) and the softmax gate (kernels.py:51-67).
#include "common.cuh"
#include "launchers.h"
#include "tma.cuh"

#include <stdexcept>

namespace vdn {

constexpr int AT_BM = 128;                         // query rows per tile (2 tiles per item)
constexpr int AT_BN = 128;                         // keys per block
constexpr int AT_D = 128;                          // head dim
constexpr int AT_KSTAGES = 3;                      // K ring
constexpr int AT_VSTAGES = 2;                      // V ring
constexpr int AT_Q_BYTES = AT_BM * AT_D * 2;       // 32 KB per Q tile (2 atoms of 16 KB)
constexpr int AT_KV_BYTES = AT_BN * AT_D * 2;      // 32 KB per K or V block (2 atoms of 16 KB)
constexpr int AT_P_BYTES = AT_BM * AT_BN * 2;      // 32 KB per P tile (2 atom columns)
constexpr int AT_THREADS = 384;
// Register split after launch (384 threads x 168): warpgroup 0 (producer, MMA, two idle
// warps) drops to 80, the two softmax warpgroups rise to 208: 128*80 + 256*208 <= 384*168.
constexpr int AT_REGS_LOW = 80;
constexpr int AT_REGS_HIGH = 208;
static_assert(128 * AT_REGS_LOW + 256 * AT_REGS_HIGH <= AT_THREADS * 168, "register split");
constexpr int AT_SMEM = 2 * AT_Q_BYTES + (AT_KSTAGES + AT_VSTAGES) * AT_KV_BYTES + 1024 + 384;
constexpr int AT_MAX_RANGES = 4;
// Kernel variants (attention_set_variant), for A/B runs of the softmax's exponential pass:
//   0  the scalar pass (one FFMA, one MUFU ex2 and one FADD per score, cvt pairs)
//   1  packed pass: scale-and-subtract and the row-sum adds on fma/add.f32x2 (two lanes per
//      issue slot), MUFU ex2 for every score
//   2, 3, 4  the packed pass with 1, 2 or 3 of every 8 score pairs exponentiated by the
//      cubic polynomial on the FMA / integer pipes instead of MUFU (2/16, 4/16, 6/16 of
//      the scores), trading MUFU cycles (16 per clock per SM) for FMA issue slots
//   5, 6, 7  timing diagnostics (wrong results): the packed pass without the MUFU ex2, without
//      the bf16 pack conversion, or without the P store to TMEM
constexpr int AT_VARIANTS = 8;
static int g_variant = 1;

struct AttnParams {
  const int* tiles;          // [n_items_per_head, 4] (q0, q_end, segment, kv_len), q_end-q0 <= 256
  const int* kv;             // [n_seg, 8] (start, end) x 4
  int n_tiles, H, T;
  const __nv_bfloat16* gate; // [T, ldg] logits per head, or null
  int64_t ldg;
  __nv_bfloat16* out;        // [T, ldo], head h at column h*128
  int64_t ldo;
  RowScatter scatter;        // optional: rows to their Ulysses owners
  long long* trace;          // optional: clock64 stamps of CTA 0's pipeline events
  float* lse;                // optional [H, T]: log2-sum-exp of each row's scores (training)
  float scale_log2;          // softmax scale * log2(e)
  int* err;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA / integer pipes only (no conversion instructions, which share the MUFU
// pipe): n = round(x) by adding and subtracting 1.5 * 2^23, f = x - n in [-0.5, 0.5],
// 2^f by a cubic fitted here for minimax relative error (8.4e-5 on [-0.5, 0.5], Lawson's
// iteratively reweighted least squares), 2^n by adding n to the exponent field read from
// the rounding sum's bits. Valid for x >= -125.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float j = x + 12582912.0f;
  const float n = j - 12582912.0f;
  const float f = x - n;
  const float p = fmaf(fmaf(fmaf(0.0552129932f, f, 0.2427141405f), f, 0.6932621603f), f,
                       0.9999195980f);
  const int ni = __float_as_int(j) - 0x4B400000;
  return __int_as_float(__float_as_int(p) + (ni << 23));
}

// The same polynomial on a pair: n = round(x) through the 1.5 * 2^23 rounding sum, the
// reduction and the cubic on fma/add.f32x2, the exponent add on the integer pipe.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 j = __fadd2_rn(x, make_float2(12582912.0f, 12582912.0f));
  const float2 n = __fadd2_rn(j, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __fadd2_rn(x, make_float2(-n.x, -n.y));
  float2 q = __ffma2_rn(make_float2(0.0552129932f, 0.0552129932f), f,
                        make_float2(0.2427141405f, 0.2427141405f));
  q = __ffma2_rn(q, f, make_float2(0.6932621603f, 0.6932621603f));
  q = __ffma2_rn(q, f, make_float2(0.9999195980f, 0.9999195980f));
  // (bits(j) << 23) == n << 23 modulo 2^32: the magic constant's bits shift out
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(j.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(j.y) << 23)));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Iterates the 128-key blocks of a segment's K/V ranges (at most four). The ranges are
// held in scalars and selected with a switch, so nothing is indexed dynamically (no local
// memory traffic in the per-block loops).
struct KvWalk {
  int a0, b0, a1, b1, a2, b2, a3, b3;
  int range, pos, end;
  __device__ void init(const int* kv_row) {
    a0 = kv_row[0]; b0 = kv_row[1]; a1 = kv_row[2]; b1 = kv_row[3];
    a2 = kv_row[4]; b2 = kv_row[5]; a3 = kv_row[6]; b3 = kv_row[7];
    range = 0;
    pos = a0;
    end = b0;
    skip_empty();
  }
  __device__ void select(int rg) {
    switch (rg) {
      case 0: pos = a0; end = b0; break;
      case 1: pos = a1; end = b1; break;
      case 2: pos = a2; end = b2; break;
      default: pos = a3; end = b3; break;
    }
  }
  __device__ void skip_empty() {
    while (range < AT_MAX_RANGES && pos >= end) {
      ++range;
      if (range < AT_MAX_RANGES) select(range);
    }
  }
  __device__ bool done() const { return range >= AT_MAX_RANGES; }
  __device__ int start() const { return pos; }
  __device__ int valid() const { return min(AT_BN, end - pos); }
  __device__ void next() {
    pos += AT_BN;
    skip_empty();
  }
};

// Pipeline tracing (diagnostics, off unless p.trace is set): CTA 0 records clock64 at
// events of its first AT_TRACE_BLOCKS blocks, slot = (event * 2 + tile) * AT_TRACE_BLOCKS + block.
constexpr int AT_TRACE_BLOCKS = 64;
constexpr int AT_TRACE_SLOTS = 12 * AT_TRACE_BLOCKS;   // + 4 clock-rate stamps
enum AtTraceEvent : int {
  TR_S_WAIT = 0, TR_S_READY, TR_LD_DONE, TR_MAX_DONE, TR_EXP_DONE, TR_P_ARRIVE, TR_EVENTS
};
__device__ __forceinline__ void at_trace(const AttnParams& p, int ev, int tile, uint32_t blk) {
  if (p.trace && blockIdx.x == 0 && blk < (uint32_t)AT_TRACE_BLOCKS)
    p.trace[(ev * 2 + tile) * AT_TRACE_BLOCKS + blk] = clock64();
}

__device__ __forceinline__ void item_coords(const AttnParams& p, int item, int& head, int& tile) {
  head = item / p.n_tiles;
  tile = item - head * p.n_tiles;
}

template <int AT_VARIANT>
__global__ void __launch_bounds__(AT_THREADS, 1)
    window_attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                            const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // [2 tiles][32 KB]
  uint8_t* sK = sQ + 2 * AT_Q_BYTES;                    // [AT_KSTAGES][32 KB]
  uint8_t* sV = sK + AT_KSTAGES * AT_KV_BYTES;          // [AT_VSTAGES][32 KB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + AT_VSTAGES * AT_KV_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;                   // [AT_KSTAGES]
  uint64_t* k_empty = k_full + AT_KSTAGES;       // [AT_KSTAGES]
  uint64_t* v_full = k_empty + AT_KSTAGES;       // [AT_VSTAGES]
  uint64_t* v_empty = v_full + AT_VSTAGES;       // [AT_VSTAGES]
  uint64_t* s_full = v_empty + AT_VSTAGES;       // [tile]
  uint64_t* p_full = s_full + 2;                 // [tile]
  uint64_t* pv_done = p_full + 2;                // [tile]
  uint64_t* o_empty = pv_done + 2;               // [tile]
  uint64_t* mma_done = o_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int n_items = p.n_tiles * p.H;
  constexpr int kIssuers = 1;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, kIssuers);
    for (int s = 0; s < AT_KSTAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], kIssuers);
    }
    for (int s = 0; s < AT_VSTAGES; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], kIssuers);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&pv_done[t], 1);
      mbar_init(&o_empty[t], 128);
    }
    mbar_init(mma_done, kIssuers);
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
  // trace mode: the SM clock rate seen by CTA 0 (globaltimer ns against clock64 cycles)
  const bool clock_probe = p.trace && blockIdx.x == 0 && threadIdx.x == 128;
  if (clock_probe) {
    p.trace[AT_TRACE_SLOTS] = (long long)globaltimer_ns();
    p.trace[AT_TRACE_SLOTS + 1] = clock64();
  }

  // The register re-split sits inside each role's branch, so every role's code is
  // dominated by exactly one limit.
  if (warp < 4) {
  setmaxnreg_dec<AT_REGS_LOW>();
  if (warp == 0) {
    // ------------------------------------------------------ TMA producer: Q + K
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      int last_phase[AT_KSTAGES + 1];
      for (int i = 0; i < AT_KSTAGES + 1; ++i) last_phase[i] = -1;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++local) {
        int head, tile;
        item_coords(p, item, head, tile);
        const int* t = p.tiles + 4 * tile;
        if (!mbar_wait(q_empty, (local & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        last_phase[AT_KSTAGES] = local & 1;
        mbar_arrive_expect_tx(q_full, 2 * AT_Q_BYTES);
#pragma unroll
        for (int qt = 0; qt < 2; ++qt) {
          tma_load_2d(sQ + qt * AT_Q_BYTES, &tmQ, q_full, head * AT_D, t[0] + qt * AT_BM);
          tma_load_2d(sQ + qt * AT_Q_BYTES + AT_Q_BYTES / 2, &tmQ, q_full, head * AT_D + 64,
                      t[0] + qt * AT_BM);
        }
        KvWalk w;
        w.init(p.kv + 8 * t[2]);
        for (; !w.done(); w.next()) {
          if (!mbar_wait(&k_empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* k = sK + stage * AT_KV_BYTES;
          last_phase[stage] = (int)phase;
          mbar_arrive_expect_tx(&k_full[stage], AT_KV_BYTES);
          tma_load_2d(k, &tmK, &k_full[stage], head * AT_D, w.start());
          tma_load_2d(k + AT_KV_BYTES / 2, &tmK, &k_full[stage], head * AT_D + 64, w.start());
          if (++stage == AT_KSTAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok || *abort_flag) {
        long long t0 = clock64();
        for (int i = 0; i < AT_KSTAGES + 1; ++i) {
          uint64_t* bar = i < AT_KSTAGES ? &k_full[i] : q_full;
          if (last_phase[i] < 0) continue;
          while (!mbar_try_wait(bar, (uint32_t)last_phase[i]) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------ TMA producer of V (its own warp, so
    // its waits never serialise with the K producer's)
    if (lane == 0) {
      tma_prefetch_desc(&tmV);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int last_phase[AT_VSTAGES];
      for (int i = 0; i < AT_VSTAGES; ++i) last_phase[i] = -1;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        int head, tile;
        item_coords(p, item, head, tile);
        const int* t = p.tiles + 4 * tile;
        KvWalk w;
        w.init(p.kv + 8 * t[2]);
        for (; !w.done(); w.next()) {
          if (!mbar_wait(&v_empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* v = sV + stage * AT_KV_BYTES;
          last_phase[stage] = (int)phase;
          mbar_arrive_expect_tx(&v_full[stage], AT_KV_BYTES);
          tma_load_2d(v, &tmV, &v_full[stage], head * AT_D, w.start());
          tma_load_2d(v + AT_KV_BYTES / 2, &tmV, &v_full[stage], head * AT_D + 64, w.start());
          if (++stage == AT_VSTAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok || *abort_flag) {
        long long t0 = clock64();
        for (int i = 0; i < AT_VSTAGES; ++i) {
          if (last_phase[i] < 0) continue;
          while (!mbar_try_wait(&v_full[i], (uint32_t)last_phase[i]) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------------- MMA issuer
    // Per block j and tile t, in this order: O_t += P_t(j-1) V(j-1) with P read from TMEM
    // (where the softmax stored it over S_t), then S_t = Q_t K(j)^T. MMAs run in issue
    // order, so the S_t write follows the P_t read. The tcgen05 issue queue is about one
    // MMA deep, so this thread's instruction count sits on the tensor pipe's critical path:
    // the loop keeps only a block count (no range walk) and builds each operand descriptor
    // once, advancing only its start-address field (addr >> 4 in the low 14 bits; shared
    // memory is < 256 KB, so the add never carries out of the field).
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(AT_BM, AT_BN, false, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(AT_BM, AT_D, false, true);
      const uint32_t dq_lo0 = (uint32_t)umma_desc_kmajor_sw128(smem_u32(sQ));
      const uint32_t dq_hi = (uint32_t)(umma_desc_kmajor_sw128(smem_u32(sQ)) >> 32);
      const uint32_t dk_lo0 = (uint32_t)umma_desc_kmajor_sw128(smem_u32(sK));
      const uint32_t dv_lo0 = (uint32_t)umma_desc_mnmajor_sw128(smem_u32(sV), AT_KV_BYTES / 2);
      const uint32_t dv_hi = (uint32_t)(umma_desc_mnmajor_sw128(smem_u32(sV), AT_KV_BYTES / 2) >> 32);
      auto desc = [](uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; };
      int kstage = 0, vstage = 0;
      uint32_t kphase = 0, vphase = 0;
      uint32_t g = 0;  // global block counter: S_t / P_t phases are g & 1
      int local = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++local) {
        int head, tile;
        item_coords(p, item, head, tile);
        const int* t = p.tiles + 4 * tile;
        // blocks of this item: 128-key blocks over its (at most four) K/V ranges
        const int* kv = p.kv + 8 * t[2];
        int nblk = 0;
#pragma unroll
        for (int rg = 0; rg < AT_MAX_RANGES; ++rg) {
          const int len = kv[2 * rg + 1] - kv[2 * rg];
          nblk += len > 0 ? (len + AT_BN - 1) / AT_BN : 0;
        }
        if (!mbar_wait(q_full, local & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        if (nblk == 0) {
          // no K/V at all: release the epilogue (it writes zeros)
          umma_commit(&pv_done[0]);
          umma_commit(&pv_done[1]);
          umma_commit(q_empty);
          continue;
        }
        for (int j = 0; j <= nblk && ok; ++j) {
          const bool have = j < nblk;
          const uint32_t dk_lo = dk_lo0 + (uint32_t)(kstage * (AT_KV_BYTES >> 4));
          const uint32_t dv_lo = dv_lo0 + (uint32_t)(vstage * (AT_KV_BYTES >> 4));
#pragma unroll
          for (int qt = 0; qt < 2; ++qt) {
            const uint32_t tS = tmem + qt * AT_BN;
            if (j > 0) {
              if ((qt == 0 && !mbar_wait(&v_full[vstage], vphase, abort_flag, p.err,
                                                 kErrTimeoutMma)) ||
                  (j == 1 && local > 0 &&
                   !mbar_wait(&o_empty[qt], (local - 1) & 1, abort_flag, p.err,
                                      kErrTimeoutMma)) ||
                  !mbar_wait(&p_full[qt], (g - 1) & 1, abort_flag, p.err,
                                     kErrTimeoutMma)) {
                ok = false;
                break;
              }
              tc_fence_after();
#pragma unroll
              for (int k = 0; k < AT_BN / 16; ++k)
                umma_f16_ts(tmem + 256 + qt * 128, tS + k * 8,
                            desc(dv_lo + (uint32_t)((k * 2048) >> 4), dv_hi), idesc_o,
                            (j > 1 || k > 0) ? 1u : 0u);
              if (!have) umma_commit(&pv_done[qt]);
            }
            if (have) {
              if (qt == 0) {
                if (!mbar_wait(&k_full[kstage], kphase, abort_flag, p.err,
                                       kErrTimeoutMma)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
              }
              const uint32_t dq_lo = dq_lo0 + (uint32_t)(qt * (AT_Q_BYTES >> 4));
#pragma unroll
              for (int k = 0; k < AT_D / 16; ++k) {
                const uint32_t off = (uint32_t)(((k >> 2) * (AT_Q_BYTES / 2) + (k & 3) * 32) >> 4);
                umma_f16_ss(tS, desc(dq_lo + off, dq_hi), desc(dk_lo + off, dq_hi), idesc_s,
                            k != 0);
              }
              umma_commit(&s_full[qt]);
            }
          }
          if (!ok) break;
          if (have) {
            umma_commit(&k_empty[kstage]);
            if (++kstage == AT_KSTAGES) {
              kstage = 0;
              kphase ^= 1;
            }
          }
          if (j > 0) {
            umma_commit(&v_empty[vstage]);
            if (++vstage == AT_VSTAGES) {
              vstage = 0;
              vphase ^= 1;
            }
          }
          if (have) ++g;
        }
        if (!ok) break;
        umma_commit(q_empty);
      }
      umma_commit(mma_done);
      long long t0 = clock64();
      while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  }
  } else {
    // ------------------------------------------------------- softmax + epilogue warps
    setmaxnreg_inc<AT_REGS_HIGH>();
    const int qt = (warp - 4) >> 2;           // which query tile
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;        // row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + qt * AT_BN;
    const uint32_t tP = tS;                   // P (bf16 pairs) over the first 64 columns of S
    const uint32_t tO = tmem + lane_off + 256 + qt * 128;
    uint32_t g = 0;
    int local = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++local) {
      int head, tile;
      item_coords(p, item, head, tile);
      const int* t = p.tiles + 4 * tile;
      KvWalk w;
      w.init(p.kv + 8 * t[2]);
      float m_ref = -INFINITY, l = 0.f;
      int j = 0;
      bool ok = true;
      const bool tr = (r == 0);
      for (; !w.done(); w.next(), ++j, ++g) {
        if (tr) at_trace(p, TR_S_WAIT, qt, g);
        if (!mbar_wait(&s_full[qt], g & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (tr) at_trace(p, TR_S_READY, qt, g);
        float s[AT_BN];
#pragma unroll
        for (int c = 0; c < AT_BN; c += 32) {
          uint32_t u[32];
          tmem_ld32(tS + c, u);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(u[i]);
        }
        tmem_wait_ld();
        if (tr) at_trace(p, TR_LD_DONE, qt, g);
        constexpr bool kPacked = AT_VARIANT >= 1;
        constexpr int kPolyPairs = (AT_VARIANT >= 2 && AT_VARIANT <= 4) ? AT_VARIANT - 1 : 0;
        constexpr bool kNoMufu = AT_VARIANT == 5, kNoCvt = AT_VARIANT == 6, kNoStore = AT_VARIANT == 7;
        // only a ragged block is masked
        const int valid = w.valid();
        if (valid < AT_BN) {
#pragma unroll
          for (int c = 0; c < AT_BN; ++c) s[c] = c < valid ? s[c] : -INFINITY;
        }
        float sums[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        // p = 2^(s * scale_log2 - m), packed bf16 pairs written over S_t in TMEM
        auto exp_pass = [&](float neg_m) {
          if constexpr (!kPacked) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t pk[32];
#pragma unroll
              for (int c = 0; c < 64; c += 8) {
                float e[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  e[i] = ex2(fmaf(s[h * 64 + c + i], p.scale_log2, neg_m));
                  sums[i] += e[i];
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) pk[c / 2 + i] = pack_bf16(e[2 * i], e[2 * i + 1]);
              }
              tmem_st32(tP + h * 32, pk);
            }
          } else {
            const float2 sc = make_float2(p.scale_log2, p.scale_log2);
            const float2 nm = make_float2(neg_m, neg_m);
            float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f)};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t pk[32];
#pragma unroll
              for (int c = 0; c < 64; c += 16) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {   // pair i of this 16-score group
                  const int col = h * 64 + c + 2 * i;
                  const float2 x = __ffma2_rn(make_float2(s[col], s[col + 1]), sc, nm);
                  float2 e;
                  if (i >= 8 - kPolyPairs) {
                    e = ex2_poly2(x);
                  } else if (kNoMufu) {
                    e = x;
                  } else {
                    e = make_float2(ex2(x.x), ex2(x.y));
                  }
                  acc[i & 3] = __fadd2_rn(acc[i & 3], e);
                  pk[c / 2 + i] = kNoCvt ? __byte_perm(__float_as_uint(e.x), __float_as_uint(e.y), 0x7632)
                                         : pack_bf16(e.x, e.y);
                }
              }
              if (!kNoStore) tmem_st32(tP + h * 32, pk);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              sums[2 * i] = acc[i].x;
              sums[2 * i + 1] = acc[i].y;
            }
          }
        };
        // O rescale (warp-collective TMEM round trip; rows that keep their max use 1)
        auto rescale_o = [&](float factor) {
#pragma unroll 1
          for (int c = 0; c < AT_D; c += 32) {
            uint32_t u[32];
            tmem_ld32(tO + c, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * factor);
            tmem_st32(tO + c, u);
          }
        };
        {
          // row max on the raw scores (8 independent chains of 3-input max)
          float mxv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) mxv[i] = s[i];
#pragma unroll
          for (int c = 8; c < AT_BN; c += 16)
#pragma unroll
            for (int i = 0; i < 8; ++i) mxv[i] = fmax3(mxv[i], s[c + i], s[c + 8 + i]);
          const float mx = fmax3(fmax3(mxv[0], mxv[1], mxv[2]), fmax3(mxv[3], mxv[4], mxv[5]),
                                 fmaxf(mxv[6], mxv[7])) * p.scale_log2;
          const float m_new = fmaxf(m_ref, mx);
          const bool need = m_new > m_ref + 8.0f;
          const bool warp_need = __any_sync(0xffffffffu, need);
          if (tr) at_trace(p, TR_MAX_DONE, qt, g);
          float factor = 1.f;
          if (need) {
            factor = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - m_new);
            m_ref = m_new;
            l *= factor;
          }
          // S_t(j) completes after P_t(j-1).V(j-1) (in-order MMAs), so O is complete and may
          // be rescaled before this block's P is published.
          if (j > 0 && warp_need) rescale_o(factor);
          exp_pass((m_ref == -INFINITY) ? 0.f : -m_ref);
        }
        l += ((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7]));
        if (tr) at_trace(p, TR_EXP_DONE, qt, g);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[qt]);
        if (tr) at_trace(p, TR_P_ARRIVE, qt, g);
      }
      if (!ok) break;
      // Epilogue: wait for the item's last P.V, O / l * gate -> bf16.
      if (!mbar_wait(&pv_done[qt], local & 1, abort_flag, p.err, kErrTimeoutSoftmax)) break;
      tc_fence_after();
      const int row = t[0] + qt * AT_BM + r;
      const bool row_ok = row < t[1];
      float gscale = j > 0 ? 1.f / l : 0.f;   // an item without K/V writes zeros
      // the softmax denominator in the exp2 domain, for the backward: p = 2^(s*c - lse)
      if (p.lse && row_ok) p.lse[(int64_t)head * p.T + row] = j > 0 ? m_ref + log2f(l) : 0.f;
      if (p.gate && row_ok) gscale *= sigmoidf_(__bfloat162float(p.gate[(int64_t)row * p.ldg + head]));
#pragma unroll 1
      for (int c = 0; c < AT_D; c += 32) {
        uint32_t u[32];
        tmem_ld32(tO + c, u);
        tmem_wait_ld();
        if (row_ok) {
          uint32_t o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            o[i] = pack_bf16(__uint_as_float(u[2 * i]) * gscale, __uint_as_float(u[2 * i + 1]) * gscale);
          uint4* dst = reinterpret_cast<uint4*>(p.scatter.row_ptr(p.out, p.ldo, row) + head * AT_D + c);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&o_empty[qt]);
    }
  }

  if (clock_probe) {
    p.trace[AT_TRACE_SLOTS + 2] = (long long)globaltimer_ns();
    p.trace[AT_TRACE_SLOTS + 3] = clock64();
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

void launch_window_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                             int64_t ldv, int T, int H, const int* tiles, int n_tiles,
                             const int* kv, const void* gate, int64_t ldg, void* out,
                             int64_t ldo, float scale, int* err, cudaStream_t stream,
                             const RowScatter* scatter, long long* trace, float* lse) {
  if (n_tiles == 0 || H == 0) return;
  static std::atomic<uint64_t> attr{0};
  using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, AttnParams);
  static const KernelFn kernels[AT_VARIANTS] = {
      window_attention_kernel<0>, window_attention_kernel<1>, window_attention_kernel<2>,
      window_attention_kernel<3>, window_attention_kernel<4>, window_attention_kernel<5>,
      window_attention_kernel<6>, window_attention_kernel<7>};
  if (attr_needed(attr)) {
    // setmaxnreg.inc waits until the registers it asks for are free: refuse to launch if
    // the compiled launch register count cannot fund the split.
    for (auto fn : kernels) {
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess ||
          fa.numRegs * AT_THREADS < 128 * AT_REGS_LOW + 256 * AT_REGS_HIGH)
        throw std::runtime_error("window attention: launch registers cannot fund the "
                                 "warpgroup register split");
    }
    attr_done(attr);
  }
  const uint64_t cols = (uint64_t)H * AT_D;
  CUtensorMap tq = make_tmap_2d(q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, T, ldq * 2, 64, AT_BM);
  CUtensorMap tk = make_tmap_2d(k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, T, ldk * 2, 64, AT_BN);
  CUtensorMap tv = make_tmap_2d(v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, T, ldv * 2, 64, AT_BN);
  AttnParams p;
  p.tiles = tiles;
  p.kv = kv;
  p.n_tiles = n_tiles;
  p.H = H;
  p.T = T;
  p.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  p.ldg = ldg;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.scatter = RowScatter{};
  if (scatter) p.scatter = *scatter;
  p.trace = trace;
  p.lse = lse;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err;
  const int items = n_tiles * H;
  const int grid = items < num_sms() ? items : num_sms();
  kernels[g_variant]<<<grid, AT_THREADS, AT_SMEM, stream>>>(tq, tk, tv, p);
}

void attention_set_variant(int v) {
  if (v < 0 || v >= AT_VARIANTS) throw std::runtime_error("window attention: variant 0..7");
  g_variant = v;
}
int attention_variant() { return g_variant; }

}  // namespace vdn
