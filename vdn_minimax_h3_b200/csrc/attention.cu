// Window softmax attention on the 5th-generation tensor cores (sm_100a).
//
// One work item = (head, 128-row query tile). The tile belongs to a plan segment whose kept
// K/V rows are at most four CONTIGUOUS row ranges of the packed sequence (globals, the
// window frames, the anchor frames; models/window.py: AttentionPlan). The kernel walks
// those ranges in 128-key blocks straight out of the [T, H, d] projections -- no gather,
// no mask tensor; only the ragged tail of each range is masked.
//
// Roles (192 threads, one CTA per SM, persistent over head-major work items so the CTAs
// in flight share one head's K/V in L2):
//   warp 0     TMA producer: Q tile once per item, K/V blocks into a 2-stage ring.
//   warp 1     MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM S buffers
//              (kind::f16, M=128, N=128, K=16 x 8), then O += P_{j-1} V_{j-1} with P from
//              shared memory (K-major) and V as an MN-major operand; commits free K/V
//              stages and signal the softmax warps.
//   warps 2-5  softmax (thread = query row): S row from TMEM (tcgen05.ld), online softmax
//              in the exp2 domain with a lazy rescale (O in TMEM is rescaled only when the
//              running max grows by more than 2^8), P (bf16) written into the 128B-swizzled
//              shared-memory operand, and the epilogue O / l * sigmoid(gate) -> bf16.
// TMEM: S0 [0,128), S1 [128,256), O [256,384) of a 512-column allocation.
//
// Every wait is bounded; a protocol failure unwinds, drains and frees TMEM (common.cuh).
// Reference parity: the window softmax of src/models/softmax_attention/ (decomposed.py's
// dense leg + varlen leg, flex_attention.py) and the softmax gate (kernels.py:51-67).
#include "common.cuh"
#include "launchers.h"
#include "tma.cuh"

namespace vdn {

constexpr int AT_BM = 128;      // query rows per tile
constexpr int AT_BN = 128;      // keys per block
constexpr int AT_D = 128;       // head dim
constexpr int AT_STAGES = 2;
constexpr int AT_TILE_BYTES = AT_BM * AT_D * 2;  // 32 KB (two 64-column swizzle atoms)
constexpr int AT_THREADS = 192;
constexpr int AT_SMEM = AT_TILE_BYTES * (1 /*Q*/ + 2 * AT_STAGES /*K,V*/ + 1 /*P*/) + 1024 + 512;
constexpr int AT_MAX_RANGES = 4;

struct AttnParams {
  const int* tiles;          // [n_tiles, 4] (q0, q1, segment, kv_len)
  const int* kv;             // [n_seg, 8] (start, end) x 4
  int n_tiles, H, T;
  const __nv_bfloat16* gate; // [T, ldg] logits per head, or null
  int64_t ldg;
  __nv_bfloat16* out;        // [T, ldo], head h at column h*128
  int64_t ldo;
  float scale_log2;          // softmax scale * log2(e)
  int* err;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Iterates the 128-key blocks of a segment's K/V ranges.
struct KvWalk {
  int r[2 * AT_MAX_RANGES];
  int range, pos;
  __device__ void init(const int* kv_row) {
#pragma unroll
    for (int i = 0; i < 2 * AT_MAX_RANGES; ++i) r[i] = kv_row[i];
    range = 0;
    pos = r[0];
    skip_empty();
  }
  __device__ void skip_empty() {
    while (range < AT_MAX_RANGES && pos >= r[2 * range + 1]) {
      ++range;
      if (range < AT_MAX_RANGES) pos = r[2 * range];
    }
  }
  __device__ bool done() const { return range >= AT_MAX_RANGES; }
  __device__ int start() const { return pos; }
  __device__ int valid() const { return min(AT_BN, r[2 * range + 1] - pos); }
  __device__ void next() {
    pos += AT_BN;
    skip_empty();
  }
};

__device__ __forceinline__ void item_coords(const AttnParams& p, int item, int& head, int& tile) {
  head = item / p.n_tiles;
  tile = item - head * p.n_tiles;
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    window_attention_kernel(const __grid_constant__ CUtensorMap tmQ,
                            const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + AT_TILE_BYTES;
  uint8_t* sV = sK + AT_STAGES * AT_TILE_BYTES;
  uint8_t* sP = sV + AT_STAGES * AT_TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + AT_TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;    // [2]
  uint64_t* k_empty = bars + 4;   // [2]
  uint64_t* v_full = bars + 6;    // [2]
  uint64_t* v_empty = bars + 8;   // [2]
  uint64_t* s_full = bars + 10;   // [2]
  uint64_t* s_empty = bars + 12;  // [2]
  uint64_t* p_full = bars + 14;
  uint64_t* pv_done = bars + 15;
  uint64_t* o_empty = bars + 16;
  uint64_t* mma_done = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int n_items = p.n_tiles * p.H;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < AT_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(o_empty, 128);
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

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      int last_phase[2 * AT_STAGES + 1];
      for (int i = 0; i < 2 * AT_STAGES + 1; ++i) last_phase[i] = -1;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++local) {
        int head, tile;
        item_coords(p, item, head, tile);
        const int* t = p.tiles + 4 * tile;
        if (!mbar_wait(q_empty, (local & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        last_phase[2 * AT_STAGES] = local & 1;
        mbar_arrive_expect_tx(q_full, AT_TILE_BYTES);
        tma_load_2d(sQ, &tmQ, q_full, head * AT_D, t[0]);
        tma_load_2d(sQ + AT_TILE_BYTES / 2, &tmQ, q_full, head * AT_D + 64, t[0]);
        KvWalk w;
        w.init(p.kv + 8 * t[2]);
        for (; !w.done(); w.next()) {
          if (!mbar_wait(&k_empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* k = sK + stage * AT_TILE_BYTES;
          last_phase[stage] = (int)phase;
          mbar_arrive_expect_tx(&k_full[stage], AT_TILE_BYTES);
          tma_load_2d(k, &tmK, &k_full[stage], head * AT_D, w.start());
          tma_load_2d(k + AT_TILE_BYTES / 2, &tmK, &k_full[stage], head * AT_D + 64, w.start());
          if (!mbar_wait(&v_empty[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* v = sV + stage * AT_TILE_BYTES;
          last_phase[AT_STAGES + stage] = (int)phase;
          mbar_arrive_expect_tx(&v_full[stage], AT_TILE_BYTES);
          tma_load_2d(v, &tmV, &v_full[stage], head * AT_D, w.start());
          tma_load_2d(v + AT_TILE_BYTES / 2, &tmV, &v_full[stage], head * AT_D + 64, w.start());
          if (++stage == AT_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // On abort, let every copy this thread issued land before the CTA exits.
      if (!ok || *abort_flag) {
        long long t0 = clock64();
        for (int i = 0; i < 2 * AT_STAGES + 1; ++i) {
          uint64_t* bar = i < AT_STAGES ? &k_full[i] : (i < 2 * AT_STAGES ? &v_full[i - AT_STAGES] : q_full);
          const int par = last_phase[i];
          if (par < 0) continue;
          while (!mbar_try_wait(bar, (uint32_t)par) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(AT_BM, AT_BN, false, false);
      constexpr uint32_t idesc_o = umma_idesc_bf16(AT_BM, AT_D, false, true);
      const uint32_t aQ = smem_u32(sQ), aP = smem_u32(sP);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t g = 0;  // global block counter (S buffer = g & 1)
      int local = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++local) {
        int head, tile;
        item_coords(p, item, head, tile);
        const int* t = p.tiles + 4 * tile;
        if (!mbar_wait(q_full, local & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        KvWalk w;
        w.init(p.kv + 8 * t[2]);
        int j = 0;
        int prev_stage = 0;
        uint32_t prev_phase = 0, g_prev = 0;
        while (true) {
          const bool have = !w.done();
          if (have) {
            // S_j = Q K_j^T into S buffer (g & 1)
            const uint32_t b = g & 1;
            if (!mbar_wait(&k_full[stage], phase, abort_flag, p.err, kErrTimeoutMma) ||
                !mbar_wait(&s_empty[b], ((g >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t aK = smem_u32(sK + stage * AT_TILE_BYTES);
#pragma unroll
            for (int k = 0; k < AT_D / 16; ++k) {
              const uint32_t off = (k >> 2) * (AT_TILE_BYTES / 2) + (k & 3) * 32;
              umma_f16_ss(tmem + b * 128, umma_desc_kmajor_sw128(aQ + off),
                          umma_desc_kmajor_sw128(aK + off), idesc_s, k != 0);
            }
            umma_commit(&k_empty[stage]);
            umma_commit(&s_full[b]);
          }
          if (j > 0) {
            // O += P_{j-1} V_{j-1}
            if (!mbar_wait(p_full, g_prev & 1, abort_flag, p.err, kErrTimeoutMma) ||
                !mbar_wait(&v_full[prev_stage], prev_phase, abort_flag, p.err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            if (j == 1 && local > 0 &&
                !mbar_wait(o_empty, (local - 1) & 1, abort_flag, p.err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t aV = smem_u32(sV + prev_stage * AT_TILE_BYTES);
#pragma unroll
            for (int k = 0; k < AT_BN / 16; ++k) {
              const uint32_t offP = (k >> 2) * (AT_TILE_BYTES / 2) + (k & 3) * 32;
              umma_f16_ss(tmem + 256, umma_desc_kmajor_sw128(aP + offP),
                          umma_desc_mnmajor_sw128(aV + k * 2048, AT_TILE_BYTES / 2), idesc_o,
                          (j > 1 || k > 0) ? 1u : 0u);
            }
            umma_commit(&v_empty[prev_stage]);
            umma_commit(pv_done);
          }
          if (!have) break;
          prev_stage = stage;
          prev_phase = phase;
          g_prev = g;
          if (++stage == AT_STAGES) {
            stage = 0;
            phase ^= 1;
          }
          ++g;
          ++j;
          w.next();
        }
        if (!ok) break;
        umma_commit(q_empty);
      }
      umma_commit(mma_done);
      long long t0 = clock64();
      while (!mbar_try_wait(mma_done, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else {
    // ------------------------------------------------------- softmax + epilogue warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
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
      for (; !w.done(); w.next(), ++j, ++g) {
        const uint32_t b = g & 1;
        if (!mbar_wait(&s_full[b], (g >> 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[AT_BN];
#pragma unroll
        for (int c = 0; c < AT_BN; c += 32) {
          uint32_t u[32];
          tmem_ld32(tmem + lane_off + b * 128 + c, u);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(u[i]);
        }
        tc_fence_before();
        mbar_arrive(&s_empty[b]);
        const int valid = w.valid();
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < AT_BN; ++c) {
          s[c] = c < valid ? s[c] * p.scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
        const float m_new = fmaxf(m_ref, mx);
        const bool need = m_new > m_ref + 8.0f;
        const bool warp_need = __any_sync(0xffffffffu, need);
        // PV_{j-1} must finish before O is touched or the P buffer is rewritten.
        if (j > 0) {
          if (!mbar_wait(pv_done, (g - 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        float factor = 1.f;
        if (need) {
          factor = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - m_new);
          m_ref = m_new;
          l *= factor;
        }
        if (warp_need && j > 0) {
#pragma unroll 1
          for (int c = 0; c < AT_D; c += 32) {
            uint32_t u[32];
            tmem_ld32(tmem + lane_off + 256 + c, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * factor);
            tmem_st32(tmem + lane_off + 256 + c, u);
          }
          tmem_wait_st();
        }
        const float mref = (m_ref == -INFINITY) ? 0.f : m_ref;
        float sum = 0.f;
        uint8_t* prow = sP + r * 128;
#pragma unroll
        for (int c = 0; c < AT_BN; c += 8) {
          float e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            e[i] = ex2(s[c + i] - mref);
            sum += e[i];
          }
          const uint4 pk = make_uint4(pack_bf16(e[0], e[1]), pack_bf16(e[2], e[3]),
                                      pack_bf16(e[4], e[5]), pack_bf16(e[6], e[7]));
          const int chunk = c >> 3;                  // 16-byte chunk along the keys
          const int atom = chunk >> 3, jj = chunk & 7;
          *reinterpret_cast<uint4*>(prow + atom * (AT_TILE_BYTES / 2) + ((jj ^ (r & 7)) << 4)) = pk;
        }
        l += sum;
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (!ok) break;
      // Epilogue: wait for the last PV, O / l * gate -> bf16.
      if (!mbar_wait(pv_done, (g - 1) & 1, abort_flag, p.err, kErrTimeoutSoftmax)) break;
      tc_fence_after();
      const int row = t[0] + r;
      const bool row_ok = row < t[1];
      float gscale = 1.f / l;
      if (p.gate && row_ok) gscale *= sigmoidf_(__bfloat162float(p.gate[(int64_t)row * p.ldg + head]));
#pragma unroll 1
      for (int c = 0; c < AT_D; c += 32) {
        uint32_t u[32];
        tmem_ld32(tmem + lane_off + 256 + c, u);
        tmem_wait_ld();
        if (row_ok) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack_bf16(__uint_as_float(u[2 * i]) * gscale, __uint_as_float(u[2 * i + 1]) * gscale);
          uint4* dst = reinterpret_cast<uint4*>(p.out + (int64_t)row * p.ldo + head * AT_D + c);
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(o_empty);
    }
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
                             int64_t ldo, float scale, int* err, cudaStream_t stream) {
  if (n_tiles == 0 || H == 0) return;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(window_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         AT_SMEM);
    attr = true;
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
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err;
  const int items = n_tiles * H;
  const int grid = items < num_sms() ? items : num_sms();
  window_attention_kernel<<<grid, AT_THREADS, AT_SMEM, stream>>>(tq, tk, tv, p);
}

}  // namespace vdn
