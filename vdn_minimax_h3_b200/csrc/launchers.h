// Raw-pointer launch API of the CUDA translation units. The .cu files include only CUDA
// headers (fast nvcc builds); ops.cpp adapts torch tensors onto these.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <cuda_bf16.h>

#include <atomic>

namespace vdn {

// Kernel attributes (dynamic shared-memory limit, carveout) are per device: a launcher
// sets them the first time it runs on each device. `attr_needed` is true until
// `attr_done` has been called for the current device (ordinals 0..63).
inline int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}
inline bool attr_needed(const std::atomic<uint64_t>& done) {
  return !(done.load(std::memory_order_acquire) & (1ull << (current_device() & 63)));
}
inline void attr_done(std::atomic<uint64_t>& done) {
  done.fetch_or(1ull << (current_device() & 63), std::memory_order_release);
}

// Row-owner scatter of an epilogue's output rows. Under Ulysses the rows of the packed
// sequence are owned in contiguous shards of `rows_per_rank`; an epilogue that produced row
// g (g = row0 + local output row) stores it to base[g / rows_per_rank] at row
// g % rows_per_rank: the owner's buffer, local or a peer's mapped into this process.
// n == 0 disables the scatter (plain out + row * ldo).
constexpr int kMaxScatterRanks = 8;
struct RowScatter {
  __nv_bfloat16* base[kMaxScatterRanks];  // bf16 pointers
  int64_t row0;
  int rows_per_rank;
  int n;
#ifdef __CUDACC__
  __device__ __forceinline__ __nv_bfloat16* row_ptr(__nv_bfloat16* out, int64_t ldo,
                                                    int64_t row) const {
    if (n == 0) return out + row * ldo;
    const int64_t g = row0 + row;
    const int r = (int)(g / rows_per_rank);
    return base[r] + (g - (int64_t)r * rows_per_rank) * ldo;
  }
#endif
};


struct GemmArgs {
  const void* A;   // [M, K] bf16, row stride lda (elements)
  const void* B;   // [N, K] bf16, row stride ldb
  int64_t lda, ldb;
  int M, N, K;
};

// mode: 0 store, 1 gated residual, 2 swiglu (interleaved), 3 accumulate
void launch_gemm_bf16(const GemmArgs& a, int mode, void* out, int64_t ldo, const float* bias,
                      const void* gate, int64_t ldg, const int* gate_idx, int* err,
                      cudaStream_t stream);

// C (+)= A @ B^T with either operand stored MN-major: a_mn = A held as [K, M] (row stride
// lda), b_mn = B held as [K, N] (row stride ldb); GemmArgs' M, N, K are the product's.
// The input and weight gradients of a Linear (gemm.cu, LAYOUT).
void launch_gemm_bf16_layout(const GemmArgs& a, bool a_mn, bool b_mn, bool accumulate, void* out,
                             int64_t ldo, int* err, cudaStream_t stream);

// Routed epilogue (see gemm.cu, EPI_ROUTE). `route` holds `planes` tables of N/8 addresses;
// every column group is stored to each plane that has an address for it, except the
// 128-wide q/k heads in [q0,q1) and [k0,k1): raw values to plane 0, normalised + rotated
// values to plane 1.
struct GemmRoute {
  const long long* route;
  int64_t route_ld[8];
  int planes;
  int q0, q1, k0, k1;
  const float* norm_q;
  const float* norm_k;
  float qk_eps;
  const float* rope_cos;
  const float* rope_sin;
  int64_t ld_rope;
};
void launch_gemm_bf16_routed(const GemmArgs& a, const GemmRoute& r, const float* bias, int* err,
                             cudaStream_t stream);

// Block-scaled fp8 GEMM (gemm_fp8.cu). A [M, K], B [N, K] E4M3 with row strides in bytes;
// sfa / sfb the blocked UE8M0 scale factors (A per 128 rows, B per 256-row tile).
struct GemmFp8Args {
  const void* A;
  const void* B;
  int64_t lda, ldb;
  const void* sfa;
  const void* sfb;
  int M, N, K;
};
// mode: 0 store bf16, 1 gated residual, 2 swiglu -> E4M3 + scale factors
void launch_gemm_fp8(const GemmFp8Args& a, int mode, void* out, int64_t ldo, const float* bias,
                     const void* gate, int64_t ldg, const int* gate_idx, void* q_out, int64_t ldq,
                     void* q_sf, int* err, cudaStream_t stream);
void gemm_fp8_set_trace(long long* t);   // diagnostics: per-CTA wait cycles (or null)
void launch_gemm_fp8_routed(const GemmFp8Args& a, const GemmRoute& r, const float* bias, int* err,
                            cudaStream_t stream);
void launch_gemm_fp8_f32_scatter(const GemmFp8Args& a, void* out, int64_t ldo, const RowScatter& sc,
                                 int* err, cudaStream_t stream);
void launch_gemm_bf16_f32_scatter(const GemmArgs& a, void* out, int64_t ldo, const RowScatter& sc,
                                  int* err, cudaStream_t stream);
void launch_residual_combine(void* x, int64_t ldx, const void* a, const void* b, int64_t ldp,
                             const float* bias, const void* gate, int64_t ldg, const int* idx,
                             int R, int D, cudaStream_t stream);
void launch_quant_rows(const void* x, int64_t ldx, int M, int K, void* q, int64_t ldq, void* sf,
                       cudaStream_t stream);

// Destinations of the AdaLN norm: up to two copies (this GPU's buffer and a peer's, for a
// tensor-parallel all-gather done by the producer) of the bf16 rows and/or their E4M3
// quantisation; local row r lands at row row0 + r of each.
struct NormDst {
  __nv_bfloat16* out[2];
  uint8_t* q[2];
  uint8_t* qsf[2];
  int64_t ldo, ldq, row0;
};
void launch_adaln_rmsnorm_dst(const void* x, int64_t ldx, const float* w, float eps,
                              const void* table, int64_t ldt, int shift_col, int scale_col,
                              const int* idx, const NormDst& dst, int T, int D,
                              cudaStream_t stream);
// out (bf16) and/or q + qsf (E4M3 with one scale per 1x128 block; D % 256 == 0)
void launch_adaln_rmsnorm(const void* x, int64_t ldx, const float* w, float eps, const void* table,
                          int64_t ldt, int shift_col, int scale_col, const int* idx, void* out,
                          int64_t ldo, int T, int D, cudaStream_t stream, void* q = nullptr,
                          int64_t ldq = 0, void* qsf = nullptr);
// Destinations of the frame sums in peers' memory (see frame_sums_kernel); n == 0: `out`.
struct FrameSumDst {
  float* base[kMaxScatterRanks];
  int64_t offset;
  int n;
};
void launch_frame_sums(const void* x, int64_t ldx, int64_t row0, int64_t nrows, int64_t vs,
                       int F, int S, int D, float* out, cudaStream_t stream,
                       const FrameSumDst* dst = nullptr);
void launch_qk_prep(const void* src, int64_t lds, int T, int H, int d, const float* w, float eps,
                    const float* cosv, const float* sinv, int rot, void* out, int64_t ldo,
                    cudaStream_t stream);

void launch_window_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                             int64_t ldv, int T, int H, const int* tiles, int n_tiles,
                             const int* kv, const void* gate, int64_t ldg, void* out,
                             int64_t ldo, float scale, int* err, cudaStream_t stream,
                             const RowScatter* scatter = nullptr, long long* trace = nullptr,
                             float* lse = nullptr);

void attention_set_variant(int v);

// Training backward of the window attention (attention_bwd.cu). q/k/v/dout/o and the
// gradients are [T, H*128] bf16 row views; lse (log2 domain, from the forward) and delta
// (written by the dq pass) are fp32 [H, T]. q_tiles/kv_ranges: the forward plan (query
// tiles of <= 128 rows here); k_tiles/q_ranges: the transposed plan (key tiles).
struct AttnBwdArgs {
  const void *q, *k, *v, *o, *dout;
  int64_t ldq, ldk, ldv, ldo, lddo;
  void *dq, *dk, *dv;
  int64_t lddq, lddk, lddv;
  const float* lse;
  float* delta;
  int T, H;
  const int* q_tiles;
  int n_q_tiles;
  const int* kv_ranges;
  const int* k_tiles;
  int n_k_tiles;
  const int* q_ranges;
  float scale;
  int* err;
};
void launch_attention_bwd(const AttnBwdArgs& a, cudaStream_t stream);
int attention_variant();

// Symmetric memory (symmetric.cu): IPC-exported regions and the peer flag barrier.
void* symm_malloc(size_t nbytes, void* handle_out);
void* symm_open(const void* handle);
void symm_close(void* peer_ptr);
void symm_free(void* p);
void launch_symm_reduce_scatter(const float* const* srcs, int P, int64_t offset, int64_t n,
                                float scale, float* out, cudaStream_t stream);

// out[q * shard_bytes ...] = srcs[q][0 .. shard_bytes) for every rank q != rank (the FSDP2
// parameter all-gather over symmetric memory; this rank's shard is already in `out`).
void launch_symm_all_gather(const void* const* srcs, int P, int rank, int64_t shard_bytes, void* out,
                            cudaStream_t stream);
void launch_symm_barrier(unsigned long long* counter, unsigned long long* local_flags,
                         unsigned long long* const* peer_flags, int rank, int P,
                         long long timeout_ns, int* err, cudaStream_t stream);
void launch_lb_activate(const void* in, int64_t ldi, int N, int H, void* out, int64_t ldo, int l2,
                        cudaStream_t stream);
void launch_lb_conv(const void* in, int64_t ldi, const float* wsp, const float* wtm, void* out,
                    int64_t ldo, int F, int gh, int gw, int H, int l2, int* err,
                    cudaStream_t stream);
// Two-pass form: spatial conv into `tmp` (bf16, [F*gh*gw, H*128] rows of stride ldt), then
// temporal conv + SiLU [+ L2] into `out`. Here `wsp` is TAP-major, [25, H*128].
void launch_lb_conv2(const void* in, int64_t ldi, const float* wsp, const float* wtm, void* tmp,
                     int64_t ldt, void* out, int64_t ldo, int F, int gh, int gw, int H, int l2,
                     int* err, cudaStream_t stream);
void launch_lb_frame_stats(const void* k, int64_t ldk, const void* v, int64_t ldv, int F, int S,
                           int H, const float* beta, float* A, float* B, int* err,
                           cudaStream_t stream);
void launch_lb_spd_factor(const float* A, const float* B, const float* alpha, float* trans,
                          float* inj, int n_mats, float a_scale, float b_scale,
                          cudaStream_t stream);
void launch_lb_scan(const float* trans, const float* inj, const float* start, int F, int H,
                    float* prefix, float* suffix, int* err, cudaStream_t stream, int ndir = 2);
// Scan cluster size: 0 = automatic (by head count), else 1, 2, 4 or 8.
void lb_scan_set_cluster(int cs);
// Backward of the AdaLN-modulated RMSNorm (norm_bwd.cu): dx from x, dy, the norm weight
// (nullable) and the scale columns of the AdaLN table rows picked by idx.
void launch_adaln_rmsnorm_bwd(const void* x, int64_t ldx, const void* dy, int64_t ldy,
                              const float* w, float eps, const void* table, int64_t ldt,
                              int scale_col, const int* idx, void* dx, int64_t ldo, int T, int D,
                              cudaStream_t stream);
// Backward of the two-pass short conv (conv_bwd.cu): dtmp is fp32 scratch [F*gh*gw, H*128];
// dwsp [25, H*128] and dwtm [H*128, 5] are accumulated into (the caller zeroes them).
void launch_lb_conv2_bwd(const void* in, int64_t ldi, const void* tmp, int64_t ldt,
                         const void* dy, int64_t ldy, const float* wsp, const float* wtm,
                         float* dtmp, void* dx, int64_t ldx, float* dwsp, float* dwtm, int F,
                         int gh, int gw, int H, int l2, cudaStream_t stream);
void launch_lb_gather(const float* prefix, const float* suffix, const int* idx, const float* ab,
                      const float* aa, const float* start, int F, int H, void* out,
                      cudaStream_t stream);
void launch_lb_readout(const void* q, int64_t ldq, const void* state, int F, int S, int H,
                       const float* w, const void* gate, int64_t ldg, int gate_logits, void* out,
                       int64_t ldo, float eps, int* err, cudaStream_t stream,
                       const RowScatter* scatter = nullptr);

}  // namespace vdn
