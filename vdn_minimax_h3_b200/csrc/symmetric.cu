// Symmetric memory over NVLink for one node: every rank cudaMallocs the same-sized region,
// exports a CUDA IPC handle, and maps the peers' regions into its own address space, so a
// kernel on this GPU can store straight into a peer's buffer (NVLink P2P writes through
// NVSwitch). The reference moves the same data with NCCL all_to_all_single
// (src/inference/utils/ulysses_runtime.py:298-305, 348-355, 407-412); here the producing
// kernels (routed GEMM epilogue, attention and readout epilogues) write the peer buffers
// themselves and a flag barrier orders the exchange.
//
// symm_barrier: one warp. Lane 0 bumps this rank's epoch counter; lane p publishes the
// epoch into peer p's flag slot for this rank (st.release.sys after a system fence, so
// everything this stream wrote before, including earlier kernels' peer stores, is visible
// first), then lane q waits for peer q's epoch in the local slot q (ld.acquire.sys). The
// wait is bounded by %globaltimer; on expiry the kernel records kErrTimeoutPeer in the
// error word and returns, leaving the context usable.
#include "common.cuh"

#include <cstring>
#include <stdexcept>
#include <string>

namespace vdn {

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void symm_barrier_kernel(unsigned long long* counter, unsigned long long* local_flags,
                                    unsigned long long* const* peer_flags, int rank, int P,
                                    long long timeout_ns, int* err) {
  const int lane = threadIdx.x;
  unsigned long long e = 0;
  if (lane == 0) {
    e = *counter + 1;
    *counter = e;
  }
  e = __shfl_sync(0xffffffffu, e, 0);
  __threadfence_system();
  if (lane < P) {
    unsigned long long* dst = peer_flags[lane] + rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(e) : "memory");
  }
  if (lane < P) {
    const uint64_t t0 = global_ns();
    while (true) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(local_flags + lane) : "memory");
      if (v >= e) break;
      if ((long long)(global_ns() - t0) > timeout_ns) {
        atomicExch(err, kErrTimeoutPeer);
        break;
      }
    }
  }
  __syncwarp();
}

static void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void* symm_malloc(size_t nbytes, void* handle_out /* cudaIpcMemHandle_t, 64 bytes */) {
  void* p = nullptr;
  ck(cudaMalloc(&p, nbytes), "cudaMalloc (symmetric region)");
  ck(cudaMemset(p, 0, nbytes), "cudaMemset (symmetric region)");
  ck(cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), p),
     "cudaIpcGetMemHandle");
  return p;
}

void* symm_open(const void* handle) {
  void* p = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return p;
}

void symm_close(void* peer_ptr) { ck(cudaIpcCloseMemHandle(peer_ptr), "cudaIpcCloseMemHandle"); }

void symm_free(void* p) { ck(cudaFree(p), "cudaFree (symmetric region)"); }

// Reduce-scatter by peer loads (the owner pulls): out[i] = scale * sum_p src_p[offset + i],
// fp32, for i < n; src_p is rank p's copy of the same symmetric buffer (this GPU's own copy
// among them). 16-byte vector loads over NVLink, one pass, no staging. Called between two
// flag barriers: the first makes every peer's input visible, the second keeps the peers
// from rewriting their inputs while this rank still reads them.
constexpr int kMaxReducePeers = 8;
struct ReduceSrc {
  const float* p[kMaxReducePeers];
};

template <typename V>
struct GatherSrcT {
  const V* p[kMaxReducePeers];
};

__global__ void __launch_bounds__(256) symm_reduce_scatter_kernel(ReduceSrc src, int P,
                                                                  int64_t offset, int64_t n,
                                                                  float scale, float* __restrict__ out) {
  const int64_t nvec = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < kMaxReducePeers; ++q) {
      if (q < P) {
        const float4 x = *reinterpret_cast<const float4*>(src.p[q] + offset + 4 * v);
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
    }
    acc.x *= scale;
    acc.y *= scale;
    acc.z *= scale;
    acc.w *= scale;
    reinterpret_cast<float4*>(out)[v] = acc;
  }
  // ragged tail (n % 4)
  const int64_t t = (nvec << 2) + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (blockIdx.x == 0 && t < n) {
    float acc = 0.f;
    for (int q = 0; q < P; ++q) acc += src.p[q][offset + t];
    out[t] = acc * scale;
  }
}

void launch_symm_reduce_scatter(const float* const* srcs, int P, int64_t offset, int64_t n,
                                float scale, float* out, cudaStream_t stream) {
  if (P < 1 || P > kMaxReducePeers) throw std::runtime_error("symm_reduce_scatter: 1..8 ranks");
  if (offset % 4 || reinterpret_cast<uintptr_t>(out) % 16)
    throw std::runtime_error("symm_reduce_scatter: offset and output must be 16-byte aligned");
  ReduceSrc s{};
  for (int q = 0; q < P; ++q) {
    if (reinterpret_cast<uintptr_t>(srcs[q]) % 16)
      throw std::runtime_error("symm_reduce_scatter: sources must be 16-byte aligned");
    s.p[q] = srcs[q];
  }
  if (n <= 0) return;
  int blocks = (int)((n / 4 + 255) / 256);
  blocks = blocks < 1 ? 1 : (blocks > 4 * 148 ? 4 * 148 : blocks);
  symm_reduce_scatter_kernel<<<blocks, 256, 0, stream>>>(s, P, offset, n, scale, out);
}

// All-gather of equal shards held in symmetric memory: out[q * shard + i] = src[q][i] for every
// rank q other than `rank` (this rank's shard is already in place). Consecutive threads read
// different peers, so every NVLink peer is streamed from at once. The copy unit V is the
// widest of 16 / 8 / 4 / 2 / 1 bytes that divides the shard size (FSDP pads each parameter's
// dim 0, not the shard total, so a shard need not be a multiple of 16 bytes).
template <typename V>
__global__ void __launch_bounds__(256) symm_all_gather_kernel(GatherSrcT<V> src, int P, int rank,
                                                              int64_t shard_units, V* __restrict__ out) {
  const int others = P - 1;
  const int64_t total = (int64_t)others * shard_units;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t w = i / others;
    const int j = (int)(i - w * others);
    const int q = j + (j >= rank ? 1 : 0);
    out[(int64_t)q * shard_units + w] = src.p[q][w];
  }
}

template <typename V>
static void launch_gather(const void* const* srcs, int P, int rank, int64_t shard_bytes, void* out,
                          cudaStream_t stream) {
  GatherSrcT<V> s{};
  for (int q = 0; q < P; ++q) s.p[q] = reinterpret_cast<const V*>(srcs[q]);
  const int64_t units = shard_bytes / (int64_t)sizeof(V);
  int64_t blocks = ((P - 1) * units + 255) / 256;
  blocks = blocks < 1 ? 1 : (blocks > 8 * 148 ? 8 * 148 : blocks);
  symm_all_gather_kernel<V><<<(int)blocks, 256, 0, stream>>>(s, P, rank, units, reinterpret_cast<V*>(out));
}

void launch_symm_all_gather(const void* const* srcs, int P, int rank, int64_t shard_bytes, void* out,
                            cudaStream_t stream) {
  if (P < 1 || P > kMaxReducePeers) throw std::runtime_error("symm_all_gather: 1..8 ranks");
  if (rank < 0 || rank >= P) throw std::runtime_error("symm_all_gather: rank out of range");
  if (reinterpret_cast<uintptr_t>(out) % 16)
    throw std::runtime_error("symm_all_gather: output must be 16-byte aligned");
  for (int q = 0; q < P; ++q)
    if (reinterpret_cast<uintptr_t>(srcs[q]) % 16)
      throw std::runtime_error("symm_all_gather: sources must be 16-byte aligned");
  if (P == 1 || shard_bytes <= 0) return;
  if (shard_bytes % 16 == 0) launch_gather<uint4>(srcs, P, rank, shard_bytes, out, stream);
  else if (shard_bytes % 8 == 0) launch_gather<uint2>(srcs, P, rank, shard_bytes, out, stream);
  else if (shard_bytes % 4 == 0) launch_gather<uint32_t>(srcs, P, rank, shard_bytes, out, stream);
  else if (shard_bytes % 2 == 0) launch_gather<uint16_t>(srcs, P, rank, shard_bytes, out, stream);
  else launch_gather<uint8_t>(srcs, P, rank, shard_bytes, out, stream);
}

void launch_symm_barrier(unsigned long long* counter, unsigned long long* local_flags,
                         unsigned long long* const* peer_flags, int rank, int P,
                         long long timeout_ns, int* err, cudaStream_t stream) {
  if (P < 1 || P > 32) throw std::runtime_error("symm_barrier: 1..32 ranks");
  symm_barrier_kernel<<<1, 32, 0, stream>>>(counter, local_flags, peer_flags, rank, P,
                                            timeout_ns, err);
}

}  // namespace vdn
