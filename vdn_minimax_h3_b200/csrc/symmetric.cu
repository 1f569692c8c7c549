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

void launch_symm_barrier(unsigned long long* counter, unsigned long long* local_flags,
                         unsigned long long* const* peer_flags, int rank, int P,
                         long long timeout_ns, int* err, cudaStream_t stream) {
  if (P < 1 || P > 32) throw std::runtime_error("symm_barrier: 1..32 ranks");
  symm_barrier_kernel<<<1, 32, 0, stream>>>(counter, local_flags, peer_flags, rank, P,
                                            timeout_ns, err);
}

}  // namespace vdn
