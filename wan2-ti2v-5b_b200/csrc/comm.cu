// Synchronisation of the fused collectives: a barrier of the ranks of a TP group over NVLink
// peer memory.  The reduce-scatter fused into the row-parallel GEMM epilogue and the all-gather
// fused into the LayerNorm store straight into peer buffers; this barrier separates those
// producers from the kernels that read the results.
#include "common.cuh"
#include "internal.h"

namespace wanb200 {

struct BarrierArgs {
  int* flags[WANB200_MAX_PEERS];
  int rank, world, epoch;
  int* err;
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp: lane p < world publishes `epoch` into rank p's flag slot for this rank, then lane
// s < world waits until rank s has published `epoch` into this rank's slot s.  Everything this
// GPU wrote before the launch (earlier kernels on the stream, including stores into peer
// memory) is ordered before the publication by the system-scope fence.
__global__ void __launch_bounds__(32) peer_barrier_kernel(const BarrierArgs a) {
  const int lane = threadIdx.x;
  __threadfence_system();
  int* dst = a.flags[0];
#pragma unroll
  for (int i = 1; i < WANB200_MAX_PEERS; ++i)
    if (lane == i) dst = a.flags[i];
  if (lane < a.world) st_release_sys(dst + a.rank, a.epoch);
  int* mine = a.flags[0];
#pragma unroll
  for (int i = 1; i < WANB200_MAX_PEERS; ++i)
    if (a.rank == i) mine = a.flags[i];
  if (lane < a.world) {
    const unsigned long long t0 = globaltimer();
    while (ld_acquire_sys(mine + lane) < a.epoch) {
      if (globaltimer() - t0 > kWaitTimeoutNs) {
        atomicCAS(a.err, 0, kErrTimeoutPeerBarrier);
        break;
      }
    }
  }
  __syncwarp();
}

int peer_barrier(int* const* flags, int rank, int world, int epoch, cudaStream_t st) {
  if (!flags || world < 1 || world > WANB200_MAX_PEERS || rank < 0 || rank >= world || epoch <= 0)
    return set_error(WANB200_EINVAL, "peer_barrier: need flags, 1 <= world <= 8, 0 <= rank < world, epoch > 0");
  BarrierArgs a;
  for (int i = 0; i < WANB200_MAX_PEERS; ++i) {
    a.flags[i] = i < world ? flags[i] : flags[0];
    if (i < world && (!flags[i] || (reinterpret_cast<uintptr_t>(flags[i]) & 3)))
      return set_error(WANB200_EINVAL, "peer_barrier: flag pointers must be non-null and 4-byte aligned");
  }
  a.rank = rank;
  a.world = world;
  a.epoch = epoch;
  a.err = device_error_word();
  if (!a.err) return WANB200_ECUDA;
  peer_barrier_kernel<<<1, 32, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("peer_barrier_kernel launch", e);
  return WANB200_OK;
}

}  // namespace wanb200
