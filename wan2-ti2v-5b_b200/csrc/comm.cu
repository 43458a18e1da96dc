// Collectives over NVLink peer memory.
//  * peer_barrier: a barrier of the ranks of a group.  The reduce-scatter fused into the
//    row-parallel GEMM epilogue, the all-gather fused into the LayerNorm and the shard gather
//    below store straight into peer buffers; this barrier separates those producers from the
//    kernels that read the results.
//  * shard_gather: the K/V all-gather of sequence-parallel self-attention, pushed by the owner
//    of each shard into every rank's gathered buffer.
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

struct GatherArgs {
  const __nv_bfloat16* src;
  int64_t src_ld, shard_rows, valid_rows, rows;  // rows = batch * valid_rows
  int vecs;                                     // 16-byte vectors per row (width / 8)
  __nv_bfloat16* dst[WANB200_MAX_PEERS];
  int64_t dst_row0[WANB200_MAX_PEERS];
  int64_t dst_ld, dst_batch_stride;
};

// One warp per (row, destination): blockIdx.y picks the destination, the warp's row is one of
// the batch * valid_rows rows of the shard.  Lanes move consecutive 16-byte vectors, so every
// store instruction of the warp writes 512 contiguous bytes of the peer's row.  CTAs of 4 warps
// at no more than 32 registers a thread (4096 registers): the push runs on a side stream while the
// local attention holds every SM with one CTA of 384 threads x 160 registers at launch, and a
// push CTA has to fit in the registers left beside it, or the push only starts once the
// attention's CTAs have exited.
__global__ void __launch_bounds__(128, 16) shard_gather_kernel(const GatherArgs a) {
  const int64_t r = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (r >= a.rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t b = r / a.valid_rows, i = r - b * a.valid_rows;
  __nv_bfloat16* dst = a.dst[blockIdx.y];  // a uniform, constant-bank read (blockIdx.y < ndst)
  const int64_t row0 = a.dst_row0[blockIdx.y];
  const uint4* s = reinterpret_cast<const uint4*>(a.src + (b * a.shard_rows + i) * a.src_ld);
  uint4* d = reinterpret_cast<uint4*>(dst + b * a.dst_batch_stride + (row0 + i) * a.dst_ld);
  const int nv = a.vecs;
  int v = lane;
  for (; v + 32 < nv; v += 64) {  // two 512-byte segments of the row in flight per warp
    const uint4 x0 = s[v], x1 = s[v + 32];
    d[v] = x0;
    d[v + 32] = x1;
  }
  if (v < nv) d[v] = s[v];
}

int shard_gather(const wanb200_shard_gather_params* p, cudaStream_t st) {
  if (!p || !p->src || p->batch <= 0 || p->shard_rows <= 0 || p->valid_rows < 0 || p->valid_rows > p->shard_rows ||
      p->width <= 0 || p->width % 8 || p->src_ld < p->width || p->src_ld % 8 || p->dst_ld < p->width || p->dst_ld % 8 ||
      p->dst_batch_stride % 8 || p->ndst < 1 || p->ndst > WANB200_MAX_PEERS)
    return set_error(WANB200_EINVAL, "shard_gather: need src, batch > 0, 0 <= valid_rows <= shard_rows, width % 8 == 0, "
                                     "src_ld/dst_ld >= width and % 8 == 0, dst_batch_stride % 8 == 0, "
                                     "1 <= ndst <= 8");
  for (int k = 0; k < p->ndst; ++k) {
    if (p->dst_row0[k] < 0) return set_error(WANB200_EINVAL, "shard_gather: dst_row0 must be >= 0");
    if (p->batch > 1 && p->dst_batch_stride < (p->dst_row0[k] + p->valid_rows) * p->dst_ld)
      return set_error(WANB200_EINVAL, "shard_gather: dst_batch_stride smaller than the rows of one batch element");
  }
  if (!aligned16(p->src)) return set_error(WANB200_EINVAL, "shard_gather: src must be 16-byte aligned");
  GatherArgs a;
  for (int k = 0; k < WANB200_MAX_PEERS; ++k) {
    a.dst[k] = reinterpret_cast<__nv_bfloat16*>(k < p->ndst ? p->dst[k] : p->dst[0]);
    a.dst_row0[k] = k < p->ndst ? p->dst_row0[k] : p->dst_row0[0];
    if (k < p->ndst && (!p->dst[k] || !aligned16(p->dst[k])))
      return set_error(WANB200_EINVAL, "shard_gather: destinations must be non-null and 16-byte aligned");
  }
  if (p->valid_rows == 0) return WANB200_OK;
  a.src = reinterpret_cast<const __nv_bfloat16*>(p->src);
  a.src_ld = p->src_ld;
  a.shard_rows = p->shard_rows;
  a.valid_rows = p->valid_rows;
  a.rows = p->batch * p->valid_rows;
  a.vecs = (int)(p->width / 8);
  a.dst_ld = p->dst_ld;
  a.dst_batch_stride = p->dst_batch_stride;
  const int64_t blocks = (a.rows + 3) / 4;  // 4 rows (warps) per CTA
  if (blocks > INT32_MAX || p->width / 8 > INT32_MAX) return set_error(WANB200_EINVAL, "shard_gather: too large");
  shard_gather_kernel<<<dim3((unsigned)blocks, (unsigned)p->ndst), 128, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("shard_gather_kernel launch", e);
  return WANB200_OK;
}

}  // namespace wanb200
