// Host-side helpers shared by the launchers (not part of the public C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "../../include/wanb200.h"

namespace wanb200 {

constexpr int kMaxDevices = 64;

// Record a message for wanb200_last_error() and return `code`.
int set_error(int code, const char* msg);
int set_cuda_error(const char* what, cudaError_t e);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device address of the current device's error word, the int that kernels write error codes
// into (a __device__ variable of the library, resolved once per device; allocates nothing;
// nullptr + last error set on failure).
int* device_error_word();
int num_sms();

// 2-D / 4-D bf16 TMA descriptors with 128-byte swizzle and zero fill out of bounds.
//   2-D: dims {inner, outer}, row stride `ld` elements, box {box_inner, box_outer}.
//   4-D: dims d[0..3] (d[0] innermost, contiguous), strides s[1..3] in elements, box b[0..3].
int make_tmap_2d(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                 int box_outer);
int make_tmap_4d(CUtensorMap* m, const void* base, const int64_t dims[4], const int64_t strides[4],
                 const int box[4]);
// The same for 8-bit elements (fp8 e4m3 tiles): strides in bytes.
int make_tmap_4d_u8(CUtensorMap* m, const void* base, const int64_t dims[4], const int64_t strides[4],
                    const int box[4]);

// Launchers (one per public entry point).
int gemm_bf16(const wanb200_gemm_params* p, cudaStream_t st);
int attn_fwd(const wanb200_attn_params* p, cudaStream_t st);
// e4m3 operands of the attention (quantised by attn_fwd_fp8)
struct AttnFp8Operands {
  const void* q8;   // [B, q_len, H, 128]
  const void* k8;   // [B, kv_len, H, 128]
  const void* v8t;  // [B, H, 128, kv_len16]
  const float* q_scale;  // [B, H, ceil(q_len / 128)]
  const float* k_scale;  // [B, H, ceil(kv_len / 128)]
  const float* v_scale;  // [B, H]
  int64_t kv_len16;
};
int attn_launch(const wanb200_attn_params* p, int* err, cudaStream_t st,
                const AttnFp8Operands* f8 = nullptr);  // validated params
int attn_fwd_fp8(const wanb200_attn_fp8_params* p, cudaStream_t st);
int64_t attn_fp8_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len);
int attn_fwd_noalloc(const wanb200_attn_params* p, cudaStream_t st);
int64_t attn_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int kv_splits);
int attn_kv_splits(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len);
int layernorm(const wanb200_ln_params* p, cudaStream_t st);
int qk_norm_rope(const wanb200_qknorm_params* p, cudaStream_t st);
int sumsq_reduce(const wanb200_sumsq_reduce_params* p, cudaStream_t st);
int bias_gate_residual(const wanb200_residual_params* p, cudaStream_t st);
int peer_barrier(int* const* flags, int rank, int world, int epoch, cudaStream_t st);
int shard_gather(const wanb200_shard_gather_params* p, cudaStream_t st);
int block_forward(const wanb200_block_params* p, cudaStream_t st);
int patchify(const wanb200_patchify_params* p, cudaStream_t st);
int unpatchify_cfg(const wanb200_unpatchify_params* p, cudaStream_t st);
int64_t block_workspace_bytes(int64_t batch, int64_t seq_len, int64_t dim, int64_t local_heads, int64_t ffn_local,
                              int64_t ctx_len, int tp_size);

}  // namespace wanb200
