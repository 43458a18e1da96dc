// The extern "C" surface of libwanb200.so (declared in include/wanb200.h) and the host-side
// services the launchers share: error strings, the per-device error word, SM counts and TMA
// descriptor encoding (through the driver entry point, so the library needs no -lcuda).
#include <mutex>
#include <string>

#include "internal.h"

namespace wanb200 {

static thread_local std::string t_last_error;

int set_error(int code, const char* msg) {
  t_last_error = msg;
  return code;
}

int set_cuda_error(const char* what, cudaError_t e) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return WANB200_ECUDA;
}

static std::mutex g_mu;
// The error word lives in the library image: a file-scope __device__ int of which every device
// that loads the library holds its own zero-initialised copy, so no entry point allocates for it.
// Host code cannot use the symbol's name as an address; the device address is resolved once per
// device (cudaGetSymbolAddress, with that device current) and cached here.
static __device__ int g_err_dev_word;
static int* g_err_word[kMaxDevices] = {};
static int g_num_sms[kMaxDevices] = {};

int* device_error_word() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error("cudaGetDevice", e);
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error(WANB200_EINVAL, "device index out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_word[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_err_dev_word);
    if (e != cudaSuccess) {
      set_cuda_error("cudaGetSymbolAddress(error word)", e);
      return nullptr;
    }
    g_err_word[dev] = static_cast<int*>(p);
  }
  return g_err_word[dev];
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (!g_num_sms[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_num_sms[dev] = n;
  }
  return g_num_sms[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static int encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                  const cuuint32_t* box, CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(WANB200_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(m, dtype, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_error = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r);
    return WANB200_EINVAL;
  }
  return WANB200_OK;
}

int make_tmap_2d(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                 int box_outer) {
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  const cuuint64_t str[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  return encode(m, base, 2, dims, str, box);
}

int make_tmap_4d(CUtensorMap* m, const void* base, const int64_t dims[4], const int64_t strides[4], const int box[4]) {
  const cuuint64_t d[4] = {(cuuint64_t)dims[0], (cuuint64_t)dims[1], (cuuint64_t)dims[2], (cuuint64_t)dims[3]};
  const cuuint64_t s[3] = {(cuuint64_t)strides[1] * 2, (cuuint64_t)strides[2] * 2, (cuuint64_t)strides[3] * 2};
  const cuuint32_t b[4] = {(cuuint32_t)box[0], (cuuint32_t)box[1], (cuuint32_t)box[2], (cuuint32_t)box[3]};
  return encode(m, base, 4, d, s, b);
}

int make_tmap_4d_u8(CUtensorMap* m, const void* base, const int64_t dims[4], const int64_t strides[4],
                    const int box[4]) {
  const cuuint64_t d[4] = {(cuuint64_t)dims[0], (cuuint64_t)dims[1], (cuuint64_t)dims[2], (cuuint64_t)dims[3]};
  const cuuint64_t s[3] = {(cuuint64_t)strides[1], (cuuint64_t)strides[2], (cuuint64_t)strides[3]};
  const cuuint32_t b[4] = {(cuuint32_t)box[0], (cuuint32_t)box[1], (cuuint32_t)box[2], (cuuint32_t)box[3]};
  return encode(m, base, 4, d, s, b, CU_TENSOR_MAP_DATA_TYPE_UINT8);
}

}  // namespace wanb200

using namespace wanb200;

extern "C" {

int wanb200_gemm_bf16(const wanb200_gemm_params* p, void* stream) {
  return gemm_bf16(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_attn_fwd(const wanb200_attn_params* p, void* stream) {
  return attn_fwd(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_attn_fwd_noalloc(const wanb200_attn_params* p, void* stream) {
  return attn_fwd_noalloc(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_attn_fwd_fp8(const wanb200_attn_fp8_params* p, void* stream) {
  return attn_fwd_fp8(p, reinterpret_cast<cudaStream_t>(stream));
}

int64_t wanb200_attn_fp8_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len) {
  return attn_fp8_workspace_bytes(batch, heads, q_len, kv_len);
}

int64_t wanb200_attn_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int kv_splits) {
  return attn_workspace_bytes(batch, heads, q_len, kv_splits);
}

int wanb200_attn_kv_splits(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len) {
  return attn_kv_splits(batch, heads, q_len, kv_len);
}

int wanb200_layernorm(const wanb200_ln_params* p, void* stream) {
  return layernorm(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_qk_norm_rope(const wanb200_qknorm_params* p, void* stream) {
  return qk_norm_rope(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_sumsq_reduce(const wanb200_sumsq_reduce_params* p, void* stream) {
  return sumsq_reduce(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_bias_gate_residual(const wanb200_residual_params* p, void* stream) {
  return bias_gate_residual(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_peer_barrier(int* const* flags, int rank, int world, int epoch, void* stream) {
  return peer_barrier(flags, rank, world, epoch, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_shard_gather(const wanb200_shard_gather_params* p, void* stream) {
  return shard_gather(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_patchify(const wanb200_patchify_params* p, void* stream) {
  return patchify(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_unpatchify_cfg(const wanb200_unpatchify_params* p, void* stream) {
  return unpatchify_cfg(p, reinterpret_cast<cudaStream_t>(stream));
}

int wanb200_block_forward(const wanb200_block_params* p, void* stream) {
  return block_forward(p, reinterpret_cast<cudaStream_t>(stream));
}

int64_t wanb200_block_workspace_bytes(int64_t batch, int64_t seq_len, int64_t dim, int64_t local_heads,
                                      int64_t ffn_local, int64_t ctx_len, int tp_size) {
  return block_workspace_bytes(batch, seq_len, dim, local_heads, ffn_local, ctx_len, tp_size);
}

const char* wanb200_last_error(void) { return t_last_error.c_str(); }

int wanb200_device_error(int reset) {
  int* w = device_error_word();
  if (!w) return WANB200_ECUDA;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_cuda_error("cudaDeviceSynchronize", e);
  int v = 0;
  e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_cuda_error("cudaMemcpy(error word)", e);
  if (reset && v) {
    e = cudaMemset(w, 0, sizeof(int));
    if (e != cudaSuccess) return set_cuda_error("cudaMemset(error word)", e);
  }
  return v;
}

int wanb200_device_error_async(int* host_out, void* stream) {
  if (!host_out) return set_error(WANB200_EINVAL, "device_error_async: null host_out");
  int* w = device_error_word();
  if (!w) return WANB200_ECUDA;
  cudaError_t e = cudaMemcpyAsync(host_out, w, sizeof(int), cudaMemcpyDeviceToHost, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_cuda_error("cudaMemcpyAsync(error word)", e);
  return WANB200_OK;
}

int wanb200_version(void) { return 201; }

int wanb200_struct_sizes(int64_t* out, int n) {
  const int64_t sizes[11] = {(int64_t)sizeof(wanb200_gemm_params), (int64_t)sizeof(wanb200_attn_params),
                             (int64_t)sizeof(wanb200_ln_params), (int64_t)sizeof(wanb200_qknorm_params),
                             (int64_t)sizeof(wanb200_residual_params), (int64_t)sizeof(wanb200_shard_gather_params),
                             (int64_t)sizeof(wanb200_attn_fp8_params), (int64_t)sizeof(wanb200_block_params),
                             (int64_t)sizeof(wanb200_patchify_params), (int64_t)sizeof(wanb200_unpatchify_params),
                             (int64_t)sizeof(wanb200_sumsq_reduce_params)};
  for (int i = 0; i < n && i < 11; ++i) out[i] = sizes[i];
  return 11;
}

}  // extern "C"
