// HBM-bound kernels of the block: LayerNorm (+ per-frame AdaLN modulation) and the
// QK-RMSNorm + 3-D RoPE pass.  Both are vectorised 16-byte loads/stores, fp32 math, one
// rounding to bf16 on the way out.
#include "common.cuh"
#include "internal.h"

namespace wanb200 {

constexpr int LN_MAX_VEC = 16;  // dim <= 16 * 256 = 4096

struct LnArgs {
  const void* x;  // bf16, or fp32 (XF32: the fp32 residual stream)
  __nv_bfloat16* out;
  int64_t rows;
  int dim;
  float eps;
  const __nv_bfloat16* modulation;
  const float* e0;
  int64_t e0_frame_stride;
  int shift_idx, scale_idx;
  int64_t seq_len, tokens_per_frame, row_offset, rows_per_seq;
  const __nv_bfloat16* weight;
  const __nv_bfloat16* bias;
  __nv_bfloat16* push_out[WANB200_MAX_PEERS];
  int npush;
  int64_t push_row0;
  int e0_one_row;
};

// RW warps per row (4 when dim % 1024 == 0, 2 when dim % 512 == 0, else 1): thread t < 32*RW of the row holds the
// 16-byte vectors at columns (i*32*RW + t)*8, i < NVEC = dim / (256*RW); the row statistics are
// reduced over the row's warps through shared memory.  The grid is 4 blocks per SM (at most 64
// registers a thread) and every warp group walks rows with a grid stride; the 32 warps per SM keep
// 8 rows in flight to HBM (a next-row prefetch into a second register buffer held only 16 warps
// per SM at 128 registers and was 3-7% slower); the warps of a row synchronise with their own
// named barrier, never with the rest of the block.  x is loaded and the output stored
// with the streaming cache hint, so the L1 keeps the frame's modulation rows that every row of the
// frame re-reads (7% faster than default caching at config 2).
//   MODE 0 (modulate): WanLayerNorm without affine (wan/modules/model.py:89-99), then
//     `_modulate` (models/fast_dit.py:172-176): y * (1 + scale[f]) + shift[f] with
//     shift/scale[f, c] = modulation[idx, c] + e0[f, idx, c] (fast_dit.py:276-277).
//   MODE 1 (affine): norm3 = WanLayerNorm(elementwise_affine=True) (model.py:207-209).
//   XF32: x is fp32 (the residual stream kept in fp32 across the step); the output stays bf16.
constexpr int LN_BLOCKS_PER_SM = 4;

template <int MODE, int NVEC, bool PUSH, int RW, bool XF32>
__global__ void __launch_bounds__(256, LN_BLOCKS_PER_SM) layernorm_kernel(const LnArgs a) {
  __shared__ float red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int RPB = 8 / RW;  // rows per block per pass
  constexpr int W = XF32 ? 2 : 1;  // 16-byte words per 8 values: bf16 1, fp32 2
  const int t = (warp % RW) * 32 + lane;
  const int64_t stride = (int64_t)gridDim.x * RPB;
  int64_t row = (int64_t)blockIdx.x * RPB + warp / RW;
  auto load = [&](int64_t r, uint4 (&v)[NVEC * W]) {
    const uint4* xr =
        reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) + r * a.dim * (XF32 ? 4 : 2));
#pragma unroll
    for (int i = 0; i < NVEC; ++i)
#pragma unroll
      for (int w = 0; w < W; ++w) v[i * W + w] = __ldcs(xr + (i * 32 * RW + t) * W + w);  // streamed once
  };
  auto values = [](const uint4 (&v)[NVEC * W], int i, float* x) {  // the 8 values of vector i as fp32
    if constexpr (XF32) {
      const uint4 lo = v[2 * i], hi = v[2 * i + 1];
      x[0] = __uint_as_float(lo.x); x[1] = __uint_as_float(lo.y); x[2] = __uint_as_float(lo.z); x[3] = __uint_as_float(lo.w);
      x[4] = __uint_as_float(hi.x); x[5] = __uint_as_float(hi.y); x[6] = __uint_as_float(hi.z); x[7] = __uint_as_float(hi.w);
    } else {
      unpack_bf16x8(v[i], x);
    }
  };
  auto row_sum = [&](float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if constexpr (RW == 1) return v;
    if (lane == 0) red[warp] = v;
    asm volatile("bar.sync %0, %1;" ::"r"(1 + warp / RW), "r"(32 * RW) : "memory");  // this row's warps
    const int g0 = warp - warp % RW;
    float tot = red[g0];
#pragma unroll
    for (int k = 1; k < RW; ++k) tot += red[g0 + k];
    asm volatile("bar.sync %0, %1;" ::"r"(1 + warp / RW), "r"(32 * RW) : "memory");  // red is reused next
    return tot;
  };
  if (row >= a.rows) return;  // uniform over a row's warps: they walk the same rows
  uint4 xv[NVEC * W];
  for (;; row += stride) {
    const bool more = row + stride < a.rows;
    load(row, xv);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < NVEC; ++i) {
      float x[8];
      values(xv, i, x);
#pragma unroll
      for (int k = 0; k < 8; ++k) sum += x[k];
    }
    const float mean = row_sum(sum) / a.dim;
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < NVEC; ++i) {
      float x[8];
      values(xv, i, x);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float d = x[k] - mean;
        var = fmaf(d, d, var);
      }
    }
    const float rstd = rsqrtf(row_sum(var) / a.dim + a.eps);

    const float* shp = nullptr;
    const float* scp = nullptr;
    if constexpr (MODE == 0) {
      const int64_t f = frame_of_row(row, a.rows_per_seq, a.row_offset, a.seq_len, a.tokens_per_frame);
      shp = a.e0 + f * a.e0_frame_stride + (a.e0_one_row ? 0 : (int64_t)a.shift_idx * a.dim);
      scp = a.e0 + f * a.e0_frame_stride + (a.e0_one_row ? 0 : (int64_t)a.scale_idx * a.dim);
    }
    uint4* outr = a.out ? reinterpret_cast<uint4*>(a.out + row * a.dim) : nullptr;
#pragma unroll
    for (int i = 0; i < NVEC; ++i) {
      const int v = i * 32 * RW + t;
      const int col = v * 8;
      float x[8], y[8];
      values(xv, i, x);
      if constexpr (MODE == 0) {
        float ms[8], mc[8];
        unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(a.modulation + (int64_t)a.shift_idx * a.dim + col)), ms);
        unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(a.modulation + (int64_t)a.scale_idx * a.dim + col)), mc);
        const float4 s0 = __ldg(reinterpret_cast<const float4*>(shp + col));
        const float4 s1 = __ldg(reinterpret_cast<const float4*>(shp + col + 4));
        const float4 c0 = __ldg(reinterpret_cast<const float4*>(scp + col));
        const float4 c1 = __ldg(reinterpret_cast<const float4*>(scp + col + 4));
        const float sh[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const float sc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) y[k] = fmaf((x[k] - mean) * rstd, 1.f + (mc[k] + sc[k]), ms[k] + sh[k]);
      } else {
        float w[8], bb[8];
        unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(a.weight + col)), w);
        unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(a.bias + col)), bb);
#pragma unroll
        for (int k = 0; k < 8; ++k) y[k] = fmaf((x[k] - mean) * rstd, w[k], bb[k]);
      }
      uint4 u;
      u.x = pack_bf16x2(y[0], y[1]);
      u.y = pack_bf16x2(y[2], y[3]);
      u.z = pack_bf16x2(y[4], y[5]);
      u.w = pack_bf16x2(y[6], y[7]);
      if (!PUSH || outr) __stcs(outr + v, u);
#pragma unroll
      for (int p = 0; p < (PUSH ? WANB200_MAX_PEERS : 0); ++p)  // all-gather fused into the norm: push the row to every rank
        if (p < a.npush) reinterpret_cast<uint4*>(a.push_out[p] + (a.push_row0 + row) * a.dim)[v] = u;
    }
    if (!more) break;
  }
}

template <int MODE, bool PUSH, bool XF32>
static void launch_ln(int dim, const LnArgs& a, int64_t rows, cudaStream_t st) {
  const int64_t resident = (int64_t)num_sms() * LN_BLOCKS_PER_SM;
  if (dim % 1024 == 0) {  // four warps per row, 2 rows per block pass
    const unsigned blocks = (unsigned)std::min<int64_t>((rows + 1) / 2, resident);
    switch (dim / 1024) {
      case 1: layernorm_kernel<MODE, 1, PUSH, 4, XF32><<<blocks, 256, 0, st>>>(a); break;
      case 2: layernorm_kernel<MODE, 2, PUSH, 4, XF32><<<blocks, 256, 0, st>>>(a); break;
      case 3: layernorm_kernel<MODE, 3, PUSH, 4, XF32><<<blocks, 256, 0, st>>>(a); break;
      default: layernorm_kernel<MODE, 4, PUSH, 4, XF32><<<blocks, 256, 0, st>>>(a); break;
    }
    return;
  }
  if (dim % 512 == 0) {  // two warps per row, 4 rows per block pass
    const unsigned blocks = (unsigned)std::min<int64_t>((rows + 3) / 4, resident);
    switch (dim / 512) {
#define WANB200_LN_CASE2(n) \
  case n: layernorm_kernel<MODE, n, PUSH, 2, XF32><<<blocks, 256, 0, st>>>(a); break;
      WANB200_LN_CASE2(1) WANB200_LN_CASE2(3) WANB200_LN_CASE2(5)
      default: layernorm_kernel<MODE, 7, PUSH, 2, XF32><<<blocks, 256, 0, st>>>(a); break;
#undef WANB200_LN_CASE2
    }
    return;
  }
  const unsigned blocks = (unsigned)std::min<int64_t>((rows + 7) / 8, resident);
  switch (dim / 256) {
#define WANB200_LN_CASE(n) \
  case n: layernorm_kernel<MODE, n, PUSH, 1, XF32><<<blocks, 256, 0, st>>>(a); break;
    WANB200_LN_CASE(1) WANB200_LN_CASE(3) WANB200_LN_CASE(5) WANB200_LN_CASE(7) WANB200_LN_CASE(9)
    WANB200_LN_CASE(11) WANB200_LN_CASE(13)
    default: layernorm_kernel<MODE, 15, PUSH, 1, XF32><<<blocks, 256, 0, st>>>(a); break;
#undef WANB200_LN_CASE
  }
}

template <int MODE, bool PUSH>
static void launch_ln(int dim, const LnArgs& a, int64_t rows, bool xf32, cudaStream_t st) {
  if (xf32)
    launch_ln<MODE, PUSH, true>(dim, a, rows, st);
  else
    launch_ln<MODE, PUSH, false>(dim, a, rows, st);
}

int layernorm(const wanb200_ln_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "layernorm: null params");
  if (!p->x || (!p->out && p->npush <= 0)) return set_error(WANB200_EINVAL, "layernorm: null x/out");
  if (p->npush < 0 || p->npush > WANB200_MAX_PEERS || p->push_row0 < 0)
    return set_error(WANB200_EINVAL, "layernorm: npush must be 0..8 and push_row0 >= 0");
  for (int i = 0; i < p->npush; ++i)
    if (!p->push_out[i] || !aligned16(p->push_out[i]))
      return set_error(WANB200_EINVAL, "layernorm: push_out pointers must be non-null and 16-byte aligned");
  if (p->rows <= 0 || p->dim <= 0 || p->dim % 256 || p->dim > 256 * LN_MAX_VEC)
    return set_error(WANB200_EINVAL, "layernorm: dim must be a positive multiple of 256, at most 4096");
  if (!aligned16(p->x) || !aligned16(p->out)) return set_error(WANB200_EINVAL, "layernorm: x/out must be 16-byte aligned");
  if (p->mode == WANB200_LN_MODULATE) {
    if (!p->modulation || !p->e0 || !aligned16(p->modulation) || !aligned16(p->e0) || p->e0_frame_stride % 4 ||
        p->shift_idx < 0 || p->shift_idx > 5 || p->scale_idx < 0 || p->scale_idx > 5 || p->seq_len <= 0 ||
        p->tokens_per_frame <= 0 || p->row_offset < 0 || p->rows_per_seq < 0)
      return set_error(WANB200_EINVAL, "layernorm: modulate mode needs modulation, e0, indices, seq_len, tokens_per_frame "
                                       "(row_offset, rows_per_seq >= 0)");
  } else if (p->mode == WANB200_LN_AFFINE) {
    if (!p->weight || !p->bias || !aligned16(p->weight) || !aligned16(p->bias))
      return set_error(WANB200_EINVAL, "layernorm: affine mode needs 16-byte aligned weight and bias");
  } else {
    return set_error(WANB200_EINVAL, "layernorm: bad mode");
  }
  LnArgs a;
  a.x = p->x;
  a.out = reinterpret_cast<__nv_bfloat16*>(p->out);
  a.rows = p->rows;
  a.dim = (int)p->dim;
  a.eps = p->eps;
  a.modulation = reinterpret_cast<const __nv_bfloat16*>(p->modulation);
  a.e0 = p->e0;
  a.e0_frame_stride = p->e0_frame_stride;
  a.shift_idx = p->shift_idx;
  a.scale_idx = p->scale_idx;
  a.seq_len = p->seq_len > 0 ? p->seq_len : 1;
  a.tokens_per_frame = p->tokens_per_frame > 0 ? p->tokens_per_frame : 1;
  a.row_offset = p->row_offset;
  a.rows_per_seq = p->rows_per_seq;
  a.weight = reinterpret_cast<const __nv_bfloat16*>(p->weight);
  a.bias = reinterpret_cast<const __nv_bfloat16*>(p->bias);
  for (int i = 0; i < WANB200_MAX_PEERS; ++i)
    a.push_out[i] = reinterpret_cast<__nv_bfloat16*>(i < p->npush ? p->push_out[i] : nullptr);
  a.npush = p->npush;
  a.push_row0 = p->push_row0;
  a.e0_one_row = p->e0_one_row != 0;
  if ((p->rows + 3) / 4 > INT32_MAX) return set_error(WANB200_EINVAL, "layernorm: too many rows");
  const bool push = a.npush > 0, xf32 = p->x_f32 != 0;
  if (p->mode == WANB200_LN_MODULATE)
    push ? launch_ln<0, true>(a.dim, a, p->rows, xf32, st) : launch_ln<0, false>(a.dim, a, p->rows, xf32, st);
  else
    push ? launch_ln<1, true>(a.dim, a, p->rows, xf32, st) : launch_ln<1, false>(a.dim, a, p->rows, xf32, st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("layernorm_kernel launch", e);
  return WANB200_OK;
}

// ------------------------------------------------------------------ QK RMSNorm + RoPE
struct QkArgs {
  __nv_bfloat16* x;
  int64_t ld, rows;
  int64_t col0[2];
  int width;
  const float* ss[2];
  int self_ss;  // ss[] == NULL: the sums of squares are formed from the sections' own values
  int ss_parts;
  int64_t ss_row_stride;
  const __nv_bfloat16* gamma[2];
  float inv_dim, eps;
  int rope;
  const float* cos;
  const float* sin;
  int seq_len;
};

// One warp per (row, section): lane l holds the 16-byte vectors l, l + 32, ... (NV of them, 8
// channels = 4 rotation pairs each) of one section of one row (q or k of self-attention, cross q
// alone), so the section's loads are all in flight at once and its sum of squares is a warp
// butterfly -- no block barrier; with one section per warp a thread needs few enough registers
// for several blocks per SM, whose load and store phases then overlap.
// `_tp_rms_qk` (models/fast_dit.py:134-147): x * rsqrt(ss/3072 + eps) * gamma, then `_rope`
// (fast_dit.py:163-169): (x0, x1) -> (x0 c - x1 s, x0 s + x1 c) with the pair's angle.  The sum
// of squares is either formed from the section's own bf16 values (ss[s] == NULL: the section is
// the whole global dim, one GPU; the squares of the rounded values, as `q.float().pow(2).sum(-1)`),
// or added from ss_parts partials per row (a SUMSQ GEMM's 32-column chunks), or read as one
// finished sum; each lane adds its share in order, then the butterfly -- the same order on every
// run.
template <int NV>
__global__ void __launch_bounds__(256, 2) qknorm_rope_kernel(const QkArgs a, int nsec) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);  // (row, section) of this warp
  const int row = nsec == 2 ? gw >> 1 : gw, sec = nsec == 2 ? gw & 1 : 0;
  if (row >= a.rows) return;  // warp-uniform
  const int vpr = a.width >> 3;
  __nv_bfloat16* xs = a.x + (int64_t)row * a.ld + (sec ? a.col0[1] : a.col0[0]);
  const float* ss = sec ? a.ss[1] : a.ss[0];
  const __nv_bfloat16* gamma = sec ? a.gamma[1] : a.gamma[0];
  uint4 raw[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = i * 32 + lane;
    raw[i] = v < vpr ? reinterpret_cast<const uint4*>(xs)[v] : make_uint4(0u, 0u, 0u, 0u);
  }
  float q = 0.f;
  if (a.self_ss) {  // grid-uniform branches
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float v[8];
      unpack_bf16x8(raw[i], v);
#pragma unroll
      for (int k = 0; k < 8; ++k) q = fmaf(v[k], v[k], q);
    }
  } else if (a.ss_parts > 1) {
    for (int k = lane; k < a.ss_parts; k += 32) q += __ldg(ss + (int64_t)row * a.ss_row_stride + k);
  } else if (lane == 0) {
    q = __ldg(ss + (int64_t)row * a.ss_row_stride);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rs = rsqrtf(q * a.inv_dim + a.eps);
  const int pos = a.rope ? row % a.seq_len : 0;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = i * 32 + lane;
    if (v >= vpr) break;
    const int cv = v * 8;
    float x[8], g[8];
    unpack_bf16x8(raw[i], x);
    unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(gamma + cv)), g);
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] *= rs * g[k];
    if (a.rope) {
      const int pair0 = (cv & 127) >> 1;
      const float4 c4 = __ldg(reinterpret_cast<const float4*>(a.cos + (int64_t)pos * 64 + pair0));
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(a.sin + (int64_t)pos * 64 + pair0));
      float x0, x1;
      x0 = x[0]; x1 = x[1]; x[0] = x0 * c4.x - x1 * s4.x; x[1] = x0 * s4.x + x1 * c4.x;
      x0 = x[2]; x1 = x[3]; x[2] = x0 * c4.y - x1 * s4.y; x[3] = x0 * s4.y + x1 * c4.y;
      x0 = x[4]; x1 = x[5]; x[4] = x0 * c4.z - x1 * s4.z; x[5] = x0 * s4.z + x1 * c4.z;
      x0 = x[6]; x1 = x[7]; x[6] = x0 * c4.w - x1 * s4.w; x[7] = x0 * s4.w + x1 * c4.w;
    }
    uint4 u;
    u.x = pack_bf16x2(x[0], x[1]);
    u.y = pack_bf16x2(x[2], x[3]);
    u.z = pack_bf16x2(x[4], x[5]);
    u.w = pack_bf16x2(x[6], x[7]);
    reinterpret_cast<uint4*>(xs)[v] = u;
  }
}

static void launch_qknorm(const QkArgs& a, int nsec, int nv, unsigned blocks, cudaStream_t st) {
  switch (nv) {
    case 1: qknorm_rope_kernel<1><<<blocks, 256, 0, st>>>(a, nsec); break;
    case 2: qknorm_rope_kernel<2><<<blocks, 256, 0, st>>>(a, nsec); break;
    case 3: qknorm_rope_kernel<3><<<blocks, 256, 0, st>>>(a, nsec); break;
    case 4: qknorm_rope_kernel<4><<<blocks, 256, 0, st>>>(a, nsec); break;
    case 6: qknorm_rope_kernel<6><<<blocks, 256, 0, st>>>(a, nsec); break;
    case 8: qknorm_rope_kernel<8><<<blocks, 256, 0, st>>>(a, nsec); break;
    case 12: qknorm_rope_kernel<12><<<blocks, 256, 0, st>>>(a, nsec); break;
    default: qknorm_rope_kernel<16><<<blocks, 256, 0, st>>>(a, nsec); break;
  }
}

// Block shape of the row-streaming kernels: x = the row's 16-byte vectors (rounded up to a warp,
// at most 1024), y = rows per block (about 256 threads, at least one row).
static dim3 row_block(int64_t vecs_per_row) {
  const int bx = (int)std::min<int64_t>(1024, (vecs_per_row + 31) / 32 * 32);
  return dim3(bx, std::max(1, 256 / bx));
}

int qk_norm_rope(const wanb200_qknorm_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "qk_norm_rope: null params");
  if (!p->x || p->rows <= 0 || p->width <= 0 || p->width % 128 || p->ld % 8 || p->ld <= 0)
    return set_error(WANB200_EINVAL, "qk_norm_rope: need x, rows > 0, width % 128 == 0, ld % 8 == 0");
  if (p->nsections < 1 || p->nsections > 2) return set_error(WANB200_EINVAL, "qk_norm_rope: nsections must be 1 or 2");
  if (!aligned16(p->x)) return set_error(WANB200_EINVAL, "qk_norm_rope: x must be 16-byte aligned");
  for (int s = 0; s < p->nsections; ++s) {
    if ((!p->ss[s]) != (!p->ss[0]) || !p->gamma[s] || !aligned16(p->gamma[s]) || p->col0[s] < 0 || p->col0[s] % 8 ||
        p->col0[s] + p->width > p->ld)
      return set_error(WANB200_EINVAL, "qk_norm_rope: bad section (ss, gamma, col0)");
  }
  if (p->rope && (!p->cos || !p->sin || !aligned16(p->cos) || !aligned16(p->sin) || p->seq_len <= 0))
    return set_error(WANB200_EINVAL, "qk_norm_rope: rope needs 16-byte aligned cos/sin tables and seq_len");
  QkArgs a;
  a.x = reinterpret_cast<__nv_bfloat16*>(p->x);
  a.ld = p->ld;
  a.rows = p->rows;
  a.col0[0] = p->col0[0];
  a.col0[1] = p->col0[1];
  a.width = (int)p->width;
  a.ss[0] = p->ss[0];
  a.ss[1] = p->ss[1];
  a.self_ss = p->ss[0] == nullptr;
  a.ss_parts = p->ss_parts > 0 ? p->ss_parts : 1;
  a.ss_row_stride = p->ss_row_stride > 0 ? p->ss_row_stride : 1;
  if (a.ss_parts > p->width / 8 || a.ss_row_stride < a.ss_parts)
    return set_error(WANB200_EINVAL, "qk_norm_rope: ss_parts must be <= width / 8 and <= ss_row_stride");
  a.gamma[0] = reinterpret_cast<const __nv_bfloat16*>(p->gamma[0]);
  a.gamma[1] = reinterpret_cast<const __nv_bfloat16*>(p->gamma[1]);
  a.inv_dim = p->inv_dim;
  a.eps = p->eps;
  a.rope = p->rope;
  a.cos = p->cos;
  a.sin = p->sin;
  if (p->seq_len > INT32_MAX) return set_error(WANB200_EINVAL, "qk_norm_rope: seq_len too large");
  a.seq_len = p->seq_len > 0 ? (int)p->seq_len : 1;
  if (p->rows > INT32_MAX / 2 || p->width > 4096)
    return set_error(WANB200_EINVAL, "qk_norm_rope: rows < 2^30, width <= 4096");
  // vectors per lane, rounded up to an instantiated count
  int nv = (int)((p->width / 8 + 31) / 32);
  nv = nv <= 4 ? nv : nv <= 6 ? 6 : nv <= 8 ? 8 : nv <= 12 ? 12 : 16;
  const unsigned blocks = (unsigned)((p->rows * p->nsections + 7) / 8);  // 8 (row, section) warps per block
  launch_qknorm(a, p->nsections, nv, blocks, st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("qknorm_rope_kernel launch", e);
  return WANB200_OK;
}

// ------------------------------------------------------------------ partial-sum reduction
// Thread = (row, section): the section's partials of the row added in order.
// The per-rank sums of squares of `_tp_rms_qk` / `_tp_rms` (fast_dit.py:138-140, 158) that the
// TP all-reduce (fast_dit.py:141, 159) then adds over ranks.
struct SumsqArgs {
  const float* part;
  int64_t rows, row_stride, part0[2], out_stride;
  int parts;
  float* out;
};

__global__ void __launch_bounds__(256) sumsq_reduce_kernel(const SumsqArgs a) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int sec = blockIdx.y;
  if (row >= a.rows) return;
  const float* src = a.part + row * a.row_stride + (sec ? a.part0[1] : a.part0[0]);
  float s = 0.f;
  for (int k = 0; k < a.parts; ++k) s += __ldg(src + k);
  a.out[sec * a.out_stride + row] = s;
}

int sumsq_reduce(const wanb200_sumsq_reduce_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "sumsq_reduce: null params");
  if (!p->part || !p->out || p->rows <= 0 || p->nsections < 1 || p->nsections > 2 || p->parts < 1 ||
      p->out_stride < p->rows)
    return set_error(WANB200_EINVAL, "sumsq_reduce: need part, out, rows > 0, 1 <= nsections <= 2, parts >= 1, "
                                     "out_stride >= rows");
  for (int s = 0; s < p->nsections; ++s)
    if (p->part0[s] < 0 || p->part0[s] + p->parts > p->row_stride)
      return set_error(WANB200_EINVAL, "sumsq_reduce: part0[s] + parts must lie in 0..row_stride");
  if ((p->rows + 255) / 256 > INT32_MAX) return set_error(WANB200_EINVAL, "sumsq_reduce: too many rows");
  SumsqArgs a;
  a.part = p->part;
  a.rows = p->rows;
  a.row_stride = p->row_stride;
  a.part0[0] = p->part0[0];
  a.part0[1] = p->nsections > 1 ? p->part0[1] : 0;
  a.out_stride = p->out_stride;
  a.parts = p->parts;
  a.out = p->out;
  sumsq_reduce_kernel<<<dim3((unsigned)((p->rows + 255) / 256), (unsigned)p->nsections), 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("sumsq_reduce_kernel launch", e);
  return WANB200_OK;
}

// ------------------------------------------------------------------ bias + gate + residual
struct ResArgs {
  void* out;             // bf16, or fp32 (out_f32)
  const void* residual;  // bf16, or fp32 (res_f32)
  int res_f32, out_f32;
  const __nv_bfloat16* y;
  int64_t rows;
  int dim;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* gate_mod;
  const float* gate_e0;
  int64_t gate_frame_stride, seq_len, tokens_per_frame, row_offset, rows_per_seq;
  int nsum;
  int64_t y_slice_stride;
};

// Thread (x, y) = 8 channels x of row blockIdx.x * blockDim.y + y (2-D blocks: no per-thread
// integer division).  `x + _gate(y + b, e[k])` / `x + (y + b)` after the TP all-reduce of a
// row-parallel projection (models/fast_dit.py:126-131, 179-181).
template <bool GATE>
__global__ void __launch_bounds__(1024) bias_gate_residual_kernel(const ResArgs a) {
  const int vpr = a.dim >> 3;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;
  if ((int)threadIdx.x >= vpr || row >= a.rows) return;
  const int col = threadIdx.x * 8;
  float r[8], y[8], b[8];
  if (a.res_f32) {
    const float4* rp = reinterpret_cast<const float4*>(static_cast<const float*>(a.residual) + row * a.dim + col);
    const float4 lo = rp[0], hi = rp[1];
    r[0] = lo.x; r[1] = lo.y; r[2] = lo.z; r[3] = lo.w; r[4] = hi.x; r[5] = hi.y; r[6] = hi.z; r[7] = hi.w;
  } else {
    unpack_bf16x8(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.residual) + row * a.dim + col), r);
  }
  unpack_bf16x8(*reinterpret_cast<const uint4*>(a.y + row * a.dim + col), y);
  for (int s = 1; s < a.nsum; ++s) {  // the inbox slices of a fused reduce-scatter
    float t[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(a.y + s * a.y_slice_stride + row * a.dim + col), t);
#pragma unroll
    for (int k = 0; k < 8; ++k) y[k] += t[k];
  }
  unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(a.bias + col)), b);
  if constexpr (GATE) {
    float g[8];
    unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(a.gate_mod + col)), g);
    const float* e = a.gate_e0 +
                     (int64_t)frame_of_row32((int)row, (int)a.rows_per_seq, (int)a.row_offset, (int)a.seq_len,
                                             (int)a.tokens_per_frame) * a.gate_frame_stride + col;
    const float4 e0 = __ldg(reinterpret_cast<const float4*>(e)), e1 = __ldg(reinterpret_cast<const float4*>(e + 4));
    g[0] += e0.x; g[1] += e0.y; g[2] += e0.z; g[3] += e0.w;
    g[4] += e1.x; g[5] += e1.y; g[6] += e1.z; g[7] += e1.w;
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = fmaf(y[k] + b[k], g[k], r[k]);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] += y[k] + b[k];
  }
  if (a.out_f32) {
    float4* op = reinterpret_cast<float4*>(static_cast<float*>(a.out) + row * a.dim + col);
    op[0] = make_float4(r[0], r[1], r[2], r[3]);
    op[1] = make_float4(r[4], r[5], r[6], r[7]);
    return;
  }
  uint4 u;
  u.x = pack_bf16x2(r[0], r[1]);
  u.y = pack_bf16x2(r[2], r[3]);
  u.z = pack_bf16x2(r[4], r[5]);
  u.w = pack_bf16x2(r[6], r[7]);
  *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + row * a.dim + col) = u;
}

int bias_gate_residual(const wanb200_residual_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "bias_gate_residual: null params");
  if (!p->out || !p->residual || !p->y || !p->bias || p->rows <= 0 || p->dim <= 0 || p->dim % 8 ||
      p->dim > INT32_MAX)
    return set_error(WANB200_EINVAL, "bias_gate_residual: need out, residual, y, bias, rows > 0, dim % 8 == 0");
  if (!aligned16(p->out) || !aligned16(p->residual) || !aligned16(p->y) || !aligned16(p->bias))
    return set_error(WANB200_EINVAL, "bias_gate_residual: pointers must be 16-byte aligned");
  const bool gate = p->gate_mod != nullptr;
  if (gate && (!p->gate_e0 || !aligned16(p->gate_mod) || !aligned16(p->gate_e0) || p->gate_frame_stride % 4 ||
               p->seq_len <= 0 || p->tokens_per_frame <= 0 || p->row_offset < 0 || p->rows_per_seq < 0))
    return set_error(WANB200_EINVAL, "bias_gate_residual: gate needs gate_e0, seq_len, tokens_per_frame "
                                     "(row_offset, rows_per_seq >= 0)");
  ResArgs a;
  a.out = p->out;
  a.residual = p->residual;
  a.res_f32 = p->residual_f32 != 0;
  a.out_f32 = p->out_f32 != 0;
  a.y = reinterpret_cast<const __nv_bfloat16*>(p->y);
  a.rows = p->rows;
  a.dim = (int)p->dim;
  a.bias = reinterpret_cast<const __nv_bfloat16*>(p->bias);
  a.gate_mod = reinterpret_cast<const __nv_bfloat16*>(p->gate_mod);
  a.gate_e0 = p->gate_e0;
  a.gate_frame_stride = p->gate_frame_stride;
  a.seq_len = p->seq_len > 0 ? p->seq_len : 1;
  a.tokens_per_frame = p->tokens_per_frame > 0 ? p->tokens_per_frame : 1;
  a.row_offset = p->row_offset;
  a.rows_per_seq = p->rows_per_seq;
  a.nsum = p->nsum;
  a.y_slice_stride = p->y_slice_stride;
  if (p->dim / 8 > 1024) return set_error(WANB200_EINVAL, "bias_gate_residual: dim <= 8192");
  if (p->rows > INT32_MAX / 2 || p->seq_len > INT32_MAX || p->tokens_per_frame > INT32_MAX ||
      p->row_offset > INT32_MAX / 2 || p->rows_per_seq > INT32_MAX)
    return set_error(WANB200_EINVAL, "bias_gate_residual: rows / frame arguments must be < 2^30");
  const dim3 blk = row_block(p->dim / 8);
  const int64_t blocks = (p->rows + blk.y - 1) / blk.y;
  if (blocks > INT32_MAX) return set_error(WANB200_EINVAL, "bias_gate_residual: too large");
  if (gate)
    bias_gate_residual_kernel<true><<<(unsigned)blocks, blk, 0, st>>>(a);
  else
    bias_gate_residual_kernel<false><<<(unsigned)blocks, blk, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("bias_gate_residual_kernel launch", e);
  return WANB200_OK;
}

}  // namespace wanb200
