// Flash attention forward for head_dim 128 on tcgen05:  O = softmax(Q K^T * scale) V.
//
// Replaces the reference's attention seam (`_sdpa` models/fast_dit.py:186-189, `_cte` 228-241)
// and its Trainium kernels: the self-attention NST kernel (kernels/self_attention_nst.py:49-289,
// online softmax over key tiles) and the cross-attention kernel over the 512 cached text keys
// (kernels/cross_attention.py:17-123).  Exact softmax (running max / running sum), no mask
// other than the key tail, non-causal.
//
// One CTA = one (batch, head, 128-query tile).  Per 128-key tile j:
//   S_j = Q K_j^T            UMMA 128x128x128, fp32 in TMEM (2 buffers, columns 0..255)
//   P_j = exp2(S_j*c - m_j)  softmax warps, bf16, written to swizzled shared memory (2 buffers)
//   O_j = P_j V_j            UMMA 128x128x128 into TMEM (2 buffers, columns 256..511)
//   O  = O * exp2(m_{j-1} - m_j) + O_j   in the softmax warps' registers
// The MMA thread issues QK_{j+1} before PV_j, so the tensor core computes the next scores
// while the softmax warps exponentiate the current ones.
//
// Warp roles (192 threads): warps 0..3 softmax (thread t owns query row t = TMEM lane t),
// warp 4 TMA producer, warp 5 TMEM allocator + UMMA issuer.
#include "common.cuh"
#include "internal.h"

namespace wanb200 {

constexpr int ABM = 128, ABN = 128, AD = 128;
constexpr int A_TILE = ABM * AD * 2;  // 32 KB: two 64-column swizzle blocks of 16 KB
constexpr int A_BLK = 16384;
constexpr int A_OFF_Q = 0;
constexpr int A_OFF_K = A_OFF_Q + A_TILE;      // 2 stages
constexpr int A_OFF_V = A_OFF_K + 2 * A_TILE;  // 2 stages
constexpr int A_OFF_P = A_OFF_V + 2 * A_TILE;  // 2 buffers
constexpr int A_TILES_END = A_OFF_P + 2 * A_TILE;  // 229376
constexpr int A_SMEM_BYTES = A_TILES_END + 256 + 1024;
constexpr uint32_t A_TMEM_COLS = 512;

struct AttnArgs {
  __nv_bfloat16* o;
  int64_t o_tok_stride, o_batch_stride;
  int Lq, Lk;
  float scale_log2;
  int* err;
};

__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint8_t* meta = smem + A_TILES_END;
  const uint32_t m0 = smem_u32(meta);
  const uint32_t q_full = m0;
  const uint32_t k_full = m0 + 8, k_empty = m0 + 24;
  const uint32_t v_full = m0 + 40, v_empty = m0 + 56;
  const uint32_t s_full = m0 + 72, s_empty = m0 + 88;
  const uint32_t p_full = m0 + 104;
  const uint32_t o_full = m0 + 120, o_empty = m0 + 136;
  const uint32_t done_bar = m0 + 152;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(meta + 160);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 164);
  int* err = args.err;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * ABM, h = blockIdx.y, b = blockIdx.z;
  const int nkv = (args.Lk + ABN - 1) / ABN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full + 8 * s, 1);
      mbar_init(k_empty + 8 * s, 1);
      mbar_init(v_full + 8 * s, 1);
      mbar_init(v_empty + 8 * s, 1);
      mbar_init(s_full + 8 * s, 1);
      mbar_init(s_empty + 8 * s, 4);
      mbar_init(p_full + 8 * s, 4);
      mbar_init(o_full + 8 * s, 1);
      mbar_init(o_empty + 8 * s, 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), A_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t k_issued = 0, v_issued = 0, k_ph = 0, v_ph = 0;
      bool ok = true;
      mbar_expect_tx(q_full, A_TILE);
      tma_load_4d(sbase + A_OFF_Q, &tmQ, q_full, 0, h, q0, b);
      tma_load_4d(sbase + A_OFF_Q + A_BLK, &tmQ, q_full, 64, h, q0, b);
      for (int j = 0; j < nkv; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(k_empty + 8 * s, ph ^ 1, abort_flag, err, kErrTimeoutAttnProducer)) { ok = false; break; }
        mbar_expect_tx(k_full + 8 * s, A_TILE);
        tma_load_4d(sbase + A_OFF_K + s * A_TILE, &tmK, k_full + 8 * s, 0, h, j * ABN, b);
        tma_load_4d(sbase + A_OFF_K + s * A_TILE + A_BLK, &tmK, k_full + 8 * s, 64, h, j * ABN, b);
        k_issued |= 1u << s;
        k_ph = (k_ph & ~(1u << s)) | (ph << s);
        if (!mbar_wait(v_empty + 8 * s, ph ^ 1, abort_flag, err, kErrTimeoutAttnProducer)) { ok = false; break; }
        mbar_expect_tx(v_full + 8 * s, A_TILE);
        tma_load_4d(sbase + A_OFF_V + s * A_TILE, &tmV, v_full + 8 * s, 0, h, j * ABN, b);
        tma_load_4d(sbase + A_OFF_V + s * A_TILE + A_BLK, &tmV, v_full + 8 * s, 64, h, j * ABN, b);
        v_issued |= 1u << s;
        v_ph = (v_ph & ~(1u << s)) | (ph << s);
      }
      if (!ok) {
        mbar_drain(q_full, 0, err);
        for (int s = 0; s < 2; ++s) {
          if ((k_issued >> s) & 1) mbar_drain(k_full + 8 * s, (k_ph >> s) & 1, err);
          if ((v_issued >> s) & 1) mbar_drain(v_full + 8 * s, (v_ph >> s) & 1, err);
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(ABM, ABN, false, false);  // Q, K both K(=d)-major
      constexpr uint32_t idesc_o = idesc_bf16_f32(ABM, AD, false, true);    // P K-major, V MN(=d)-major
      bool ok = mbar_wait(q_full, 0, abort_flag, err, kErrTimeoutAttnMma);
      auto issue_qk = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(k_full + 8 * s, ph, abort_flag, err, kErrTimeoutAttnMma)) return false;
        if (!mbar_wait(s_empty + 8 * s, ph ^ 1, abort_flag, err, kErrTimeoutAttnMma)) return false;
        tc_fence_after();
        const uint32_t d = tmem_base + s * ABN;
        const uint32_t kb = sbase + A_OFF_K + s * A_TILE;
#pragma unroll
        for (int kk = 0; kk < AD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * A_BLK + (kk & 3) * 32;
          umma_bf16(d, sw128_desc(sbase + A_OFF_Q + off, 16, 1024), sw128_desc(kb + off, 16, 1024), idesc_s, kk != 0);
        }
        umma_commit(s_full + 8 * s);
        umma_commit(k_empty + 8 * s);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(p_full + 8 * s, ph, abort_flag, err, kErrTimeoutAttnMma)) return false;
        if (!mbar_wait(v_full + 8 * s, ph, abort_flag, err, kErrTimeoutAttnMma)) return false;
        if (!mbar_wait(o_empty + 8 * s, ph ^ 1, abort_flag, err, kErrTimeoutAttnMma)) return false;
        tc_fence_after();
        const uint32_t d = tmem_base + 2 * ABN + s * AD;
        const uint32_t pb = sbase + A_OFF_P + s * A_TILE;
        const uint32_t vb = sbase + A_OFF_V + s * A_TILE;
#pragma unroll
        for (int kk = 0; kk < ABN / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * A_BLK + (kk & 3) * 32;
          // V tile: key row k at k*128 B inside each 64-wide d block; d blocks 16 KB apart.
          umma_bf16(d, sw128_desc(pb + poff, 16, 1024), sw128_desc(vb + kk * 2048, A_BLK, 1024), idesc_o, kk != 0);
        }
        umma_commit(o_full + 8 * s);
        umma_commit(v_empty + 8 * s);
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 1 < nkv && !issue_qk(j + 1)) break;
        if (!issue_pv(j)) break;
      }
      umma_commit(done_bar);
      mbar_drain(done_bar, 0, err);
    }
  } else {
    // ------------------------------------------------------------ softmax + output (warps 0..3)
    const int r = threadIdx.x;  // query row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    const float sl2 = args.scale_log2;
    float o_acc[AD];
#pragma unroll
    for (int i = 0; i < AD; ++i) o_acc[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;
    bool ok = true;

    auto accumulate = [&](int i, float a) -> bool {
      const int s = i & 1;
      if (!mbar_wait_warp(o_full + 8 * s, (i >> 1) & 1, abort_flag, err, kErrTimeoutAttnSoftmax)) return false;
      tc_fence_after();
      const uint32_t t = tmem_base + lane_off + 2 * ABN + s * AD;
#pragma unroll
      for (int c = 0; c < AD / 32; ++c) {
        float v[32];
        tmem_ld32(t + c * 32, v);
#pragma unroll
        for (int k = 0; k < 32; ++k) o_acc[c * 32 + k] = fmaf(o_acc[c * 32 + k], a, v[k]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty + 8 * s);
      return true;
    };

    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      if (!mbar_wait_warp(s_full + 8 * s, (j >> 1) & 1, abort_flag, err, kErrTimeoutAttnSoftmax)) { ok = false; break; }
      tc_fence_after();
      const uint32_t t_s = tmem_base + lane_off + s * ABN;
      const int kbase = j * ABN;
      const bool tail = kbase + ABN > args.Lk;  // CTA-uniform
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < ABN / 32; ++c) {
        float v[32];
        tmem_ld32(t_s + c * 32, v);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const bool valid = !tail || (kbase + c * 32 + k < args.Lk);
          mx = valid ? fmaxf(mx, v[k]) : mx;
        }
      }
      const float m_new = fmaxf(m_run, mx * sl2);
      const float alpha = ex2_approx(m_run - m_new);
      // pass 2: p = exp2(s*c - m), bf16 into the swizzled P tile (K-major, 128 B rows)
      float rowsum = 0.f;
      uint8_t* pbuf = smem + A_OFF_P + s * A_TILE;
#pragma unroll
      for (int c = 0; c < ABN / 32; ++c) {
        float v[32];
        tmem_ld32(t_s + c * 32, v);
        uint32_t pk[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const bool v0 = !tail || (kbase + c * 32 + k < args.Lk);
          const bool v1 = !tail || (kbase + c * 32 + k + 1 < args.Lk);
          const float p0 = v0 ? ex2_approx(fmaf(v[k], sl2, -m_new)) : 0.f;
          const float p1 = v1 ? ex2_approx(fmaf(v[k + 1], sl2, -m_new)) : 0.f;
          rowsum += p0 + p1;
          pk[k >> 1] = pack_bf16x2(p0, p1);
        }
        uint8_t* rowp = pbuf + (c >> 1) * A_BLK + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int ch = (c & 1) * 4 + t;
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * t], pk[4 * t + 1], pk[4 * t + 2], pk[4 * t + 3]);
        }
      }
      // S buffer consumed
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty + 8 * s);
      // P tile ready for the async proxy
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + 8 * s);
      l_run = l_run * alpha + rowsum;
      m_run = m_new;
      if (j >= 1 && !accumulate(j - 1, alpha_prev)) { ok = false; break; }
      alpha_prev = alpha;
    }
    if (ok) ok = accumulate(nkv - 1, alpha_prev);
    if (ok) {
      const int qrow = q0 + r;
      if (qrow < args.Lq) {
        const float inv_l = 1.f / l_run;
        uint4* dst = reinterpret_cast<uint4*>(args.o + (int64_t)b * args.o_batch_stride +
                                              (int64_t)qrow * args.o_tok_stride + (int64_t)h * AD);
#pragma unroll
        for (int q = 0; q < AD / 8; ++q) {
          uint4 u;
          u.x = pack_bf16x2(o_acc[q * 8 + 0] * inv_l, o_acc[q * 8 + 1] * inv_l);
          u.y = pack_bf16x2(o_acc[q * 8 + 2] * inv_l, o_acc[q * 8 + 3] * inv_l);
          u.z = pack_bf16x2(o_acc[q * 8 + 4] * inv_l, o_acc[q * 8 + 5] * inv_l);
          u.w = pack_bf16x2(o_acc[q * 8 + 6] * inv_l, o_acc[q * 8 + 7] * inv_l);
          dst[q] = u;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem_base, A_TMEM_COLS);
}

// ------------------------------------------------------------------ host launcher
int attn_fwd(const wanb200_attn_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "attn: null params");
  if (!p->q || !p->k || !p->v || !p->o) return set_error(WANB200_EINVAL, "attn: null q/k/v/o");
  if (p->head_dim != AD) return set_error(WANB200_EINVAL, "attn: head_dim must be 128");
  if (p->batch <= 0 || p->heads <= 0 || p->q_len <= 0 || p->kv_len <= 0)
    return set_error(WANB200_EINVAL, "attn: batch, heads, q_len, kv_len must be positive");
  if (p->batch > 65535 || p->heads > 65535 || p->q_len > (int64_t)INT32_MAX - ABM || p->kv_len > (int64_t)INT32_MAX - ABN)
    return set_error(WANB200_EINVAL, "attn: batch/heads/lengths too large");
  const int64_t strides[8] = {p->q_tok_stride, p->q_batch_stride, p->k_tok_stride, p->k_batch_stride,
                              p->v_tok_stride, p->v_batch_stride, p->o_tok_stride, p->o_batch_stride};
  for (int i = 0; i < 8; ++i)
    if (strides[i] <= 0 || strides[i] % 8) return set_error(WANB200_EINVAL, "attn: strides must be positive multiples of 8");
  if (p->q_tok_stride < p->heads * AD || p->k_tok_stride < p->heads * AD || p->v_tok_stride < p->heads * AD ||
      p->o_tok_stride < p->heads * AD)
    return set_error(WANB200_EINVAL, "attn: token stride smaller than heads*128");
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->o))
    return set_error(WANB200_EINVAL, "attn: q/k/v/o must be 16-byte aligned");
  if (!(p->softmax_scale > 0.f)) return set_error(WANB200_EINVAL, "attn: softmax_scale must be positive");

  int* err = device_error_word();
  if (!err) return WANB200_ECUDA;
  CUtensorMap tq, tk, tv;
  const int box[4] = {64, 1, ABM, 1};
  {
    const int64_t dims[4] = {AD, p->heads, p->q_len, p->batch};
    const int64_t str[4] = {1, AD, p->q_tok_stride, p->q_batch_stride};
    int rc = make_tmap_4d(&tq, p->q, dims, str, box);
    if (rc) return rc;
  }
  {
    const int64_t dims[4] = {AD, p->heads, p->kv_len, p->batch};
    const int64_t sk[4] = {1, AD, p->k_tok_stride, p->k_batch_stride};
    int rc = make_tmap_4d(&tk, p->k, dims, sk, box);
    if (rc) return rc;
    const int64_t sv[4] = {1, AD, p->v_tok_stride, p->v_batch_stride};
    rc = make_tmap_4d(&tv, p->v, dims, sv, box);
    if (rc) return rc;
  }
  AttnArgs aa;
  aa.o = reinterpret_cast<__nv_bfloat16*>(p->o);
  aa.o_tok_stride = p->o_tok_stride;
  aa.o_batch_stride = p->o_batch_stride;
  aa.Lq = (int)p->q_len;
  aa.Lk = (int)p->kv_len;
  aa.scale_log2 = p->softmax_scale * 1.4426950408889634f;
  aa.err = err;

  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, A_SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(attn)", e);
    attr_set[dev] = true;
  }
  dim3 grid((unsigned)((p->q_len + ABM - 1) / ABM), (unsigned)p->heads, (unsigned)p->batch);
  attn_fwd_kernel<<<grid, 192, A_SMEM_BYTES, st>>>(tq, tk, tv, aa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("attn_fwd_kernel launch", e);
  return WANB200_OK;
}

}  // namespace wanb200
