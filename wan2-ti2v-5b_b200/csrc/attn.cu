// Flash attention forward for head_dim 128 on tcgen05:  O = softmax(Q K^T * scale) V.
//
// Replaces the reference's attention seam (`_sdpa` models/fast_dit.py:186-189, `_cte` 228-241)
// and its Trainium kernels: the self-attention NST kernel (kernels/self_attention_nst.py:49-289,
// online softmax over key tiles) and the cross-attention kernel over the 512 cached text keys
// (kernels/cross_attention.py:17-123).  Exact softmax (running max / running sum), no mask
// other than the key tail, non-causal.
//
// One work unit = one (batch, head), one key range and TWO 128-query tiles (t = 0, 1).  Per
// 128-key tile j:
//   S_t = Q_t K_j^T          UMMA 128x128x128 into TMEM (S_0 cols 0..127, S_1 cols 128..255)
//   P_t = exp2(S_t*c - m_t)  softmax warpgroup t; bf16 kernel: bf16 pairs written back into
//                            TMEM over the first 64 columns of S_t; e4m3 kernel: e4m3 in
//                            swizzled shared memory
//   O_t += P_t V_j           UMMA (bf16: A = P_t read from TMEM) into TMEM (O_0 cols 256..383,
//                            O_1 cols 384..511)
// Two kernels: attn_persistent_kernel (bf16, the product path; one CTA per SM walking the units)
// and attn_fp8_kernel (e4m3 operands, one CTA per unit).
// The tensor core alternates between the tiles, so the MMAs of one tile run while the other
// tile's warpgroup exponentiates.  O stays in TMEM for the whole key loop; the running max used
// for the exponent is only raised when a tile's max exceeds it by more than 8 (a factor 256 in
// P), and only then is O rescaled in place (tcgen05.ld / st).  The result is exact: P and the
// row sum use the same stale max, which cancels in O / l.
//
// Ordering facts the protocol relies on: UMMAs issued by one thread execute in order, and a
// tcgen05.commit arrives only when every earlier UMMA of that thread has completed.  So when
// S_t(j+1) is signalled complete, PV_t(j) has completed too: P_t's buffer is free and O_t may
// be rescaled before PV_t(j+1) is issued (which waits for this warpgroup's p_full).
//
// Warp roles (320 threads): warps 0-3 softmax of tile 0, warps 4-7 softmax of tile 1 (thread
// row = TMEM lane), warp 8 TMA producer, warp 9 TMEM allocator + UMMA issuer.  The persistent
// bf16 kernel launches 384: warps 10 and 11 only complete the producer / MMA warpgroup, so that
// setmaxnreg can move registers from it to the two softmax warpgroups (192 each, no spills), and
// hands P to the P V MMA in two parts (the first 96 keys, then the last 32).  K and V tiles
// stream through one ring (K_0, V_0, K_1, V_1, ...): 5 slots of 32 KB in the bf16 kernel, whose
// P needs no shared memory, 3 slots of 16 KB in the e4m3 one.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace wanb200 {

constexpr int ABM = 128, ABN = 128, AD = 128;
constexpr int A_TILE = ABM * AD * 2;  // 32 KB: two 64-column swizzle blocks of 16 KB
constexpr int A_BLK = 16384;
constexpr int A_RING = 3;    // e4m3 variant: K/V ring slots (Q_0, Q_1, P_0, P_1 and the ring in shared memory)
constexpr int A_RING16 = 5;  // bf16: P lives in tensor memory, so the ring takes P's 64 KB: Q_0, Q_1, 5 slots
constexpr int A_TILES_END = (2 + A_RING16) * A_TILE;  // 229376
constexpr int A_SMEM_BYTES = A_TILES_END + 256 + 1024;
// e4m3 variant: every tile is one 16 KB swizzle block (128 rows x 128 one-byte elements)
constexpr int A_TILES_END8 = (2 + 2 + A_RING) * A_BLK;  // 114688
constexpr int A_SMEM_BYTES8 = A_TILES_END8 + 256 + 1024;
constexpr float A_E4M3_MAX = 448.f;
constexpr uint32_t A_TMEM_COLS = 512;
constexpr int A_THREADS = 320;
constexpr int A_THREADS_P = 384;  // persistent kernel: 10 working warps + 2 idle (setmaxnreg warpgroups)
constexpr float A_RESCALE_THRESHOLD = 8.0f;  // log2 units
constexpr int A_P_SPLIT = 96;  // bf16 kernel: keys of P handed to the P V MMA ahead of the rest
static_assert(A_P_SPLIT % 32 == 0 && A_P_SPLIT > 0 && A_P_SPLIT < 128,
              "the softmax hands P over in 32-key chunks");

struct AttnArgs {
  __nv_bfloat16* o;
  int64_t o_tok_stride, o_batch_stride;
  int Lq, Lk, heads;
  float scale_log2;
  // split-KV: CTA blockIdx.x = q_pair * kv_splits + split covers key tiles
  // [split * kv_tiles_per_split, ...); with kv_splits > 1 it writes its unnormalised O and
  // (running max, row sum) to o_part / ml_part and attn_combine_kernel merges the splits.
  int kv_splits, kv_tiles_per_split;
  // partial slots: with part_nslots > 1 split s writes slot part_slot0 + s and the merge reads
  // slots 0 .. part_nslots-1 (several launches over different key sets may fill one workspace)
  int part_slot0, part_nslots;
  float* o_part;   // [part_nslots, B*H*Lq, 128]
  float* ml_part;  // [part_nslots, B*H*Lq, 2]
  int64_t part_rows;  // B*H*Lq
  // e4m3 variant: q / k dequantisation scales per (batch, head, 128-token block), v per
  // (batch, head); nqb / nkb = blocks per (batch, head)
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  int nqb, nkb;
  int units, nqp;  // persistent kernel: (query pair, split, head, batch) units; query-tile pairs
  int* err;
};

// FP8: Q, K e4m3 [B, L, H, 128] and V transposed e4m3 [B, H, 128, L] (keys contiguous, so both
// MMAs take K-major operands), P packed to e4m3; S is dequantised by the q and k block scales
// inside the exponent's multiplier, O by the v scale at the end.
__global__ void __launch_bounds__(A_THREADS, 1)
    attn_fp8_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  constexpr int TILE = A_BLK;
  constexpr int RING = A_RING;
  // [Q_0 Q_1 | P_0 P_1 | ring]
  constexpr int OFF_Q = 0, OFF_P = 2 * TILE, OFF_R = 4 * TILE, TILES_END = OFF_R + RING * TILE;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint8_t* meta = smem + TILES_END;
  const uint32_t m0 = smem_u32(meta);
  const uint32_t q_full = m0;                 // 1
  const uint32_t kv_full = m0 + 8;            // RING (<= 5)
  const uint32_t kv_empty = m0 + 48;          // RING
  const uint32_t s_full = m0 + 88;            // 2
  const uint32_t p_full = m0 + 104;           // 2
  const uint32_t o_done = m0 + 120;           // 2
  const uint32_t done_bar = m0 + 136;         // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(meta + 144);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 148);
  int* err = args.err;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x % args.kv_splits;
  const int q0 = (blockIdx.x / args.kv_splits) * 2 * ABM, h = blockIdx.y, b = blockIdx.z;
  const int kv0 = split * args.kv_tiles_per_split;  // first key tile of this CTA
  const int nkv = min((args.Lk + ABN - 1) / ABN - kv0, args.kv_tiles_per_split);  // >= 1 (host)

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < RING; ++s) {
      mbar_init(kv_full + 8 * s, 1);
      mbar_init(kv_empty + 8 * s, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full + 8 * t, 1);
      mbar_init(p_full + 8 * t, 4);
      mbar_init(o_done + 8 * t, 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), A_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t issued = 0, last_ph = 0;
      bool ok = true;
      mbar_expect_tx(q_full, 2 * TILE);
      for (int t = 0; t < 2; ++t) {
        tma_load_4d(sbase + OFF_Q + t * TILE, &tmQ, q_full, 0, h, q0 + t * ABM, b);
      }
      for (int i = 0; i < 2 * nkv; ++i) {
        const int slot = i % RING;
        const uint32_t ph = (i / RING) & 1;
        if (!mbar_wait(kv_empty + 8 * slot, ph ^ 1, abort_flag, err, kErrTimeoutAttnProducer)) {
          ok = false;
          break;
        }
        const void* map = (i & 1) ? static_cast<const void*>(&tmV) : static_cast<const void*>(&tmK);
        const uint32_t dst = sbase + OFF_R + slot * TILE;
        const int key0 = (kv0 + (i >> 1)) * ABN;
        mbar_expect_tx(kv_full + 8 * slot, TILE);
        if (i & 1)
          tma_load_4d(dst, map, kv_full + 8 * slot, key0, 0, h, b);  // V^T: (key, d, head, batch)
        else
          tma_load_4d(dst, map, kv_full + 8 * slot, 0, h, key0, b);
        issued |= 1u << slot;
        last_ph = (last_ph & ~(1u << slot)) | (ph << slot);
      }
      if (!ok) {
        mbar_drain(q_full, 0, err);
        for (int s = 0; s < RING; ++s)
          if ((issued >> s) & 1) mbar_drain(kv_full + 8 * s, (last_ph >> s) & 1, err);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      // every e4m3 operand is K-major (V is stored transposed)
      constexpr uint32_t idesc_s = idesc_e4m3_f32(ABM, ABN, false, false);
      constexpr uint32_t idesc_o = idesc_e4m3_f32(ABM, AD, false, false);
      auto kv_wait = [&](int i) -> bool {
        return mbar_wait(kv_full + 8 * (i % RING), (i / RING) & 1, abort_flag, err, kErrTimeoutAttnMma);
      };
      auto qk = [&](int t, int j) {
        const int slot = (2 * j) % RING;
        tc_fence_after();
        const uint32_t d = tmem_base + t * ABN;
        const uint32_t qb = sbase + OFF_Q + t * TILE;
        const uint32_t kb = sbase + OFF_R + slot * TILE;
        #pragma unroll
        for (int kk = 0; kk < AD / 32; ++kk)  // 32 one-byte elements = 32 B per instruction
          umma_e4m3(d, sw128_desc(qb + kk * 32, 16, 1024), sw128_desc(kb + kk * 32, 16, 1024), idesc_s, kk != 0);
        umma_commit(s_full + 8 * t);
        if (t == 1) umma_commit(kv_empty + 8 * slot);
      };
      auto pv = [&](int t, int j) -> bool {
        if (!mbar_wait(p_full + 8 * t, j & 1, abort_flag, err, kErrTimeoutAttnMma)) return false;
        const int slot = (2 * j + 1) % RING;
        tc_fence_after();
        const uint32_t d = tmem_base + 2 * ABN + t * AD;
        const uint32_t vb = sbase + OFF_R + slot * TILE;
        const uint32_t pb = sbase + OFF_P + t * TILE;
#pragma unroll
        for (int kk = 0; kk < ABN / 32; ++kk)  // P (query x key) and V^T (d x key), both key-major
          umma_e4m3(d, sw128_desc(pb + kk * 32, 16, 1024), sw128_desc(vb + kk * 32, 16, 1024), idesc_o,
                    (j | kk) != 0);
        if (t == 1) umma_commit(kv_empty + 8 * slot);
        if (j == nkv - 1) umma_commit(o_done + 8 * t);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, err, kErrTimeoutAttnMma) && kv_wait(0);
      if (ok) {
        qk(0, 0);
        qk(1, 0);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        if (!kv_wait(2 * j + 1) || !pv(0, j)) break;
        if (j + 1 < nkv) {
          if (!kv_wait(2 * j + 2)) break;
          qk(0, j + 1);
        }
        if (!pv(1, j)) break;
        if (j + 1 < nkv) qk(1, j + 1);
      }
      umma_commit(done_bar);
      mbar_drain(done_bar, 0, err);
    }
  } else {
    // ------------------------------------------------------------ softmax + output (warps 0..7)
    const int t = warp >> 2;                    // query tile of this warpgroup
    const int r = threadIdx.x & 127;            // query row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem_base + lane_off + t * ABN;
    const uint32_t t_o = tmem_base + lane_off + 2 * ABN + t * AD;
    uint8_t* pbuf = smem + OFF_P + t * TILE;
    const float sl2_base = args.scale_log2;
    // the second tile of the last pair may lie past q_len (its rows are never stored)
    const float qsc = __ldg(args.q_scale + ((int64_t)b * args.heads + h) * args.nqb + min(q0 / ABM + t, args.nqb - 1));
    const float* ksc = args.k_scale + ((int64_t)b * args.heads + h) * args.nkb + kv0;
    float m_used = -INFINITY, l_run = 0.f;
    bool ok = true;

    for (int j = 0; j < nkv; ++j) {
      if (!mbar_wait_warp(s_full + 8 * t, j & 1, abort_flag, err, kErrTimeoutAttnSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[ABN];
#pragma unroll
      for (int c = 0; c < ABN / 32; ++c) tmem_ld32_nowait(t_s + c * 32, sr + c * 32);
      tmem_wait_ld();
      float* s = reinterpret_cast<float*>(sr);
      const float sl2 = sl2_base * qsc * __ldg(ksc + j);  // scores carry the q and k block scales
      const int kbase = (kv0 + j) * ABN;
      if (kbase + ABN > args.Lk) {  // CTA-uniform: mask the key tail
#pragma unroll
        for (int k = 0; k < ABN; ++k)
          if (kbase + k >= args.Lk) s[k] = -INFINITY;
      }
      // row max with 8 independent partial maxima of three-input FMNMX (a single chain of 127
      // dependent FMNMX would dominate the warp's latency; two values per instruction)
      float m8[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) m8[c] = fmaxf(s[2 * c], s[2 * c + 1]);
#pragma unroll
      for (int i = 1; i < ABN / 16; ++i)
#pragma unroll
        for (int c = 0; c < 8; ++c) m8[c] = fmax3(m8[c], s[16 * i + 2 * c], s[16 * i + 2 * c + 1]);
      const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      const float m_cand = mx * sl2;
      const bool need = m_cand > m_used + A_RESCALE_THRESHOLD;
      const bool any_need = __any_sync(0xffffffffu, need);
      float alpha = 1.f;  // 0 on the first tile, 1 where !need
      if (any_need) {
        const float m_new = need ? m_cand : m_used;
        alpha = ex2_approx(m_used - m_new);
        l_run *= alpha;
        m_used = m_new;
      }
      const float neg = -m_used;
      float r8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // 8 partial row sums (short dependency chains)
      // P in e4m3 (at most 2^8 under the lazy max, inside the 448 range): 32 keys = 32 bytes
      uint8_t* rowp = pbuf + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
      for (int c = 0; c < ABN / 32; ++c) {
        uint32_t pk[8];
#pragma unroll
        for (int k = 0; k < 32; k += 4) {
          const float p0 = ex2_approx(fmaf(s[c * 32 + k], sl2, neg));
          const float p1 = ex2_approx(fmaf(s[c * 32 + k + 1], sl2, neg));
          const float p2 = ex2_approx(fmaf(s[c * 32 + k + 2], sl2, neg));
          const float p3 = ex2_approx(fmaf(s[c * 32 + k + 3], sl2, neg));
          r8[(k >> 2) & 7] += (p0 + p1) + (p2 + p3);
          pk[k >> 2] = pack_e4m3x2(p0, p1) | (pack_e4m3x2(p2, p3) << 16);
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int ch = c * 2 + q;
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      l_run += ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
      // Rescale O_t (rare).  PV_t(j-1) has completed (see the ordering note above) and PV_t(j)
      // is not issued before this warpgroup's p_full arrival below.
      if (any_need && j > 0) {
#pragma unroll 1
        for (int c = 0; c < AD / 32; ++c) {
          float o[32];
          tmem_ld32(t_o + c * 32, o);
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] *= alpha;
          tmem_st32(t_o + c * 32, o);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();  // e4m3 P in shared memory, read by the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + 8 * t);
    }
    if (ok) ok = mbar_wait_warp(o_done + 8 * t, 0, abort_flag, err, kErrTimeoutAttnSoftmax);
    const float vsc = __ldg(  // O carries the v scale
        args.v_scale + (int64_t)b * args.heads + h);
    if (ok && args.part_nslots > 1) {
      // partial result of this key range: unnormalised O, running max (log2 units), row sum
      tc_fence_after();
      const int qrow = q0 + t * ABM + r;
      const int64_t prow =
          (int64_t)(args.part_slot0 + split) * args.part_rows + ((int64_t)b * args.heads + h) * args.Lq + qrow;
      float4* dst = reinterpret_cast<float4*>(args.o_part + prow * AD);
#pragma unroll
      for (int c = 0; c < AD / 32; ++c) {
        float o[32];
        tmem_ld32(t_o + c * 32, o);
        if (qrow < args.Lq) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            dst[c * 8 + q] = make_float4(o[4 * q] * vsc, o[4 * q + 1] * vsc, o[4 * q + 2] * vsc, o[4 * q + 3] * vsc);
        }
      }
      if (qrow < args.Lq) *reinterpret_cast<float2*>(args.ml_part + prow * 2) = make_float2(m_used, l_run);
    } else if (ok) {
      tc_fence_after();
      const int qrow = q0 + t * ABM + r;
      const float inv_l = vsc / l_run;
      uint4* dst = reinterpret_cast<uint4*>(args.o + (int64_t)b * args.o_batch_stride +
                                            (int64_t)qrow * args.o_tok_stride + (int64_t)h * AD);
#pragma unroll
      for (int c = 0; c < AD / 32; ++c) {
        float o[32];
        tmem_ld32(t_o + c * 32, o);
        if (qrow < args.Lq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 u;
            u.x = pack_bf16x2(o[q * 8 + 0] * inv_l, o[q * 8 + 1] * inv_l);
            u.y = pack_bf16x2(o[q * 8 + 2] * inv_l, o[q * 8 + 3] * inv_l);
            u.z = pack_bf16x2(o[q * 8 + 4] * inv_l, o[q * 8 + 5] * inv_l);
            u.w = pack_bf16x2(o[q * 8 + 6] * inv_l, o[q * 8 + 7] * inv_l);
            dst[c * 4 + q] = u;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem_base, A_TMEM_COLS);
}

// Persistent bf16 attention.  The grid is at most one CTA per SM; CTA c walks the units
// u = c, c + grid, ... of (query-tile pair, key split, head, batch), consecutive units sharing a
// head's K / V in L2.  Within a unit the roles and the per-tile protocol are the ones described at
// the top of this file (those of attn_fp8_kernel, with P in TMEM).  Across units comes the
// hand-over, so that a unit's prologue and epilogue overlap the neighbouring units' work instead
// of costing a CTA launch each (a cross-attention unit has only four key tiles; a 1080-token
// self-attention unit nine):
//   * Q has one buffer: the producer loads unit i+1's Q as soon as unit i's last QK has completed
//     (q_empty), while the softmax warps finish unit i's last tile and epilogue;
//   * the first QKs of unit i+1 write S while the softmax warps still read unit i's O from TMEM;
//     unit i+1's first P V (which overwrites O) waits for their o_free arrival;
//   * the K/V ring, s_full and p_full run on across units (their phases count tiles globally).
__global__ void __maxnreg__(160)
    attn_persistent_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  constexpr int TILE = A_TILE, RING = A_RING16;
  constexpr int OFF_Q = 0, OFF_R = 2 * TILE, TILES_END = OFF_R + RING * TILE;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint8_t* meta = smem + TILES_END;
  const uint32_t m0 = smem_u32(meta);
  const uint32_t q_full = m0;           // 1
  const uint32_t q_empty = m0 + 8;      // 1
  const uint32_t kv_full = m0 + 16;     // RING
  const uint32_t kv_empty = m0 + 56;    // RING
  const uint32_t s_full = m0 + 96;      // 2
  const uint32_t p_full = m0 + 112;     // 2
  const uint32_t o_done = m0 + 128;     // 2
  const uint32_t o_free = m0 + 144;     // 2
  const uint32_t done_bar = m0 + 160;   // 1
  const uint32_t p_part = m0 + 168;     // 2: the first A_P_SPLIT key columns of P_t are in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(meta + 184);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 188);
  int* err = args.err;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = (args.Lk + ABN - 1) / ABN;  // key tiles of the whole key set
  // unit u -> (query pair, split, head, batch); splits and pairs of one head are consecutive
  auto unit = [&](int u, int& q0, int& split, int& h, int& b, int& kv0, int& nkv) {
    split = u % args.kv_splits;
    int r = u / args.kv_splits;
    const int qp = r % args.nqp;
    r /= args.nqp;
    h = r % args.heads;
    b = r / args.heads;
    q0 = qp * 2 * ABM;
    kv0 = split * args.kv_tiles_per_split;
    nkv = min(nkt - kv0, args.kv_tiles_per_split);
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < RING; ++s) {
      mbar_init(kv_full + 8 * s, 1);
      mbar_init(kv_empty + 8 * s, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full + 8 * t, 1);
      mbar_init(p_full + 8 * t, 4);
      mbar_init(p_part + 8 * t, 4);
      mbar_init(o_done + 8 * t, 1);
      mbar_init(o_free + 8 * t, 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), A_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Registers by warpgroup (setmaxnreg acts on whole warpgroups, hence the two idle warps 10, 11):
  // the producer / MMA warpgroup gives up what the softmax warpgroups take, 256 x 192 + 128 x 96 =
  // 61440 = 384 x 160 at launch; the softmax code then runs without spills, and the 4096 registers
  // the launch leaves free fit a K/V push CTA beside it (wanb200_shard_gather on a side stream).
  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 96;\n" ::: "memory");
  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t issued = 0, last_ph = 0, q_ph = 0;
      int g = 0, i = 0;
      bool ok = true, q_pending = false;
      for (int u = blockIdx.x; ok && u < args.units; u += gridDim.x, ++i) {
        int q0, split, h, b, kv0, nkv;
        unit(u, q0, split, h, b, kv0, nkv);
        if (!mbar_wait(q_empty, (i & 1) ^ 1, abort_flag, err, kErrTimeoutAttnProducer)) {
          ok = false;
          break;
        }
        mbar_expect_tx(q_full, 2 * TILE);
        for (int t = 0; t < 2; ++t) {
          tma_load_4d(sbase + OFF_Q + t * TILE, &tmQ, q_full, 0, h, q0 + t * ABM, b);
          tma_load_4d(sbase + OFF_Q + t * TILE + A_BLK, &tmQ, q_full, 64, h, q0 + t * ABM, b);
        }
        q_pending = true;
        q_ph = i & 1;  // the phase of q_full this load completes
        for (int k = 0; k < 2 * nkv; ++k, ++g) {
          const int slot = g % RING;
          const uint32_t ph = (g / RING) & 1;
          if (!mbar_wait(kv_empty + 8 * slot, ph ^ 1, abort_flag, err, kErrTimeoutAttnProducer)) {
            ok = false;
            break;
          }
          const void* map = (k & 1) ? static_cast<const void*>(&tmV) : static_cast<const void*>(&tmK);
          const uint32_t dst = sbase + OFF_R + slot * TILE;
          const int key0 = (kv0 + (k >> 1)) * ABN;
          mbar_expect_tx(kv_full + 8 * slot, TILE);
          tma_load_4d(dst, map, kv_full + 8 * slot, 0, h, key0, b);
          tma_load_4d(dst + A_BLK, map, kv_full + 8 * slot, 64, h, key0, b);
          issued |= 1u << slot;
          last_ph = (last_ph & ~(1u << slot)) | (ph << slot);
        }
      }
      if (!ok) {  // let every load in flight land before the CTA's shared memory goes away
        if (q_pending) mbar_drain(q_full, q_ph, err);
        for (int s = 0; s < RING; ++s)
          if ((issued >> s) & 1) mbar_drain(kv_full + 8 * s, (last_ph >> s) & 1, err);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(ABM, ABN, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(ABM, AD, false, true);
      auto kv_wait = [&](int r) -> bool {
        return mbar_wait(kv_full + 8 * (r % RING), (r / RING) & 1, abort_flag, err, kErrTimeoutAttnMma);
      };
      int g = 0, jg = 0, i = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < args.units; u += gridDim.x, ++i) {
        int q0, split, h, b, kv0, nkv;
        unit(u, q0, split, h, b, kv0, nkv);
        auto qk = [&](int t, int j) {
          const int slot = (g + 2 * j) % RING;
          tc_fence_after();
          const uint32_t d = tmem_base + t * ABN;
          const uint32_t qb = sbase + OFF_Q + t * TILE;
          const uint32_t kb = sbase + OFF_R + slot * TILE;
#pragma unroll
          for (int kk = 0; kk < AD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * A_BLK + (kk & 3) * 32;
            umma_bf16(d, sw128_desc(qb + off, 16, 1024), sw128_desc(kb + off, 16, 1024), idesc_s, kk != 0);
          }
          umma_commit(s_full + 8 * t);
          if (t == 1) {
            umma_commit(kv_empty + 8 * slot);
            if (j == nkv - 1) umma_commit(q_empty);  // the unit's last QK: Q may be overwritten
          }
        };
        auto pv = [&](int t, int j) -> bool {
          // P_t arrives in two parts: the K-steps over its first A_P_SPLIT keys start while the
          // softmax warps still exponentiate the rest
          if (!mbar_wait(p_part + 8 * t, (jg + j) & 1, abort_flag, err, kErrTimeoutAttnMma)) return false;
          // the unit's first P V overwrites O_t: the softmax warps must have read the last unit's
          if (j == 0 && !mbar_wait(o_free + 8 * t, (i & 1) ^ 1, abort_flag, err, kErrTimeoutAttnMma)) return false;
          const int slot = (g + 2 * j + 1) % RING;
          tc_fence_after();
          const uint32_t d = tmem_base + 2 * ABN + t * AD;
          const uint32_t pa = tmem_base + t * ABN;  // P_t over the first 64 columns of S_t
          const uint32_t vb = sbase + OFF_R + slot * TILE;
#pragma unroll
          for (int kk = 0; kk < A_P_SPLIT / 16; ++kk)
            umma_bf16_tmem_a(d, pa + kk * 8, sw128_desc(vb + kk * 2048, A_BLK, 1024), idesc_o, (j | kk) != 0);
          if (!mbar_wait(p_full + 8 * t, (jg + j) & 1, abort_flag, err, kErrTimeoutAttnMma)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = A_P_SPLIT / 16; kk < ABN / 16; ++kk)
            umma_bf16_tmem_a(d, pa + kk * 8, sw128_desc(vb + kk * 2048, A_BLK, 1024), idesc_o, true);
          if (t == 1) umma_commit(kv_empty + 8 * slot);
          if (j == nkv - 1) umma_commit(o_done + 8 * t);
          return true;
        };
        ok = mbar_wait(q_full, i & 1, abort_flag, err, kErrTimeoutAttnMma) && kv_wait(g);
        if (!ok) break;
        qk(0, 0);
        qk(1, 0);
        for (int j = 0; j < nkv; ++j) {
          if (!kv_wait(g + 2 * j + 1) || !pv(0, j)) {
            ok = false;
            break;
          }
          if (j + 1 < nkv) {
            if (!kv_wait(g + 2 * j + 2)) {
              ok = false;
              break;
            }
            qk(0, j + 1);
          }
          if (!pv(1, j)) {
            ok = false;
            break;
          }
          if (j + 1 < nkv) qk(1, j + 1);
        }
        g += 2 * nkv;
        jg += nkv;
      }
      umma_commit(done_bar);
      mbar_drain(done_bar, 0, err);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 192;\n" ::: "memory");
    // ------------------------------------------------------------ softmax + output (warps 0..7)
    const int t = warp >> 2;                    // query tile of this warpgroup
    const int r = threadIdx.x & 127;            // query row within the tile == TMEM lane
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem_base + lane_off + t * ABN;
    const uint32_t t_o = tmem_base + lane_off + 2 * ABN + t * AD;
    const float sl2 = args.scale_log2;
    int jg = 0, i = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < args.units; u += gridDim.x, ++i) {
      int q0, split, h, b, kv0, nkv;
      unit(u, q0, split, h, b, kv0, nkv);
      float m_used = -INFINITY, l_run = 0.f;
      for (int j = 0; j < nkv; ++j) {
        if (!mbar_wait_warp(s_full + 8 * t, (jg + j) & 1, abort_flag, err, kErrTimeoutAttnSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[ABN];
#pragma unroll
        for (int c = 0; c < ABN / 32; ++c) tmem_ld32_nowait(t_s + c * 32, sr + c * 32);
        tmem_wait_ld();
        float* s = reinterpret_cast<float*>(sr);
        const int kbase = (kv0 + j) * ABN;
        if (kbase + ABN > args.Lk) {  // CTA-uniform: mask the key tail
#pragma unroll
          for (int k = 0; k < ABN; ++k)
            if (kbase + k >= args.Lk) s[k] = -INFINITY;
        }
        float m8[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) m8[c] = fmaxf(s[2 * c], s[2 * c + 1]);
#pragma unroll
        for (int q = 1; q < ABN / 16; ++q)
#pragma unroll
          for (int c = 0; c < 8; ++c) m8[c] = fmax3(m8[c], s[16 * q + 2 * c], s[16 * q + 2 * c + 1]);
        const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        const float m_cand = mx * sl2;
        const bool need = m_cand > m_used + A_RESCALE_THRESHOLD;
        const bool any_need = __any_sync(0xffffffffu, need);
        float alpha = 1.f;
        if (any_need) {
          const float m_new = need ? m_cand : m_used;
          alpha = ex2_approx(m_used - m_new);
          l_run *= alpha;
          m_used = m_new;
        }
        // Rescale O_t (rare) before any of this tile's P V: S_t(j) was issued after P V_t(j-1), so
        // that has completed, and P V_t(j) waits for this warpgroup's p_part arrival below
        if (any_need && j > 0) {
#pragma unroll 1
          for (int c = 0; c < AD / 32; ++c) {
            float o[32];
            tmem_ld32(t_o + c * 32, o);
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] *= alpha;
            tmem_st32(t_o + c * 32, o);
          }
        }
        const float neg = -m_used;
        const float2 sl2v = make_float2(sl2, sl2), negv = make_float2(neg, neg);
        float2 acc2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < ABN / 32; ++c) {
          if (c == A_P_SPLIT / 32) {  // the first part of P_t is in TMEM: hand it to the P V MMA
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_part + 8 * t);
          }
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float2 x = __ffma2_rn(make_float2(s[c * 32 + k], s[c * 32 + k + 1]), sl2v, negv);
            const float p0 = ex2_approx(x.x), p1 = ex2_approx(x.y);
            acc2[(k >> 1) & 1] = __fadd2_rn(acc2[(k >> 1) & 1], make_float2(p0, p1));
            pk[k >> 1] = pack_bf16x2(p0, p1);
          }
          tmem_st16_nowait(t_s + c * 16, pk);
        }
        tmem_wait_st();
        l_run += (acc2[0].x + acc2[0].y) + (acc2[1].x + acc2[1].y);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + 8 * t);
      }
      if (!ok) break;
      if (!mbar_wait_warp(o_done + 8 * t, i & 1, abort_flag, err, kErrTimeoutAttnSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int qrow = q0 + t * ABM + r;
      if (args.part_nslots > 1) {
        // partial result of this key range: unnormalised O, running max (log2 units), row sum
        const int64_t prow =
            (int64_t)(args.part_slot0 + split) * args.part_rows + ((int64_t)b * args.heads + h) * args.Lq + qrow;
        float4* dst = reinterpret_cast<float4*>(args.o_part + prow * AD);
#pragma unroll
        for (int c = 0; c < AD / 32; ++c) {
          float o[32];
          tmem_ld32(t_o + c * 32, o);
          if (qrow < args.Lq) {
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[c * 8 + q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
          }
        }
        if (qrow < args.Lq) *reinterpret_cast<float2*>(args.ml_part + prow * 2) = make_float2(m_used, l_run);
      } else {
        const float inv_l = 1.f / l_run;
        uint4* dst = reinterpret_cast<uint4*>(args.o + (int64_t)b * args.o_batch_stride +
                                              (int64_t)qrow * args.o_tok_stride + (int64_t)h * AD);
#pragma unroll
        for (int c = 0; c < AD / 32; ++c) {
          float o[32];
          tmem_ld32(t_o + c * 32, o);
          if (qrow < args.Lq) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              w.x = pack_bf16x2(o[q * 8 + 0] * inv_l, o[q * 8 + 1] * inv_l);
              w.y = pack_bf16x2(o[q * 8 + 2] * inv_l, o[q * 8 + 3] * inv_l);
              w.z = pack_bf16x2(o[q * 8 + 4] * inv_l, o[q * 8 + 5] * inv_l);
              w.w = pack_bf16x2(o[q * 8 + 6] * inv_l, o[q * 8 + 7] * inv_l);
              dst[c * 4 + q] = w;
            }
          }
        }
      }
      // O_t has been read into registers: the next unit's first P V may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free + 8 * t);
      jg += nkv;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem_base, A_TMEM_COLS);
}

// Merge of the split-KV partials: one warp per (batch, head, query row), lane l owns head
// dimensions 4l..4l+3.  O = sum_s 2^(m_s - m) O_s / sum_s 2^(m_s - m) l_s with m = max_s m_s.
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a) {
  const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= a.part_rows) return;
  const int q = (int)(w % a.Lq);
  const int64_t bh = w / a.Lq;
  const int h = (int)(bh % a.heads), b = (int)(bh / a.heads);
  float m = -INFINITY;
  for (int s = 0; s < a.part_nslots; ++s) m = fmaxf(m, a.ml_part[(s * a.part_rows + w) * 2]);
  float l = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < a.part_nslots; ++s) {
    const float2 ml = *reinterpret_cast<const float2*>(a.ml_part + (s * a.part_rows + w) * 2);
    const float wgt = ex2_approx(ml.x - m);
    l = fmaf(wgt, ml.y, l);
    const float4 o = reinterpret_cast<const float4*>(a.o_part + (s * a.part_rows + w) * AD)[lane];
    acc.x = fmaf(wgt, o.x, acc.x);
    acc.y = fmaf(wgt, o.y, acc.y);
    acc.z = fmaf(wgt, o.z, acc.z);
    acc.w = fmaf(wgt, o.w, acc.w);
  }
  const float inv = 1.f / l;
  uint2 u;
  u.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  u.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(a.o + (int64_t)b * a.o_batch_stride + (int64_t)q * a.o_tok_stride + (int64_t)h * AD +
                            lane * 4) = u;
}

// ------------------------------------------------------------------ host launcher
int64_t attn_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int kv_splits) {
  return kv_splits > 1 ? (int64_t)kv_splits * batch * heads * q_len * (AD + 2) * 4 : 0;
}

// Host validation of everything but the workspace, shared by every attention entry point (bf16,
// e4m3 and the allocation-free variant); *out = the params with the defaults filled in
// (kv_splits 0 -> 1, part_nslots 0 -> kv_splits).
static int attn_validate_shape(const wanb200_attn_params* p, wanb200_attn_params* out) {
  if (!p) return set_error(WANB200_EINVAL, "attn: null params");
  if (!p->q || !p->k || !p->v || !p->o) return set_error(WANB200_EINVAL, "attn: null q/k/v/o");
  if (p->head_dim != AD) return set_error(WANB200_EINVAL, "attn: head_dim must be 128");
  if (p->batch <= 0 || p->heads <= 0 || p->q_len <= 0 || p->kv_len <= 0)
    return set_error(WANB200_EINVAL, "attn: batch, heads, q_len, kv_len must be positive");
  if (p->batch > 65535 || p->heads > 65535 || p->q_len > (int64_t)INT32_MAX - 2 * ABM ||
      p->kv_len > (int64_t)INT32_MAX - ABN)
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

  wanb200_attn_params pp = *p;  // kv_splits 0 means 1 (no split)
  if (pp.kv_splits == 0) pp.kv_splits = 1;
  if (pp.kv_splits < 1 || pp.kv_splits > 64) return set_error(WANB200_EINVAL, "attn: kv_splits must be 0..64");
  const int nkv = (int)((pp.kv_len + ABN - 1) / ABN);
  const int per = (nkv + pp.kv_splits - 1) / pp.kv_splits;
  if ((int64_t)(pp.kv_splits - 1) * per >= nkv)
    return set_error(WANB200_EINVAL, "attn: kv_splits leaves a split without key tiles (use attn_kv_splits)");
  if (pp.part_nslots == 0) {
    if (pp.part_slot0 != 0 || pp.defer_combine != 0)
      return set_error(WANB200_EINVAL, "attn: part_slot0 / defer_combine need part_nslots > 0");
    pp.part_nslots = pp.kv_splits;
  } else if (pp.part_nslots < 1 || pp.part_nslots > 64 || pp.part_slot0 < 0 ||
             pp.part_slot0 + pp.kv_splits > pp.part_nslots) {
    return set_error(WANB200_EINVAL, "attn: need 0 <= part_slot0 and part_slot0 + kv_splits <= part_nslots <= 64");
  }
  *out = pp;
  return WANB200_OK;
}

// Shape validation plus the caller's workspace (bf16 and e4m3 entry points).
static int attn_validate(const wanb200_attn_params* p, wanb200_attn_params* out) {
  wanb200_attn_params pp;
  const int rc = attn_validate_shape(p, &pp);
  if (rc) return rc;
  const int64_t need = attn_workspace_bytes(pp.batch, pp.heads, pp.q_len, pp.part_nslots);
  if (need > 0 && (!pp.workspace || !aligned16(pp.workspace) || pp.workspace_bytes < need))
    return set_error(WANB200_EINVAL, "attn: partial slots (kv_splits or part_nslots > 1) need a 16-byte aligned "
                                     "workspace of wanb200_attn_workspace_bytes(.., part_nslots)");
  *out = pp;
  return WANB200_OK;
}

int attn_fwd(const wanb200_attn_params* p, cudaStream_t st) {
  wanb200_attn_params pp;
  const int rc = attn_validate(p, &pp);
  if (rc) return rc;
  int* err = device_error_word();
  if (!err) return WANB200_ECUDA;
  return attn_launch(&pp, err, st);
}

int attn_launch(const wanb200_attn_params* p, int* err, cudaStream_t st, const AttnFp8Operands* f8) {
  CUtensorMap tq, tk, tv;
  const int box[4] = {64, 1, ABM, 1};
  if (f8) {  // e4m3 operands: one 128 x 128-byte box per tile
    const int box8[4] = {128, 1, ABM, 1};
    const int64_t dq[4] = {AD, p->heads, p->q_len, p->batch};
    const int64_t sq[4] = {1, AD, p->heads * AD, p->q_len * p->heads * AD};
    int rc = make_tmap_4d_u8(&tq, f8->q8, dq, sq, box8);
    if (rc) return rc;
    const int64_t dk[4] = {AD, p->heads, p->kv_len, p->batch};
    const int64_t sk[4] = {1, AD, p->heads * AD, p->kv_len * p->heads * AD};
    rc = make_tmap_4d_u8(&tk, f8->k8, dk, sk, box8);
    if (rc) return rc;
    const int boxv[4] = {ABN, AD, 1, 1};
    const int64_t dv[4] = {p->kv_len, AD, p->heads, p->batch};
    const int64_t sv[4] = {1, f8->kv_len16, AD * f8->kv_len16, p->heads * AD * f8->kv_len16};
    rc = make_tmap_4d_u8(&tv, f8->v8t, dv, sv, boxv);
    if (rc) return rc;
  } else {
    const int64_t dq[4] = {AD, p->heads, p->q_len, p->batch};
    const int64_t sq[4] = {1, AD, p->q_tok_stride, p->q_batch_stride};
    int rc = make_tmap_4d(&tq, p->q, dq, sq, box);
    if (rc) return rc;
    const int64_t dims[4] = {AD, p->heads, p->kv_len, p->batch};
    const int64_t sk[4] = {1, AD, p->k_tok_stride, p->k_batch_stride};
    rc = make_tmap_4d(&tk, p->k, dims, sk, box);
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
  aa.heads = (int)p->heads;
  aa.scale_log2 = p->softmax_scale * 1.4426950408889634f;
  aa.kv_splits = p->kv_splits;
  aa.kv_tiles_per_split = (int)(((p->kv_len + ABN - 1) / ABN + p->kv_splits - 1) / p->kv_splits);
  aa.part_slot0 = p->part_slot0;
  aa.part_nslots = p->part_nslots > 0 ? p->part_nslots : p->kv_splits;
  aa.part_rows = p->batch * p->heads * p->q_len;
  aa.o_part = reinterpret_cast<float*>(p->workspace);
  aa.ml_part = aa.o_part ? aa.o_part + (int64_t)aa.part_nslots * aa.part_rows * AD : nullptr;
  aa.q_scale = f8 ? f8->q_scale : nullptr;
  aa.k_scale = f8 ? f8->k_scale : nullptr;
  aa.v_scale = f8 ? f8->v_scale : nullptr;
  aa.nqb = (int)((p->q_len + ABM - 1) / ABM);
  aa.nkb = (int)((p->kv_len + ABN - 1) / ABN);
  aa.err = err;

  // the shared-memory opt-in, once per device and variant (any host thread may get here first;
  // setting the attribute twice is harmless, the flag only saves the call)
  static std::atomic<bool> attr_set[kMaxDevices][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return set_error(WANB200_EINVAL, "device index out of range");
  if (!attr_set[dev][f8 ? 1 : 0].load(std::memory_order_acquire)) {
    cudaError_t e = f8 ? cudaFuncSetAttribute(attn_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              A_SMEM_BYTES8)
                       : cudaFuncSetAttribute(attn_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              A_SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(attn)", e);
    attr_set[dev][f8 ? 1 : 0].store(true, std::memory_order_release);
  }
  const int64_t nqp = (p->q_len + 2 * ABM - 1) / (2 * ABM);
  const int64_t gx = nqp * p->kv_splits;
  const int64_t units = gx * p->heads * p->batch;
  if (gx > INT32_MAX || units > INT32_MAX) return set_error(WANB200_EINVAL, "attn: grid too large");
  aa.units = (int)units;
  aa.nqp = (int)nqp;
  if (f8) {
    dim3 grid((unsigned)gx, (unsigned)p->heads, (unsigned)p->batch);
    attn_fp8_kernel<<<grid, A_THREADS, A_SMEM_BYTES8, st>>>(tq, tk, tv, aa);
  } else {  // bf16: persistent, at most one CTA per SM walking the units
    const unsigned grid = (unsigned)std::min<int64_t>(units, num_sms());
    attn_persistent_kernel<<<grid, A_THREADS_P, A_SMEM_BYTES, st>>>(tq, tk, tv, aa);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("attention kernel launch", e);
  if (aa.part_nslots > 1 && !p->defer_combine) {
    attn_combine_kernel<<<(unsigned)((aa.part_rows + 7) / 8), 256, 0, st>>>(aa);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("attn_combine_kernel launch", e);
  }
  return WANB200_OK;
}

// ------------------------------------------------------------------ e4m3 operands
// Q and K: a scale per (batch, head, 128-token block) = amax / 448 and e4m3(x / scale) in
// [B, L, H, 128]; V: e4m3(v / scale) transposed to [B, H, 128, kv_len16] with one scale per
// (batch, head) = amax over the head / 448 (a per-block V scale would have to be folded into
// P, whose small entries would then underflow e4m3).
struct QuantArgs {
  const __nv_bfloat16* src[3];
  int64_t tok_stride[3], batch_stride[3];
  int len[3], nb[3];
  uint8_t* dst[2];  // q8, k8
  float* scale[3];  // q_scale, k_scale, v block amax
  int heads;
};

// One CTA per (batch, head, 128-token block) of q (z % 3 == 0), k (1) or v (2, amax only);
// thread t: token t / 2 of the block, head dims 64 * (t % 2) .. + 63.
__global__ void __launch_bounds__(256) attn_quant_blocks_kernel(const QuantArgs a) {
  __shared__ float red[8];
  const int which = blockIdx.z % 3, b = blockIdx.z / 3, h = blockIdx.y, blk = blockIdx.x;
  if (blk >= a.nb[which]) return;  // CTA-uniform
  const int row = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int tok = blk * ABM + row;
  const bool live = tok < a.len[which];
  uint4 x[8];
  float amax = 0.f;
  if (live) {
    const uint4* src = reinterpret_cast<const uint4*>(a.src[which] + (int64_t)b * a.batch_stride[which] +
                                                      (int64_t)tok * a.tok_stride[which] + h * AD + half * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = src[i];
      float f[8];
      unpack_bf16x8(x[i], f);
#pragma unroll
      for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(f[k]));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  if (threadIdx.x == 0)
    a.scale[which][((int64_t)b * a.heads + h) * a.nb[which] + blk] = which == 2 ? amax : amax / A_E4M3_MAX;
  if (which == 2 || !live) return;
  const float inv = amax > 0.f ? A_E4M3_MAX / amax : 0.f;
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float f[8];
    unpack_bf16x8(x[i], f);
    w[2 * i] = pack_e4m3x2(f[0] * inv, f[1] * inv) | (pack_e4m3x2(f[2] * inv, f[3] * inv) << 16);
    w[2 * i + 1] = pack_e4m3x2(f[4] * inv, f[5] * inv) | (pack_e4m3x2(f[6] * inv, f[7] * inv) << 16);
  }
  uint4* dst = reinterpret_cast<uint4*>(a.dst[which] + (((int64_t)b * a.len[which] + tok) * a.heads + h) * AD +
                                        half * 64);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

struct VtArgs {
  const __nv_bfloat16* v;
  int64_t tok_stride, batch_stride, len16;
  int len, heads, nkb;
  const float* v_amax;
  float* v_scale;
  uint8_t* v8t;
};

// One CTA per (batch, head, 128-key block): e4m3 of the block with the head's scale, transposed
// through shared memory so that each d row of V^T gets 128 consecutive keys.
__global__ void __launch_bounds__(256) attn_quant_vt_kernel(const VtArgs a) {
  __shared__ __align__(16) uint8_t tile[AD][ABN + 16];  // [d][key], rows padded against bank conflicts
  __shared__ float red[8];
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const float* am = a.v_amax + ((int64_t)b * a.heads + h) * a.nkb;
  float m = 0.f;
  for (int i = threadIdx.x; i < a.nkb; i += blockDim.x) m = fmaxf(m, am[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
  if (blk == 0 && threadIdx.x == 0) a.v_scale[(int64_t)b * a.heads + h] = m / A_E4M3_MAX;
  const float inv = m > 0.f ? A_E4M3_MAX / m : 0.f;
  const int key = threadIdx.x >> 1, half = threadIdx.x & 1;
  const int tok = blk * ABN + key;
  float f[64];
  if (tok < a.len) {
    const uint4* src =
        reinterpret_cast<const uint4*>(a.v + (int64_t)b * a.batch_stride + (int64_t)tok * a.tok_stride + h * AD + half * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) unpack_bf16x8(src[i], f + 8 * i);
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) f[i] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < 64; i += 2) {
    const uint32_t pr = pack_e4m3x2(f[i] * inv, f[i + 1] * inv);
    tile[half * 64 + i][key] = (uint8_t)(pr & 0xff);
    tile[half * 64 + i + 1][key] = (uint8_t)(pr >> 8);
  }
  __syncthreads();
  // thread t: d row t / 2, keys 64 * (t % 2) .. + 63 as four 16-byte stores
  const int d = threadIdx.x >> 1, k0 = (threadIdx.x & 1) * 64;
  uint8_t* dst = a.v8t + (((int64_t)b * a.heads + h) * AD + d) * a.len16 + (int64_t)blk * ABN + k0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    if ((int64_t)blk * ABN + k0 + c * 16 < a.len16)
      *reinterpret_cast<uint4*>(dst + c * 16) = *reinterpret_cast<const uint4*>(&tile[d][k0 + c * 16]);
  }
}

// Workspace carve-up of the e4m3 entry point (each region 256-byte aligned).
struct Fp8Layout {
  int64_t q8, k8, v8t, qs, ks, vam, vs, total, len16;
  int nqb, nkb;
};

static Fp8Layout fp8_layout(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len) {
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  Fp8Layout l;
  l.nqb = (int)((q_len + ABM - 1) / ABM);
  l.nkb = (int)((kv_len + ABN - 1) / ABN);
  l.len16 = (kv_len + 15) / 16 * 16;
  int64_t off = 0;
  l.q8 = off;
  off += up(batch * q_len * heads * AD);
  l.k8 = off;
  off += up(batch * kv_len * heads * AD);
  l.v8t = off;
  off += up(batch * heads * AD * l.len16);
  l.qs = off;
  off += up(batch * heads * l.nqb * 4);
  l.ks = off;
  off += up(batch * heads * l.nkb * 4);
  l.vam = off;
  off += up(batch * heads * l.nkb * 4);
  l.vs = off;
  off += up(batch * heads * 4);
  l.total = off;
  return l;
}

int64_t attn_fp8_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len) {
  if (batch <= 0 || heads <= 0 || q_len <= 0 || kv_len <= 0) return 0;
  return fp8_layout(batch, heads, q_len, kv_len).total;
}

int attn_fwd_fp8(const wanb200_attn_fp8_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "attn_fp8: null params");
  wanb200_attn_params pp;
  int rc = attn_validate(&p->attn, &pp);
  if (rc) return rc;
  const Fp8Layout l = fp8_layout(pp.batch, pp.heads, pp.q_len, pp.kv_len);
  if (!p->fp8_workspace || (reinterpret_cast<uintptr_t>(p->fp8_workspace) & 255) || p->fp8_workspace_bytes < l.total)
    return set_error(WANB200_EINVAL, "attn_fp8: needs a 256-byte aligned fp8_workspace of "
                                     "wanb200_attn_fp8_workspace_bytes() bytes");
  int* err = device_error_word();
  if (!err) return WANB200_ECUDA;
  uint8_t* ws = reinterpret_cast<uint8_t*>(p->fp8_workspace);
  QuantArgs qa;
  qa.src[0] = reinterpret_cast<const __nv_bfloat16*>(pp.q);
  qa.src[1] = reinterpret_cast<const __nv_bfloat16*>(pp.k);
  qa.src[2] = reinterpret_cast<const __nv_bfloat16*>(pp.v);
  qa.tok_stride[0] = pp.q_tok_stride;
  qa.tok_stride[1] = pp.k_tok_stride;
  qa.tok_stride[2] = pp.v_tok_stride;
  qa.batch_stride[0] = pp.q_batch_stride;
  qa.batch_stride[1] = pp.k_batch_stride;
  qa.batch_stride[2] = pp.v_batch_stride;
  qa.len[0] = (int)pp.q_len;
  qa.len[1] = qa.len[2] = (int)pp.kv_len;
  qa.nb[0] = l.nqb;
  qa.nb[1] = qa.nb[2] = l.nkb;
  qa.dst[0] = ws + l.q8;
  qa.dst[1] = ws + l.k8;
  qa.scale[0] = reinterpret_cast<float*>(ws + l.qs);
  qa.scale[1] = reinterpret_cast<float*>(ws + l.ks);
  qa.scale[2] = reinterpret_cast<float*>(ws + l.vam);
  qa.heads = (int)pp.heads;
  if ((int64_t)pp.batch * 3 > 65535) return set_error(WANB200_EINVAL, "attn_fp8: batch too large");
  attn_quant_blocks_kernel<<<dim3((unsigned)std::max(l.nqb, l.nkb), (unsigned)pp.heads, (unsigned)(3 * pp.batch)),
                             256, 0, st>>>(qa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("attn_quant_blocks_kernel launch", e);
  VtArgs va;
  va.v = qa.src[2];
  va.tok_stride = pp.v_tok_stride;
  va.batch_stride = pp.v_batch_stride;
  va.len16 = l.len16;
  va.len = (int)pp.kv_len;
  va.heads = (int)pp.heads;
  va.nkb = l.nkb;
  va.v_amax = qa.scale[2];
  va.v_scale = reinterpret_cast<float*>(ws + l.vs);
  va.v8t = ws + l.v8t;
  attn_quant_vt_kernel<<<dim3((unsigned)l.nkb, (unsigned)pp.heads, (unsigned)pp.batch), 256, 0, st>>>(va);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("attn_quant_vt_kernel launch", e);
  AttnFp8Operands f8;
  f8.q8 = ws + l.q8;
  f8.k8 = ws + l.k8;
  f8.v8t = ws + l.v8t;
  f8.q_scale = qa.scale[0];
  f8.k_scale = qa.scale[1];
  f8.v_scale = va.v_scale;
  f8.kv_len16 = l.len16;
  return attn_launch(&pp, err, st, &f8);
}

int attn_kv_splits(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len) {
  // Wave-quantisation model in key-tile units: a CTA costs the key tiles of its split plus a
  // fixed 1.5 (Q load, output epilogue) plus 2.5 when split (fp32 partial stores and the merge
  // pass).  Pick s in 1..4 with the smallest makespan ceil(units*s / SMs) * cost(s); s is capped
  // so that no split is empty.  Short key ranges (cross-attention over 512 keys) stay unsplit.
  const int64_t units = ((q_len + 2 * ABM - 1) / (2 * ABM)) * heads * batch;
  const int nkv = (int)((kv_len + ABN - 1) / ABN);
  const int sms = num_sms();
  int best = 1;
  double best_t = 1e300;
  for (int s = 1; s <= 4; ++s) {
    const int per = (nkv + s - 1) / s;
    if ((int64_t)(s - 1) * per >= nkv) break;
    const double waves = (double)((units * s + sms - 1) / sms);
    const double t = waves * ((double)per + 1.5 + (s > 1 ? 2.5 : 0.0));
    if (t < best_t - 1e-9) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

// ------------------------------------------------------------------ allocation-free variant
// Some callers cannot let a library allocate device memory: applications that hand all GPU memory
// to their own pool or allocator at start-up (an allocation behind their back either fails for
// lack of memory or escapes their accounting), and latency-critical loops that must not pay for
// cudaMalloc / cudaFree, which can block on the device.  wanb200_attn_fwd_noalloc serves them: it
// keeps the split-KV partials in the fixed-size array below instead of a caller-provided or
// library-allocated workspace, and calls no allocating routine.
//
// The array is part of the library image, so every GPU that loads the library holds it until the
// process exits.  All calls on a device share it and it keeps the last call's contents; every
// call overwrites the partials it reads, so nothing has to start at zero.  Calls that overlap on
// the GPU (different streams, no ordering between them) race on the array.
constexpr int64_t kNoAllocScratchBytes = int64_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* g_noalloc_dev[kMaxDevices] = {};
static std::mutex g_noalloc_mu;

// Device address of the array for the current device.  In host code the array's name only stands
// in for the symbol; the address a kernel may use comes from cudaGetSymbolAddress, resolved once
// per device, with that device current, on the first call.
static int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return set_error(WANB200_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_dev[dev]) {
    void* scratch = nullptr;
    e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
    if (e != cudaSuccess) return set_cuda_error("cudaGetSymbolAddress(static attention workspace)", e);
    g_noalloc_dev[dev] = scratch;
  }
  *out = g_noalloc_dev[dev];
  return WANB200_OK;
}

int attn_fwd_noalloc(const wanb200_attn_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "attn_noalloc: null params");
  if (p->part_slot0 || p->part_nslots || p->defer_combine)
    return set_error(WANB200_EINVAL, "attn_noalloc: partial slots (part_slot0, part_nslots, defer_combine) need "
                                     "wanb200_attn_fwd and a caller workspace");
  wanb200_attn_params pp;
  int rc = attn_validate_shape(p, &pp);  // the same checks as every other attention entry point
  if (rc) return rc;
  if (attn_workspace_bytes(pp.batch, pp.heads, pp.q_len, pp.kv_splits) > kNoAllocScratchBytes)
    return set_error(WANB200_EINVAL,
                     "attn_noalloc: the split-KV partials need more than the fixed 16 MiB static workspace "
                     "(kv_splits * batch * heads * q_len * 520 bytes); use fewer splits or wanb200_attn_fwd");
  rc = noalloc_scratch(&pp.workspace);
  if (rc) return rc;
  pp.workspace_bytes = kNoAllocScratchBytes;
  // the library's error word is a __device__ variable too: resolving it allocates nothing
  int* err = device_error_word();
  if (!err) return WANB200_ECUDA;
  return attn_launch(&pp, err, st);
}

}  // namespace wanb200
