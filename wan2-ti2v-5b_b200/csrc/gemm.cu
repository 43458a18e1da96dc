// Persistent tcgen05 GEMM with fused epilogues:  D[M,N] = epi(A[M,K] . W[N,K]^T).
//
// The projections of the Wan2.2 DiT block (`_lin` / `_mm`, models/fast_dit.py:103-109, on
// nn.Linear weights [out, in]): fused QKV (3072 -> 9216), self/cross out-projection,
// cross-q, FFN up (3072 -> 14336, GELU-tanh) and FFN down (14336 -> 3072, gate + residual).
//
// Tile 128 x BN x 64 with BN <= 256 chosen per launch (a multiple of 32; 256 unless a narrower
// tile fills the last wave of the persistent grid better), a TMA ring of 4-6 stages (as many as
// fit: 16 KB of A + BN*128 B of W each), fp32 accumulators in TMEM, two accumulator buffers (2 x 256 columns) so the epilogue
// of tile t overlaps the main loop of tile t+1.  One CTA per SM, tiles strided over the
// persistent grid in grouped order so the CTAs running together share A rows and W.
//
// Warp roles (320 threads):
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM allocator + UMMA issuer (one lane)
//   warps 2..9  epilogue: warp w drains TMEM lanes 32*(w%4)..+31 (= tile rows); the two warps
//               on a lane quarter take alternate 32-column chunks (one tcgen05.ld each), apply
//               the epilogue in fp32 and store.  Two warps per row block double the loads of the
//               residual / gate in flight, which the fp32 residual stream needs to stay hidden
//               behind the next tile's main loop.
#include <atomic>

#include "common.cuh"
#include "internal.h"

namespace wanb200 {

constexpr int GBM = 128, GBN = 256, GBK = 64;
constexpr int G_A_BYTES = GBM * GBK * 2;  // 16 KB
constexpr uint32_t G_TMEM_COLS = 512;

// Shared-memory plan per epilogue.  The scatter epilogue (reduce-scatter fused into the GEMM)
// stages each warp's 32 x 256 output rows in shared memory so that every remote store is one
// coalesced 512-byte row segment (16-byte stores per thread scattered over rows run at a
// fraction of the NVLink bandwidth); it gives up one pipeline stage for the staging buffer.
// The TMA ring has as many stages as fit (at most G_MAX_STAGES): a stage holds the A tile and a
// BN-wide W tile, so narrow tiles get a deeper ring to cover the load latency of short K loops.
constexpr int G_MAX_STAGES = 6;
constexpr int G_EPI_WARPS = 8;
constexpr int G_THREADS = 64 + 32 * G_EPI_WARPS;
constexpr int G_SMEM_LIMIT = 232448;  // 227 KB of dynamic shared memory per CTA
template <int EPI>
struct GemmCfg {
  static constexpr int STAGING_ROW = GBN * 2 + 16;  // padded: the 16-byte row writes of a warp hit distinct banks
  static constexpr int STAGING = EPI == WANB200_EPI_SCATTER ? 4 * 32 * STAGING_ROW : 0;
  static constexpr int FIXED = STAGING + 256 + 1024;  // staging + barriers + alignment slack
};
// The fp32 residual epilogues (GATE_RES / RES with an fp32 residual and output) can pass each
// 32 x 32 accumulator chunk through 4 KB of shared memory per epilogue warp, so that the
// residual loads and the output stores run along rows (8 lanes per 128-byte row segment, 4 rows
// per instruction) instead of one row per lane (32 rows touched by every 16-byte access).  The
// host uses it on 256-wide tiles, where it costs the TMA ring no stage.
constexpr int G_RES_STAGING = G_EPI_WARPS * 32 * 32 * 4;  // 32 KB

struct GemmArgs {
  void* d;  // bf16, or fp32 when out_f32
  int64_t ldd;
  int M, N, K;
  const __nv_bfloat16* bias;
  const void* residual;  // bf16, or fp32 when res_f32
  int64_t ldr;
  int res_f32, out_f32;  // the fp32 residual stream (GATE_RES / RES epilogues)
  const __nv_bfloat16* gate_mod;
  const float* gate_e0;
  int64_t gate_frame_stride;
  int seq_len, tokens_per_frame;
  int64_t row_offset, rows_per_seq;
  float* rowss;  // SUMSQ: [M, ss_cols / 32] chunk partials
  int ss_cols;
  __nv_bfloat16* peer_out[WANB200_MAX_PEERS];
  int npeers, src_rank;
  int64_t shard_rows;
  int bn;  // tile width along N: multiple of 32, <= GBN
  int stages;             // TMA ring depth
  int res_staging;        // bytes of the fp32 residual staging (0 or G_RES_STAGING)
  uint32_t stage_bytes;   // A tile + BN-wide W tile
  uint32_t tiles_bytes;   // stages * stage_bytes
  int* err;
};

// Row r's destination for the fused reduce-scatter: the inbox slice of this source rank on the
// rank that owns r (a uniform select instead of a dynamically indexed parameter array).
__device__ __forceinline__ __nv_bfloat16* scatter_row_ptr(const GemmArgs& a, int row) {
  const int o = (int)((int64_t)row / a.shard_rows);
  __nv_bfloat16* base = a.peer_out[0];
#pragma unroll
  for (int i = 1; i < WANB200_MAX_PEERS; ++i)
    if (o == i) base = a.peer_out[i];
  return base + ((int64_t)a.src_rank * a.shard_rows + row - (int64_t)o * a.shard_rows) * a.ldd;
}

// Grouped rasterisation: tiles are numbered in groups of G_GROUP_M row-blocks; inside a group
// the row-block index runs fastest.  The ~148 tiles in flight then cover ~16 row-blocks x ~9
// column-blocks, so the A rows of the group stay L2-resident while W is streamed once per
// group (instead of once per row-block with a plain row-major order).
constexpr int G_GROUP_M = 16;

__device__ __forceinline__ void tile_origin(int tile, int num_m, int num_n, int bn, int& m0, int& n0) {
  const int per_group = G_GROUP_M * num_n;
  const int g = tile / per_group;
  const int first_m = g * G_GROUP_M;
  const int gm = min(num_m - first_m, G_GROUP_M);
  const int r = tile - g * per_group;
  m0 = (first_m + r % gm) * GBM;
  n0 = (r / gm) * bn;
}

constexpr bool epi_has_residual(int epi) {
  return epi == WANB200_EPI_BIAS_GATE_RES || epi == WANB200_EPI_BIAS_RES;
}

// The residual chunk of `row` at col0 (32 values: 4 x 16 B of bf16, or 8 x 16 B of fp32), loaded
// one chunk ahead of its use so the HBM latency of the residual overlaps the previous chunk's TMEM
// load and arithmetic.
__device__ __forceinline__ void load_residual_chunk(const GemmArgs& a, int row, int col0, uint4 (&r)[8]) {
  if (row < a.M && col0 < a.N) {
    if (a.res_f32) {
      const uint4* rp =
          reinterpret_cast<const uint4*>(static_cast<const float*>(a.residual) + (int64_t)row * a.ldr + col0);
#pragma unroll
      for (int q = 0; q < 8; ++q) r[q] = rp[q];
    } else {
      const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.residual) +
                                                       (int64_t)row * a.ldr + col0);
#pragma unroll
      for (int q = 0; q < 4; ++q) r[q] = rp[q];
    }
  }
}

// The 32 residual values of a chunk as fp32.
__device__ __forceinline__ void residual_values(const GemmArgs& a, const uint4 (&res)[8], float* r) {
  if (a.res_f32) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      r[4 * q] = __uint_as_float(res[q].x);
      r[4 * q + 1] = __uint_as_float(res[q].y);
      r[4 * q + 2] = __uint_as_float(res[q].z);
      r[4 * q + 3] = __uint_as_float(res[q].w);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) unpack_bf16x8(res[q], r + 8 * q);
  }
}

template <int EPI>
__device__ __forceinline__ void gemm_epilogue_chunk(const GemmArgs& a, float* v, int row, int col0,
                                                    const uint4 (&res)[8], const float* gate_row) {
  if constexpr (EPI != WANB200_EPI_NONE && EPI != WANB200_EPI_SCATTER) {
    const uint4* bp = reinterpret_cast<const uint4*>(a.bias + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float b[8];
      unpack_bf16x8(__ldg(bp + q), b);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[q * 8 + i] += b[i];
    }
  }
  if constexpr (EPI == WANB200_EPI_BIAS_GELU) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
  }
  if constexpr (EPI == WANB200_EPI_BIAS_SILU) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = silu(v[i]);
  }
  if constexpr (EPI == WANB200_EPI_BIAS_GATE_RES || EPI == WANB200_EPI_BIAS_RES) {
    if (row < a.M) {
      float r[32];
      residual_values(a, res, r);
      if constexpr (EPI == WANB200_EPI_BIAS_GATE_RES) {
        const float4* ep = reinterpret_cast<const float4*>(gate_row + col0);
        const uint4* mp = reinterpret_cast<const uint4*>(a.gate_mod + col0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float g[8];
          unpack_bf16x8(__ldg(mp + q), g);
          const float4 e_lo = __ldg(ep + 2 * q), e_hi = __ldg(ep + 2 * q + 1);
          g[0] += e_lo.x; g[1] += e_lo.y; g[2] += e_lo.z; g[3] += e_lo.w;
          g[4] += e_hi.x; g[5] += e_hi.y; g[6] += e_hi.z; g[7] += e_hi.w;
#pragma unroll
          for (int i = 0; i < 8; ++i) v[q * 8 + i] = r[q * 8 + i] + v[q * 8 + i] * g[i];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += r[i];
      }
    }
  }
  if constexpr (EPI == WANB200_EPI_BIAS_SUMSQ) {
    // this chunk's sum of squares, stored once (no atomics); the consumer adds a row's partials
    // in a fixed order
    if (col0 < a.ss_cols && row < a.M) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        s0 = fmaf(v[i], v[i], s0);
        s1 = fmaf(v[i + 1], v[i + 1], s1);
      }
      a.rowss[(int64_t)row * (a.ss_cols >> 5) + (col0 >> 5)] = s0 + s1;
    }
  }
  if (EPI != WANB200_EPI_SCATTER && EPI != WANB200_EPI_BIAS_SUMSQ && a.out_f32) {
    if (row < a.M) {
      float4* dp = reinterpret_cast<float4*>(static_cast<float*>(a.d) + (int64_t)row * a.ldd + col0);
#pragma unroll
      for (int q = 0; q < 8; ++q) dp[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  } else if (row < a.M) {
    __nv_bfloat16* drow;
    if constexpr (EPI == WANB200_EPI_SCATTER)
      drow = scatter_row_ptr(a, row);
    else
      drow = static_cast<__nv_bfloat16*>(a.d) + (int64_t)row * a.ldd;
    uint4* dp = reinterpret_cast<uint4*>(drow + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u;
      u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
      u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
      u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
      u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
      dp[q] = u;
    }
  }
}

// The bf16 pair packed in one 32-bit word, as two floats (exact).
__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// The fp32 residual epilogue of one tile for the epilogue warp on lane quarter `quad` that takes
// the 32-column chunks half, half + 2, ...  Each 32 x 32 accumulator chunk (lane = row after the
// tcgen05.ld) goes to the warp's 4 KB staging buffer and comes back with lane = (sub, cg): rows
// 4i + sub (i = 0..7) of the chunk at columns 4cg..4cg+3, so every residual load and output store
// covers 4 whole 128-byte row segments.  The 16-byte column groups of a staging row are XOR-
// swizzled by the row's low three bits: the row-per-lane writes and the row-segment reads are
// both free of bank conflicts.  The arithmetic per element is gemm_epilogue_chunk's (bias add,
// then r + v * g for GATE_RES, v + r for RES), so both paths give the same bits.
template <int EPI>
__device__ __forceinline__ void residual_tile_staged(const GemmArgs& a, float* stg, uint32_t t_row, int m0, int n0,
                                                     int quad, int half, int lane) {
  const int sub = lane >> 3, cg = lane & 7;
  const int rbase = m0 + quad * 32 + sub;  // the row of i = 0; a lane's rows step by 4
  int fr[8];
  if constexpr (EPI == WANB200_EPI_BIAS_GATE_RES) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = rbase + 4 * i;
      fr[i] = row < a.M ? (int)frame_of_row(row, a.rows_per_seq, a.row_offset, a.seq_len, a.tokens_per_frame) : 0;
    }
  }
  const float* res = static_cast<const float*>(a.residual);
  float* out = static_cast<float*>(a.d);
  const int nchunks = a.bn / 32;
  // r[i]: the residual of row 4i + sub in the current chunk; each is reloaded for the warp's next
  // chunk right after its use, so the loads run under the rest of this chunk and the next
  // chunk's TMEM load
  float4 r[8] = {};
  if (n0 + half * 32 < a.N) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = rbase + 4 * i;
      if (row < a.M) r[i] = *reinterpret_cast<const float4*>(res + (int64_t)row * a.ldr + n0 + half * 32 + 4 * cg);
    }
  }
#pragma unroll 1
  for (int c = half; c < nchunks; c += 2) {
    const int col0 = n0 + c * 32;
    if (col0 >= a.N) break;  // warp-uniform (N is a multiple of 32)
    const bool more = c + 2 < nchunks && col0 + 64 < a.N;
    float v[32];
    tmem_ld32(t_row + c * 32, v);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4*>(stg + lane * 32 + ((q ^ (lane & 7)) << 2)) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    __syncwarp();
    const uint2 bu = __ldg(reinterpret_cast<const uint2*>(a.bias + col0 + 4 * cg));
    const float b[4] = {bf16_lo(bu.x), bf16_hi(bu.x), bf16_lo(bu.y), bf16_hi(bu.y)};
    float gm[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (EPI == WANB200_EPI_BIAS_GATE_RES) {
      const uint2 gu = __ldg(reinterpret_cast<const uint2*>(a.gate_mod + col0 + 4 * cg));
      gm[0] = bf16_lo(gu.x);
      gm[1] = bf16_hi(gu.x);
      gm[2] = bf16_lo(gu.y);
      gm[3] = bf16_hi(gu.y);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rl = 4 * i + sub;
      const int row = m0 + quad * 32 + rl;
      const float4 x = *reinterpret_cast<const float4*>(stg + rl * 32 + ((cg ^ (rl & 7)) << 2));
      if (row < a.M) {
        float xv[4] = {x.x + b[0], x.y + b[1], x.z + b[2], x.w + b[3]};
        const float rv[4] = {r[i].x, r[i].y, r[i].z, r[i].w};
        if constexpr (EPI == WANB200_EPI_BIAS_GATE_RES) {
          const float4 e = __ldg(reinterpret_cast<const float4*>(a.gate_e0 + (int64_t)fr[i] * a.gate_frame_stride +
                                                                 col0 + 4 * cg));
          const float g[4] = {gm[0] + e.x, gm[1] + e.y, gm[2] + e.z, gm[3] + e.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) xv[j] = rv[j] + xv[j] * g[j];
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) xv[j] += rv[j];
        }
        float* orow = out + (int64_t)row * a.ldd + col0 + 4 * cg;
        *reinterpret_cast<float4*>(orow) = make_float4(xv[0], xv[1], xv[2], xv[3]);
        if (more) r[i] = *reinterpret_cast<const float4*>(res + (int64_t)row * a.ldr + col0 + 64 + 4 * cg);
      }
    }
    __syncwarp();  // the staging buffer is rewritten by the next chunk
  }
}

template <int EPI>
__global__ void __launch_bounds__(G_THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t tiles = smem_u32(smem);
  const int GSTAGES = args.stages;
  const uint32_t SB = args.stage_bytes;
  uint8_t* meta = smem + args.tiles_bytes + GemmCfg<EPI>::STAGING + args.res_staging;
  const uint32_t full0 = smem_u32(meta);             // G_MAX_STAGES x 8
  const uint32_t empty0 = full0 + 8 * G_MAX_STAGES;  // G_MAX_STAGES x 8
  const uint32_t tfull0 = empty0 + 8 * G_MAX_STAGES;  // 2 x 8
  const uint32_t tempty0 = tfull0 + 16;            // 2 x 8
  const uint32_t done_bar = tempty0 + 16;          // 8
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(meta + 8 * (2 * G_MAX_STAGES + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* err = args.err;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < GSTAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 32 * G_EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), G_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int bn = args.bn;
  const int num_n = (args.N + bn - 1) / bn;
  const int num_m = (args.M + GBM - 1) / GBM;
  const int num_tiles = num_m * num_n;
  const int kblocks = args.K / GBK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued = 0, last_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int m0, n0;
        tile_origin(tile, num_m, num_n, bn, m0, n0);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag, err, kErrTimeoutGemmProducer)) {
            ok = false;
            break;
          }
          const uint32_t a_dst = tiles + stage * SB;
          mbar_expect_tx(full0 + 8 * stage, G_A_BYTES + bn * GBK * 2);
          tma_load_2d(a_dst, &tmA, full0 + 8 * stage, kb * GBK, m0);
          tma_load_2d(a_dst + G_A_BYTES, &tmB, full0 + 8 * stage, kb * GBK, n0);
          issued |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == GSTAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // let every load in flight land before the CTA's shared memory goes away
        for (int s = 0; s < GSTAGES; ++s)
          if ((issued >> s) & 1) mbar_drain(full0 + 8 * s, (last_phase >> s) & 1, err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(GBM, bn, false, false);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1, abort_flag, err, kErrTimeoutGemmMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * GBN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, err, kErrTimeoutGemmMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = tiles + stage * SB;
          const uint32_t b_addr = a_addr + G_A_BYTES;
#pragma unroll
          for (int kk = 0; kk < GBK / 16; ++kk) {
            umma_bf16(d_tmem, sw128_desc(a_addr + kk * 32, 16, 1024), sw128_desc(b_addr + kk * 32, 16, 1024), idesc,
                      (kb | kk) != 0);
          }
          umma_commit(empty0 + 8 * stage);
          if (++stage == GSTAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull0 + 8 * acc);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // every UMMA issued by this thread has completed once done_bar flips
      umma_commit(done_bar);
      mbar_drain(done_bar, 0, err);
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // which of the two warps on this lane quarter
    const int r = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      if (!mbar_wait_warp(tfull0 + 8 * acc, acc_phase, abort_flag, err, kErrTimeoutGemmEpilogue)) break;
      tc_fence_after();
      int m0, n0;
      tile_origin(tile, num_m, num_n, bn, m0, n0);
      const int row = m0 + r;
      const uint32_t t_row = tmem_base + (uint32_t(quad * 32) << 16) + acc * GBN;
      if constexpr (EPI == WANB200_EPI_SCATTER) {
        // stage this warp's 32 rows (lane = row), then write each row as one 512-byte segment
        // (the first warp of each lane quarter does the whole tile; the second only arrives)
        constexpr int SR = GemmCfg<EPI>::STAGING_ROW;
        uint8_t* stg = smem + args.tiles_bytes + quad * 32 * SR;
        const int ncols = half ? 0 : min(bn, args.N - n0);  // multiple of 32
#pragma unroll 1
        for (int c = 0; c < ncols / 32; ++c) {
          float v[32];
          tmem_ld32(t_row + c * 32, v);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(stg + lane * SR + c * 64 + q * 16) =
                make_uint4(pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]), pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]),
                           pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]), pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]));
        }
        __syncwarp();
#pragma unroll 1
        for (int rr = 0; rr < (half ? 0 : 32); ++rr) {
          const int orow = m0 + quad * 32 + rr;
          if (orow < args.M && lane * 8 < ncols)
            *reinterpret_cast<uint4*>(scatter_row_ptr(args, orow) + n0 + lane * 8) =
                *reinterpret_cast<const uint4*>(stg + rr * SR + lane * 16);
        }
        __syncwarp();
      } else if (epi_has_residual(EPI) && args.res_staging) {
        if constexpr (epi_has_residual(EPI)) {
          float* stg = reinterpret_cast<float*>(smem + args.tiles_bytes + GemmCfg<EPI>::STAGING) + (warp - 2) * 1024;
          residual_tile_staged<EPI>(args, stg, t_row, m0, n0, quad, half, lane);
        }
      } else {
        uint4 res_next[8] = {}, res_cur[8];
        if constexpr (epi_has_residual(EPI)) load_residual_chunk(args, row, n0 + half * 32, res_next);
        // the gate row of this tile row's latent frame (once per tile, not per chunk)
        const float* gate_row = nullptr;
        if constexpr (EPI == WANB200_EPI_BIAS_GATE_RES) {
          const int f = row < args.M ? (int)frame_of_row(row, args.rows_per_seq, args.row_offset, args.seq_len,
                                                         args.tokens_per_frame)
                                     : 0;
          gate_row = args.gate_e0 + (int64_t)f * args.gate_frame_stride;
        }
#pragma unroll 1
        for (int c = half; c < bn / 32; c += 2) {
          const int col0 = n0 + c * 32;
          if (col0 >= args.N) break;  // warp-uniform
#pragma unroll
          for (int q = 0; q < 8; ++q) res_cur[q] = res_next[q];
          if constexpr (epi_has_residual(EPI)) {
            if (c + 2 < bn / 32) load_residual_chunk(args, row, col0 + 64, res_next);
          }
          float v[32];
          tmem_ld32(t_row + c * 32, v);
          gemm_epilogue_chunk<EPI>(args, v, row, col0, res_cur, gate_row);
        }
      }
      tc_fence_before();
      mbar_arrive(tempty0 + 8 * acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, G_TMEM_COLS);
}

// ------------------------------------------------------------------ host launcher
template <int EPI>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& ga, int grid, cudaStream_t st) {
  // the shared-memory opt-in, once per device (setting it twice from racing threads is harmless)
  static std::atomic<bool> attr_set[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return set_error(WANB200_EINVAL, "device index out of range");
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e =
        cudaFuncSetAttribute(gemm_bf16_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM_LIMIT);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(gemm)", e);
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int smem = (int)ga.tiles_bytes + GemmCfg<EPI>::FIXED + ga.res_staging;
  gemm_bf16_kernel<EPI><<<grid, G_THREADS, smem, st>>>(ta, tb, ga);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("gemm_bf16_kernel launch", e);
  return WANB200_OK;
}

// Tile width along N for a launch: the candidate (multiples of 32 from 256 down to 128) with the
// smallest makespan waves * (BN + c), waves = ceil(tiles / SMs) over the persistent grid.  c
// stands for the per-tile cost that does not shrink with BN (the A tile loads, the accumulator
// hand-off); it keeps BN at 256 unless a narrower tile removes a mostly empty last wave.
static int choose_tile_n(int64_t M, int64_t N, int sms) {
  const int64_t num_m = (M + GBM - 1) / GBM;
  int best = GBN;
  double best_t = 1e300;
  for (int bn = GBN; bn >= 128; bn -= 32) {
    const int64_t tiles = num_m * ((N + bn - 1) / bn);
    const double t = (double)((tiles + sms - 1) / sms) * (bn + 64.0);
    if (t < best_t - 1e-9) {
      best_t = t;
      best = bn;
    }
  }
  return best;
}

int gemm_bf16(const wanb200_gemm_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "gemm: null params");
  const int epi = p->epilogue;
  if (epi < WANB200_EPI_NONE || epi > WANB200_EPI_BIAS_SILU) return set_error(WANB200_EINVAL, "gemm: bad epilogue");
  const bool scatter = epi == WANB200_EPI_SCATTER;
  if (!p->a || !p->w || (!p->d && !scatter)) return set_error(WANB200_EINVAL, "gemm: null a/w/d");
  if (p->M <= 0 || p->N <= 0 || p->K <= 0) return set_error(WANB200_EINVAL, "gemm: M, N, K must be positive");
  if (p->K % GBK) return set_error(WANB200_EINVAL, "gemm: K must be a multiple of 64");
  if (p->N % 32) return set_error(WANB200_EINVAL, "gemm: N must be a multiple of 32");
  if (p->M > INT32_MAX / 2 || p->N > INT32_MAX / 2 || p->K > INT32_MAX / 2)
    return set_error(WANB200_EINVAL, "gemm: dimension too large");
  if (p->lda < p->K || p->ldw < p->K || p->ldd < p->N || (p->lda % 8) || (p->ldw % 8) || (p->ldd % 8))
    return set_error(WANB200_EINVAL, "gemm: leading dims must be >= the row length and multiples of 8");
  if (!aligned16(p->a) || !aligned16(p->w) || (!scatter && !aligned16(p->d)))
    return set_error(WANB200_EINVAL, "gemm: a/w/d must be 16-byte aligned");
  if (epi != WANB200_EPI_NONE && !scatter && (!p->bias || !aligned16(p->bias)))
    return set_error(WANB200_EINVAL, "gemm: epilogue needs a 16-byte aligned bias");
  if (scatter) {
    if (p->npeers < 1 || p->npeers > WANB200_MAX_PEERS || p->src_rank < 0 || p->src_rank >= p->npeers ||
        p->shard_rows <= 0 || p->M > (int64_t)p->npeers * p->shard_rows)
      return set_error(WANB200_EINVAL, "gemm: scatter needs 1..8 peers, a valid src_rank and M <= npeers*shard_rows");
    for (int i = 0; i < p->npeers; ++i)
      if (!p->peer_out[i] || !aligned16(p->peer_out[i]))
        return set_error(WANB200_EINVAL, "gemm: scatter peer_out pointers must be non-null and 16-byte aligned");
  }
  if (epi == WANB200_EPI_BIAS_GATE_RES || epi == WANB200_EPI_BIAS_RES) {
    if (!p->residual || !aligned16(p->residual) || p->ldr < p->N || (p->ldr % 8))
      return set_error(WANB200_EINVAL, "gemm: residual epilogue needs an aligned residual with ldr >= N, ldr % 8 == 0");
  } else if (p->residual_f32) {
    return set_error(WANB200_EINVAL, "gemm: residual_f32 applies to the GATE_RES and RES epilogues only");
  }
  if (p->out_f32 && (epi == WANB200_EPI_SCATTER || epi == WANB200_EPI_BIAS_SUMSQ))
    return set_error(WANB200_EINVAL, "gemm: out_f32 does not apply to the SUMSQ and SCATTER epilogues");
  if (epi == WANB200_EPI_BIAS_GATE_RES) {
    if (!p->gate_mod || !p->gate_e0 || !aligned16(p->gate_mod) || !aligned16(p->gate_e0) ||
        (p->gate_frame_stride % 4) || p->seq_len <= 0 || p->tokens_per_frame <= 0 || p->seq_len > INT32_MAX ||
        p->tokens_per_frame > INT32_MAX || p->row_offset < 0 || p->rows_per_seq < 0)
      return set_error(WANB200_EINVAL, "gemm: gate epilogue needs gate_mod, gate_e0, seq_len, tokens_per_frame "
                                       "(row_offset, rows_per_seq >= 0)");
  }
  if (p->tile_n != 0 && (p->tile_n < 64 || p->tile_n > GBN || p->tile_n % 32))
    return set_error(WANB200_EINVAL, "gemm: tile_n must be 0 (library's choice) or a multiple of 32 in 64..256");
  if (epi == WANB200_EPI_BIAS_SUMSQ) {
    if (!p->rowss || p->ss_cols <= 0 || (p->ss_cols % 32) || p->ss_cols > p->N)
      return set_error(WANB200_EINVAL, "gemm: sumsq epilogue needs rowss and ss_cols, a multiple of 32 in 32..N");
  }

  int* err = device_error_word();
  if (!err) return WANB200_ECUDA;
  const int sms = num_sms();
  const int bn = p->tile_n ? p->tile_n : choose_tile_n(p->M, p->N, sms);
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, p->a, p->K, p->M, p->lda, GBK, GBM);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, p->w, p->K, p->N, p->ldw, GBK, bn);
  if (rc) return rc;

  GemmArgs ga;
  ga.d = p->d;
  ga.ldd = p->ldd;
  ga.res_f32 = p->residual_f32 != 0;
  ga.out_f32 = p->out_f32 != 0;
  ga.M = (int)p->M;
  ga.N = (int)p->N;
  ga.K = (int)p->K;
  ga.bias = reinterpret_cast<const __nv_bfloat16*>(p->bias);
  ga.residual = p->residual;
  ga.ldr = p->ldr;
  ga.gate_mod = reinterpret_cast<const __nv_bfloat16*>(p->gate_mod);
  ga.gate_e0 = p->gate_e0;
  ga.gate_frame_stride = p->gate_frame_stride;
  ga.seq_len = (int)(p->seq_len > 0 ? p->seq_len : 1);
  ga.tokens_per_frame = (int)(p->tokens_per_frame > 0 ? p->tokens_per_frame : 1);
  ga.row_offset = p->row_offset;
  ga.rows_per_seq = p->rows_per_seq;
  ga.rowss = p->rowss;
  ga.ss_cols = epi == WANB200_EPI_BIAS_SUMSQ ? (int)p->ss_cols : 0;
  for (int i = 0; i < WANB200_MAX_PEERS; ++i)
    ga.peer_out[i] = reinterpret_cast<__nv_bfloat16*>(i < p->npeers ? p->peer_out[i] : p->peer_out[0]);
  ga.npeers = p->npeers;
  ga.src_rank = p->src_rank;
  ga.shard_rows = p->shard_rows > 0 ? p->shard_rows : 1;
  ga.bn = bn;
  ga.stage_bytes = (uint32_t)(G_A_BYTES + bn * GBK * 2);
  {
    const int fixed = scatter ? GemmCfg<WANB200_EPI_SCATTER>::FIXED : GemmCfg<WANB200_EPI_NONE>::FIXED;
    ga.stages = std::min<int>(G_MAX_STAGES, (G_SMEM_LIMIT - fixed) / (int)ga.stage_bytes);
    // the row-segment fp32 residual epilogue on full-width tiles, where its staging leaves the
    // ring depth as it is (measured at 15708 x 3072 x 3072: +6% GATE_RES, +10% RES; on 128-wide
    // tiles it lost 0-5%, so narrower tiles keep one row per lane)
    ga.res_staging = 0;
    if ((epi == WANB200_EPI_BIAS_GATE_RES || epi == WANB200_EPI_BIAS_RES) && ga.res_f32 && ga.out_f32 &&
        bn == GBN &&
        std::min<int>(G_MAX_STAGES, (G_SMEM_LIMIT - fixed - G_RES_STAGING) / (int)ga.stage_bytes) == ga.stages)
      ga.res_staging = G_RES_STAGING;
  }
  ga.tiles_bytes = (uint32_t)ga.stages * ga.stage_bytes;
  ga.err = err;

  const int64_t tiles = ((p->M + GBM - 1) / GBM) * ((p->N + bn - 1) / bn);
  const int grid = (int)std::min<int64_t>(tiles, sms);
  switch (epi) {
    case WANB200_EPI_NONE: return launch_gemm<WANB200_EPI_NONE>(ta, tb, ga, grid, st);
    case WANB200_EPI_BIAS: return launch_gemm<WANB200_EPI_BIAS>(ta, tb, ga, grid, st);
    case WANB200_EPI_BIAS_GELU: return launch_gemm<WANB200_EPI_BIAS_GELU>(ta, tb, ga, grid, st);
    case WANB200_EPI_BIAS_SILU: return launch_gemm<WANB200_EPI_BIAS_SILU>(ta, tb, ga, grid, st);
    case WANB200_EPI_BIAS_GATE_RES: return launch_gemm<WANB200_EPI_BIAS_GATE_RES>(ta, tb, ga, grid, st);
    case WANB200_EPI_BIAS_RES: return launch_gemm<WANB200_EPI_BIAS_RES>(ta, tb, ga, grid, st);
    case WANB200_EPI_SCATTER: return launch_gemm<WANB200_EPI_SCATTER>(ta, tb, ga, grid, st);
    default: return launch_gemm<WANB200_EPI_BIAS_SUMSQ>(ta, tb, ga, grid, st);
  }
}

}  // namespace wanb200
