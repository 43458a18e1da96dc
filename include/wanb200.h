/*
 * wanb200.h -- C ABI of libwanb200.so, the B200 (sm_100a) kernels behind the Wan2.2-TI2V-5B
 * DiT block forward.
 *
 * The reference (yahavb/wan2-ti2v-5b) has no C boundary: its block is the Python unit
 * `_FastBlock.forward(x, e, cos, sin, ck, cv)` (models/fast_dit.py:270-311), built from
 * PyTorch ops (`_lin` fast_dit.py:108, `_modulate` 172-176, `_tp_rms_qk` 134-147, `_tp_rms`
 * 156-160, `_rope` 163-169, `_gate` 179-181) and an attention backend seam
 * `fn(q[B,Lq,n,d], k[B,Lk,n,d], v) -> [B,Lq,n,d]` (`_sdpa` 186-189, `_cte` 228-241,
 * `_nki_cross` 244-255).  Each entry point below replaces one of those ops; the Python package
 * `wanb200` sequences them behind the same call signature.
 *
 * Conventions.  All tensors are device pointers to row-major bf16 ("bf16" below) unless typed
 * float.  Strides are in elements.  `stream` is a cudaStream_t passed as void*.  Every entry
 * point validates its arguments on the host, launches asynchronously on `stream`, and returns
 * 0 or a negative WANB200_E* code; wanb200_last_error() gives a message for the calling
 * thread's last failure.  No entry point allocates device memory: scratch comes from the caller
 * (workspace pointers) or, for wanb200_attn_fwd_noalloc, from an array inside the library, and
 * the device error word is a variable of the library image (see wanb200_device_error).
 */
#ifndef WANB200_H_
#define WANB200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WANB200_OK 0
#define WANB200_EINVAL (-1)   /* bad argument: shape, stride, alignment, null pointer */
#define WANB200_ECUDA (-2)    /* a CUDA runtime/driver call failed */
#define WANB200_EDEVICE (-3)  /* a kernel reported a device-side error (see wanb200_device_error) */

/* ---------------------------------------------------------------- GEMM
 * d[M, N] = epilogue(a[M, K] . w[N, K]^T)  -- nn.Linear with the weight as stored.
 * Replaces `_lin` / `_mm` (fast_dit.py:103-109) and the elementwise ops that follow them:
 *   WANB200_EPI_BIAS          d = acc + bias                                  (_lin)
 *   WANB200_EPI_BIAS_GELU     d = gelu_tanh(acc + bias)                       (ffn[0], ffn[1]; text_embedding)
 *   WANB200_EPI_BIAS_SILU     d = silu(acc + bias)                            (time_embedding[0..1], the
 *                             SiLU in front of time_projection, wan/modules/model.py:381-386)
 *   WANB200_EPI_BIAS_GATE_RES d = residual + (acc + bias) * gate[frame(row)]  (_gate + residual, 294/311)
 *   WANB200_EPI_BIAS_RES      d = residual + acc + bias                       (cross-attn residual, 305)
 *   WANB200_EPI_BIAS_SUMSQ    d = acc + bias; for every 32-column chunk k < P = ss_cols / 32,
 *                             rowss[row*P + k] = sum over the chunk of d^2 (fp32, before rounding)
 *                             -- the partial sums of squares of `_tp_rms_qk` 138-140 / `_tp_rms`
 *                             158.  Each entry is written once by a plain store (no atomics, no
 *                             pre-zeroing), and wanb200_qk_norm_rope or wanb200_sumsq_reduce
 *                             add a row's partials in a fixed order, so the norms are
 *                             bit-reproducible run to run
 *   WANB200_EPI_NONE          d = acc (row-parallel partial sum before the TP all-reduce, 127)
 *   WANB200_EPI_SCATTER       the reduce-scatter half of that all-reduce, fused: row r of acc is
 *                             stored (bf16, over NVLink) into the inbox of its owner o = r / shard_rows,
 *                             peer_out[o] + ((src_rank * shard_rows) + r - o * shard_rows) * ldd;
 *                             d is unused.  The owner sums the slices (wanb200_bias_gate_residual
 *                             with nsum) after a wanb200_peer_barrier.
 * gate[f, n] = gate_mod[n] + gate_e0[f * gate_frame_stride + n] (modulation + e0 chunk,
 * fast_dit.py:276-277), frame(row) = (token(row) % seq_len) / tokens_per_frame with
 * token(row) = (rows_per_seq > 0 ? row % rows_per_seq : row) + row_offset.
 * For a whole sequence row_offset = rows_per_seq = 0; for a token shard of the flattened
 * sequence row_offset is the index of row 0; for a [batch, shard] buffer holding tokens
 * row_offset .. row_offset + rows_per_seq - 1 of every batch element, rows_per_seq = shard.
 * Limits: K % 64 == 0, N % 32 == 0, lda/ldw/ldd/ldr % 8 == 0, 16-byte aligned pointers.
 * d may alias residual (in place). */
#define WANB200_EPI_NONE 0
#define WANB200_EPI_BIAS 1
#define WANB200_EPI_BIAS_GELU 2
#define WANB200_EPI_BIAS_GATE_RES 3
#define WANB200_EPI_BIAS_RES 4
#define WANB200_EPI_BIAS_SUMSQ 5
#define WANB200_EPI_SCATTER 6
#define WANB200_EPI_BIAS_SILU 7
#define WANB200_MAX_PEERS 8

typedef struct wanb200_gemm_params {
  const void* a; int64_t lda;      /* [M, K] bf16 */
  const void* w; int64_t ldw;      /* [N, K] bf16 */
  void* d; int64_t ldd;            /* [M, N] bf16 */
  int64_t M, N, K;
  int epilogue;                    /* WANB200_EPI_* */
  const void* bias;                /* [N] bf16 (required unless EPI_NONE) */
  const void* residual; int64_t ldr;               /* [M, N] bf16 for *_RES */
  const void* gate_mod;                            /* [N] bf16 for GATE_RES */
  const float* gate_e0; int64_t gate_frame_stride; /* e0 row of frame 0, stride between frames */
  int64_t seq_len, tokens_per_frame, row_offset, rows_per_seq; /* frame(row) for GATE_RES */
  float* rowss; int64_t ss_cols;   /* SUMSQ: [M, ss_cols / 32] fp32 partials; ss_cols % 32 == 0, <= N */
  void* peer_out[WANB200_MAX_PEERS]; int npeers; int src_rank; int64_t shard_rows; /* SCATTER */
  int tile_n;  /* tile width along N: 0 = the library's choice (fills the SMs' last wave), else a
                * multiple of 32 in 64..256 (for tuning; results do not depend on it) */
  /* fp32 residual stream: residual_f32 != 0 (GATE_RES / RES only) reads residual as fp32
   * [M, ldr]; out_f32 != 0 (every epilogue but SUMSQ and SCATTER) writes d as fp32 [M, ldd]
   * (strides still in elements).  The sums x + y stay in fp32 across a step instead of being
   * rounded to bf16 after every block's three updates, the dominant error of a 30-layer bf16
   * step; the patch embedding writes the stream's first value and the time embedding its
   * fp32 modulation rows the same way. */
  int residual_f32, out_f32;
} wanb200_gemm_params;

int wanb200_gemm_bf16(const wanb200_gemm_params* p, void* stream);

/* ---------------------------------------------------------------- attention
 * o[b, i, h, :] = softmax_j(q[b,i,h,:] . k[b,j,h,:] * softmax_scale) v[b, j, h, :]
 * Exact (online-softmax) non-causal attention, head_dim 128, any q_len / kv_len >= 1.
 * Replaces the attention seam `_sdpa` (fast_dit.py:186-189) / `_cte` (228-241) / the NKI NST
 * kernel `wan_flash_self_attn` (kernels/self_attention_nst.py:49-117) for self-attention and
 * `_nki_cross` / `wan_cross_attn` (kernels/cross_attention.py:17-123) for cross-attention.
 * Layout [B, L, H, 128] with the head stride fixed at 128 and token / batch strides given, so
 * q, k and v may be column slices of one fused QKV buffer.
 * Limits: head_dim == 128, strides % 8 == 0, 16-byte aligned pointers. */
typedef struct wanb200_attn_params {
  const void* q; int64_t q_tok_stride, q_batch_stride;
  const void* k; int64_t k_tok_stride, k_batch_stride;
  const void* v; int64_t v_tok_stride, v_batch_stride;
  void* o; int64_t o_tok_stride, o_batch_stride;
  int64_t batch, heads, q_len, kv_len, head_dim;
  float softmax_scale;
  /* split-KV (flash-decoding style) for grids that fill the SMs in few waves: kv_splits CTAs
   * per query tile each take a contiguous range of key tiles and write unnormalised partials
   * (workspace, wanb200_attn_workspace_bytes() bytes) that a merge kernel combines.  0 or 1 =
   * no split; wanb200_attn_kv_splits() gives the split count the library would pick. */
  int kv_splits; void* workspace; int64_t workspace_bytes;
  /* partial slots, for one attention over a key set given in pieces (e.g. the keys of this rank
   * while the other ranks' keys are still in flight, then those): with part_nslots > 0 this
   * launch's kv_splits splits write unnormalised partials into slots part_slot0 .. part_slot0 +
   * kv_splits - 1 of a workspace of wanb200_attn_workspace_bytes(batch, heads, q_len,
   * part_nslots) bytes, and unless defer_combine != 0 the merge of slots 0 .. part_nslots - 1
   * into o follows.  Every slot must have been written (by this or an earlier launch on the
   * stream over the same q) before the merging launch.  0, 0, 0 = the whole key set here. */
  int part_slot0, part_nslots, defer_combine;
} wanb200_attn_params;

int wanb200_attn_fwd(const wanb200_attn_params* p, void* stream);
/* Allocation-free variant of wanb200_attn_fwd (no counterpart in the reference, which has no C
 * boundary).  For callers that cannot have a library allocate device memory: applications that
 * give all GPU memory to their own pool or allocator (an allocation behind their back fails or
 * escapes their accounting) and latency-critical loops that avoid cudaMalloc / cudaFree because
 * those can block on the device.  It takes the same parameters (workspace ignored; partial slots
 * refused) with the same checks and calls no allocating routine: the split-KV partials live in a
 * fixed 16 MiB array inside the library, which every GPU that loads the library holds until the
 * process exits.  Shapes whose partials need more (kv_splits * batch * heads * q_len * 520 bytes
 * > 16 MiB) are rejected with WANB200_EINVAL; kv_splits 0 or 1 needs none.  The first call on a
 * device resolves the array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture.  All calls on a device share the array: calls
 * that overlap on the GPU (unordered streams) race.  Deadline expiries inside its kernels are
 * reported through wanb200_device_error / wanb200_device_error_async like every other entry
 * point's. */
int wanb200_attn_fwd_noalloc(const wanb200_attn_params* p, void* stream);
int64_t wanb200_attn_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int kv_splits);

/* FP8 (e4m3) variant of the attention (no counterpart in the reference, whose trn2 runs never
 * used FP8).  Takes the same bf16 q, k, v, o and options; inside, q and k are quantised with one
 * scale per (batch, head, 128-token block) and v with one per (batch, head) (scale = amax / 448,
 * round to nearest, saturating), the scores and P @ V run as kind::f8f6f4 tcgen05 MMAs with
 * P in e4m3, and the scales are folded into the exponent and the output.  Results differ from
 * the bf16 path by the e4m3 rounding (about 2-3% relative RMS).  fp8_workspace holds the e4m3
 * operands and scales: wanb200_attn_fp8_workspace_bytes() bytes, 256-byte aligned. */
typedef struct wanb200_attn_fp8_params {
  wanb200_attn_params attn;
  void* fp8_workspace; int64_t fp8_workspace_bytes;
} wanb200_attn_fp8_params;

int wanb200_attn_fwd_fp8(const wanb200_attn_fp8_params* p, void* stream);
int64_t wanb200_attn_fp8_workspace_bytes(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len);
int wanb200_attn_kv_splits(int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len);

/* ---------------------------------------------------------------- LayerNorm (+ modulation)
 * mode WANB200_LN_MODULATE: out = LN(x) * (1 + scale[frame]) + shift[frame]
 *   (`blk.norm1/norm2` = WanLayerNorm, wan/modules/model.py:89-99, then `_modulate`,
 *   fast_dit.py:172-176), shift/scale[f, c] = modulation[idx, c] + e0[f, idx, c].
 * mode WANB200_LN_AFFINE: out = LN(x) * weight + bias   (`blk.norm3`, model.py:207-209)
 * LN has no affine in MODULATE mode, eps as given (1e-6).
 * Limits: dim % 256 == 0, dim <= 4096. */
#define WANB200_LN_MODULATE 0
#define WANB200_LN_AFFINE 1

typedef struct wanb200_ln_params {
  const void* x; void* out; int64_t rows, dim; float eps;
  int mode;
  const void* modulation;                 /* [6, dim] bf16 */
  const float* e0; int64_t e0_frame_stride; /* [F, 6, dim] fp32 -> frame stride 6*dim */
  int shift_idx, scale_idx;
  int64_t seq_len, tokens_per_frame, row_offset, rows_per_seq; /* frame(row) as for the GEMM */
  const void* weight; const void* bias;   /* [dim] bf16 for AFFINE */
  /* all-gather fused into the norm: when npush > 0 every output row is also stored at
   * push_out[p] + (push_row0 + row) * dim for p < npush (peer-mapped buffers; out may be NULL) */
  void* push_out[WANB200_MAX_PEERS]; int npush; int64_t push_row0;
  int x_f32;  /* x is fp32 (the fp32 residual stream); out stays bf16 */
  /* e0_one_row != 0: shift and scale both add the same row e0 + frame * e0_frame_stride (the
   * head's modulation `head.modulation + e`, one time-embedding row per frame, fast_dit.py:496-498;
   * modulation is then [2, dim] with shift_idx 0, scale_idx 1) */
  int e0_one_row;
} wanb200_ln_params;

int wanb200_layernorm(const wanb200_ln_params* p, void* stream);

/* ---------------------------------------------------------------- QK RMSNorm + 3-D RoPE
 * In place on column sections of x: y = x * rsqrt(S(row) * inv_dim + eps) * gamma[c], then
 * (if rope) the interleaved-pair rotation with cos/sin[pos, pair], pos = row % seq_len,
 * pair = (c % 128) / 2.  `_tp_rms_qk` + `_rope` (fast_dit.py:134-147, 163-169) for self-attn
 * q and k (nsections 2); `_tp_rms` (fast_dit.py:156-160) for cross-attn q (nsections 1,
 * rope 0).  S(row) is the sum of squares over the global 3072 channels:
 *   ss[s] == NULL (every section): formed here from the section's own bf16 values, which then
 *     hold the whole global dim (one GPU) -- the squares of the rounded values, as the
 *     reference's `q.float().pow(2).sum(-1)`;
 *   else ss_parts partial sums per row and section, S = sum over k < ss_parts of
 *     ss[s][row * ss_row_stride + k] (a SUMSQ GEMM's chunk partials), or ss_parts = 1 for
 *     finished sums (after wanb200_sumsq_reduce and the TP all-reduce), ss_row_stride 1 for a
 *     packed [rows] array.
 * Every sum is added in a fixed order (a warp butterfly, then the row's warps in order), so the
 * results are bit-reproducible run to run.
 * Limits: width % 128 == 0 (<= 4096), ld % 8 == 0, 1 <= ss_parts <= width / 8, ss_row_stride >= ss_parts. */
typedef struct wanb200_qknorm_params {
  void* x; int64_t ld, rows;
  int nsections; int64_t col0[2]; int64_t width;
  const float* ss[2]; const void* gamma[2];
  int ss_parts; int64_t ss_row_stride;  /* 0, 0 are read as 1, 1: one finished sum per row */
  float inv_dim, eps;
  int rope; const float* cos; const float* sin; int64_t seq_len; /* tables [seq_len, 64] fp32 */
} wanb200_qknorm_params;

int wanb200_qk_norm_rope(const wanb200_qknorm_params* p, void* stream);

/* ---------------------------------------------------------------- partial-sum reduction
 * out[s * out_stride + row] = sum over k < parts of part[row * row_stride + part0[s] + k], for
 * s < nsections and row < rows, added in the order k = 0, 1, ... -- the per-rank sums of
 * squares of `_tp_rms_qk` / `_tp_rms` (fast_dit.py:138-140, 158) from the SUMSQ GEMM's chunk
 * partials, before the TP all-reduce of those sums (fast_dit.py:141, 159).
 * Limits: 1 <= nsections <= 2, parts >= 1, part0[s] + parts <= row_stride, out_stride >= rows. */
typedef struct wanb200_sumsq_reduce_params {
  const float* part; int64_t rows, row_stride;
  int nsections; int64_t part0[2]; int parts;
  float* out; int64_t out_stride;
} wanb200_sumsq_reduce_params;

int wanb200_sumsq_reduce(const wanb200_sumsq_reduce_params* p, void* stream);

/* ---------------------------------------------------------------- bias + gate + residual
 * out = residual + (y + bias) * gate[frame(row)]   (gate_mod != NULL)
 * out = residual + y + bias                        (gate_mod == NULL)
 * The tail of `_row_linear` + `_gate` + residual (fast_dit.py:126-131, 179-181, 294, 305, 311)
 * when the projection is row-parallel: y is the all-reduced partial sum (the GEMM ran with
 * WANB200_EPI_NONE; or the nsum inbox slices a WANB200_EPI_SCATTER GEMM wrote).  All tensors
 * [rows, dim] contiguous; out may alias residual.
 * Limits: dim % 8 == 0. */
typedef struct wanb200_residual_params {
  void* out; const void* residual; const void* y; int64_t rows, dim;
  const void* bias;
  const void* gate_mod; const float* gate_e0; int64_t gate_frame_stride;
  int64_t seq_len, tokens_per_frame, row_offset, rows_per_seq; /* frame(row) as for the GEMM */
  int nsum; int64_t y_slice_stride; /* y = sum of nsum slices y + s * y_slice_stride (0/1: y alone) */
  int residual_f32, out_f32;        /* residual / out are fp32 (the fp32 residual stream); y stays bf16 */
} wanb200_residual_params;

int wanb200_bias_gate_residual(const wanb200_residual_params* p, void* stream);

/* ---------------------------------------------------------------- peer barrier
 * Barrier of the `world` ranks of a TP group over NVLink peer memory, the synchronisation step
 * of the fused collectives above.  flags[p] points to rank p's int32[world] flag array
 * (peer-mapped).  This rank stores `epoch` into flags[p][rank] for every p (system-scope
 * release after a system-scope fence), then waits (system-scope acquire) until its own
 * flags[rank][s] >= epoch for every s.  Every rank calls it with the same increasing epochs.
 * The wait is bounded (2 s); on timeout the device error word is set and the kernel returns. */
int wanb200_peer_barrier(int* const* flags, int rank, int world, int epoch, void* stream);

/* ---------------------------------------------------------------- shard gather (push)
 * The K/V all-gather of sequence-parallel self-attention: `WanSelfAttentionSP.forward`
 * (models/dit_attention_sp.py:88-99) all-gathers the normed, rotated k and v of every rank's
 * query shard over the attn-sp group (`ps.all_gather_into_tensor`, parallel_state.py) so each
 * rank attends its own queries to all keys.  Here the owner of a shard stores it into the
 * gathered buffers of the other ranks over NVLink: row i < valid_rows of batch element b of
 * the shard, src + (b * shard_rows + i) * src_ld (width bf16), goes to
 * dst[p] + b * dst_batch_stride + (dst_row0[p] + i) * dst_ld for every p < ndst (peer-mapped
 * buffers; each destination places the shard at its own row; rows >= valid_rows are the padding
 * of the last shard and are not sent).  Every rank calls wanb200_peer_barrier before it reads
 * the gathered rows.
 * Limits: width % 8 == 0, src_ld, dst_ld, dst_batch_stride % 8 == 0, 16-byte aligned pointers. */
typedef struct wanb200_shard_gather_params {
  const void* src; int64_t src_ld;
  int64_t batch, shard_rows, valid_rows, width;
  void* dst[WANB200_MAX_PEERS]; int ndst;
  int64_t dst_ld, dst_batch_stride, dst_row0[WANB200_MAX_PEERS];
} wanb200_shard_gather_params;

int wanb200_shard_gather(const wanb200_shard_gather_params* p, void* stream);

/* ---------------------------------------------------------------- embeddings and head
 * The gathers around the patch-embedding and head GEMMs of the step driver (`_FastPatch`,
 * models/fast_dit.py:527-537; `_FastHead` / `_FastHeadCfgPar` 480-524).
 *
 * wanb200_patchify: the Conv3d patchify (stride = kernel) of a latent [C, F, H, W] (fp32 or
 * bf16) into the patch-embedding GEMM's A operand out [batch, L, C*pf*ph*pw] bf16 (the same rows
 * for every batch copy, the CFG branches), token l = (f*H/ph + h)*W/pw + w, entry
 * k = ((c*pf + i)*ph + j)*pw + u as the Conv3d weight [C_out, C, pf, ph, pw] flattens. */
typedef struct wanb200_patchify_params {
  const void* latent; int latent_f32;
  int64_t channels, frames, height, width;
  int pf, ph, pw;
  int64_t batch;
  void* out;
} wanb200_patchify_params;

int wanb200_patchify(const wanb200_patchify_params* p, void* stream);

/* wanb200_unpatchify_cfg: the head GEMM's output y [batch, L, pf*ph*pw*C] fp32 (row entry
 * ((i*ph + j)*pw + u)*C + c) back to the latent layout out [C, F*pf, H*ph, W*pw] with the CFG
 * combine: WANB200_CFG_COMBINE (batch 2 = cond, uncond): uncond + guide * (cond - uncond);
 * WANB200_CFG_SCALE: guide * y[0] (a CFG-parallel rank's weighted branch, summed over the pair
 * by the caller).  out is bf16 (the reference's output dtype) or fp32 (out_f32). */
#define WANB200_CFG_COMBINE 0
#define WANB200_CFG_SCALE 1

typedef struct wanb200_unpatchify_params {
  const float* y; int64_t batch;
  int64_t frames, height, width;  /* the token grid */
  int pf, ph, pw; int64_t channels;
  int mode; float guide;
  void* out; int out_f32;
} wanb200_unpatchify_params;

int wanb200_unpatchify_cfg(const wanb200_unpatchify_params* p, void* stream);

/* ---------------------------------------------------------------- whole block
 * One WanAttentionBlock forward in one call: `_FastBlock.forward(x, e, cos, sin, ck, cv)`
 * (models/fast_dit.py:260-311; the unit the reference compiles whole, fast_dit.py:586, 646-649)
 * with batched CFG, per-frame modulation and TP by heads.  Queues the block's launches on
 * `stream` (LN1 + modulation, QKV GEMM with the Σq², Σk² epilogue, QK-norm + RoPE,
 * self-attention, out-projection with gate + residual, LN3, cross-q GEMM with Σ, cross-q norm,
 * cross-attention over ck / cv, cross out-projection with residual, LN2 + modulation, FFN up with
 * GELU, FFN down with gate + residual).  The residual stream is fp32 in the workspace; x and
 * x_out are bf16 or fp32 (x_f32, out_f32).  Weights as `shard_model_tp` slices them for this
 * TP rank (tp_utils.py:378-458): w_qkv = [q; k; v] rows of this rank's heads [3*C_l, C], g_q /
 * g_k / g_cq the RMSNorm gains of those heads, w_o / w_co the matching input columns [C, C_l],
 * w1 rows [F_l, C], w2 columns [C, F_l], full biases of the row-parallel projections.
 * The library issues no collective.  With tp_size > 1 the caller's all_reduce callback is called
 * (on the calling thread, in stream order) to queue an in-place sum over the TP group on `stream`
 * at the reference's points (fast_dit.py:141, 159, 293, 305, 310): buf, count elements, dtype
 * 0 = fp32 (the Σx² rows), 1 = bf16 (the projection partial sums); it returns 0 on success.
 * Limits: dim % 512 == 0, dim <= 4096, local_heads * 128 * tp_size == dim, ffn_local % 64 == 0,
 * seq_len a multiple of num_frames; ck / cv [B, ctx_len, local_heads, 128] with the given token
 * and batch strides (e.g. the two halves of the cross K/V buffer). */
typedef int (*wanb200_allreduce_fn)(void* buf, int64_t count, int dtype, void* ctx, void* stream);

typedef struct wanb200_block_weights {
  const void* modulation;                              /* [6, C] */
  const void* w_qkv; const void* b_qkv;                /* [3*C_l, C], [3*C_l] */
  const void* g_q; const void* g_k;                    /* [C_l] */
  const void* w_o; const void* b_o;                    /* [C, C_l], [C] */
  const void* ln3_w; const void* ln3_b;                /* [C] */
  const void* w_cq; const void* b_cq; const void* g_cq; /* [C_l, C], [C_l], [C_l] */
  const void* w_co; const void* b_co;                  /* [C, C_l], [C] */
  const void* w1; const void* b1;                      /* [F_l, C], [F_l] */
  const void* w2; const void* b2;                      /* [C, F_l], [C] */
} wanb200_block_weights;

typedef struct wanb200_block_params {
  const void* x; int x_f32;          /* [B*L, C] residual stream in (bf16, or fp32) */
  void* x_out; int out_f32;          /* [B*L, C] out, distinct from x */
  int64_t batch, seq_len, dim, local_heads, ffn_local, num_frames;
  float eps;                         /* 1e-6 */
  const float* e0;                   /* [F, 6, C] per-frame time projection */
  const float* cos; const float* sin; /* [seq_len, 64] RoPE tables */
  const void* ck; const void* cv; int64_t ctx_len, ckv_tok_stride, ckv_batch_stride;
  wanb200_block_weights w;
  void* workspace; int64_t workspace_bytes; /* 256-byte aligned, wanb200_block_workspace_bytes() */
  int tp_size; wanb200_allreduce_fn all_reduce; void* all_reduce_ctx;
} wanb200_block_params;

int64_t wanb200_block_workspace_bytes(int64_t batch, int64_t seq_len, int64_t dim, int64_t local_heads,
                                      int64_t ffn_local, int64_t ctx_len, int tp_size);
int wanb200_block_forward(const wanb200_block_params* p, void* stream);

/* ---------------------------------------------------------------- status */
const char* wanb200_last_error(void);
/* Device-side error word of the current device: 0 or a code (a bounded wait expired inside a
 * kernel; the first code wins and stays until reset).  Synchronizes the device.  reset != 0
 * clears it.  The word is a __device__ variable of the library (one per device), so neither
 * this call nor any kernel launch allocates for it. */
int wanb200_device_error(int reset);
/* The same word without synchronizing: queues a 4-byte device-to-host copy of it into *host_out
 * on `stream`, behind the work already queued there.  The value is valid once the stream has
 * passed this point (record an event after the call and wait for or query it); host_out should
 * be page-locked for the copy to be asynchronous.  Lets a step driver check every step at no
 * cost to the pipeline (the word is sticky, so a later read also reports an earlier expiry). */
int wanb200_device_error_async(int* host_out, void* stream);
/* Library version, e.g. 201 for 0.2.1. */
int wanb200_version(void);
/* sizeof of the parameter structs (gemm, attn, ln, qknorm, residual, shard_gather, attn_fp8, block,
 * patchify, unpatchify, sumsq_reduce)
 * written to out[0..n); returns the number of structs.  Lets a binding detect a library built
 * from a different header. */
int wanb200_struct_sizes(int64_t* out, int n);

#ifdef __cplusplus
}
#endif

#endif /* WANB200_H_ */
