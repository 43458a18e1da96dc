// One WanAttentionBlock forward as a single C call: `_FastBlock.forward(x, e, cos, sin, ck, cv)`
// of models/fast_dit.py:260-311 (batched CFG, per-frame modulation, TP by heads).  It queues the
// block's launches on one stream with the library's own launchers, in the order of the Python
// block op (wanb200/block.py):
//    1  h   = LN1(x) * (1 + scale) + shift
//    2  qkv = h W_qkv^T + b                                 [TP: Σq², Σk² per row and 32 columns,
//                                                              reduced, all-reduced]
//    3  q, k = RoPE(x * rsqrt(Σ/C + eps) * γ)                 in place (one GPU: Σ formed here)
//    4  y   = softmax(q k^T / sqrt(d)) v
//    5  x1  = x + (y W_o^T + b_o) * gate2                     [TP: partial -> all-reduce -> residual pass]
//    6  h   = LN3_affine(x1)
//    7  qc  = h W_cq^T + b                                  [TP: Σqc² partials, reduce, all-reduce]
//    8  qc  = qc * rsqrt(Σ/C + eps) * γ
//    9  y   = attention(qc, ck, cv)
//   10  x1 += y W_co^T + b_co                                 [TP: AR path]
//   11  h   = LN2(x1) * (1 + scale) + shift
//   12  f   = gelu_tanh(h W_1^T + b_1)
//   13  out = x1 + (f W_2^T + b_2) * gate5                    [TP: AR path]
// The residual stream x1 is fp32 in the caller's workspace.  The library issues no collective:
// with tp_size > 1 the caller's all_reduce callback queues each in-place sum over the TP group
// on the stream (NCCL, torch.distributed, ...), at the reference's points (fast_dit.py:141, 159,
// 293, 305, 310).
#include "internal.h"

namespace wanb200 {

namespace {

struct BlockLayout {
  int64_t h, qkv, y, cq, f, ss, ssr, x1, part, attn, total;
  int splits_self, splits_cross;
};

int64_t up256(int64_t x) { return (x + 255) / 256 * 256; }

BlockLayout block_layout(int64_t batch, int64_t seq_len, int64_t dim, int64_t local_heads, int64_t ffn_local,
                         int64_t ctx_len, int tp_size) {
  BlockLayout l;
  const int64_t N = batch * seq_len, Cl = local_heads * 128;
  int64_t off = 0;
  l.h = off;
  off += up256(N * dim * 2);
  l.qkv = off;
  off += up256(N * 3 * Cl * 2);
  l.y = off;
  off += up256(N * Cl * 2);
  l.cq = off;
  off += up256(N * Cl * 2);
  l.f = off;
  off += up256(N * ffn_local * 2);
  l.ss = off;  // TP: Σx² chunk partials of q and k, [N, 2 Cl / 32] (the cross-q GEMM: [N, Cl / 32])
  if (tp_size > 1) off += up256(2 * (Cl / 32) * N * 4);
  l.ssr = off;  // TP: the partials reduced per section, all-reduced in place
  if (tp_size > 1) off += up256(3 * N * 4);
  l.x1 = off;
  off += up256(N * dim * 4);
  l.part = off;
  if (tp_size > 1) off += up256(N * dim * 2);
  l.splits_self = attn_kv_splits(batch, local_heads, seq_len, seq_len);
  l.splits_cross = attn_kv_splits(batch, local_heads, seq_len, ctx_len);
  l.attn = off;
  off += up256(std::max(attn_workspace_bytes(batch, local_heads, seq_len, l.splits_self),
                        attn_workspace_bytes(batch, local_heads, seq_len, l.splits_cross)));
  l.total = off;
  return l;
}

bool shape_ok(const wanb200_block_params* p) {
  return p->batch > 0 && p->seq_len > 0 && p->dim > 0 && p->dim % 512 == 0 && p->dim <= 4096 &&
         p->local_heads > 0 && p->ffn_local > 0 && p->ffn_local % 64 == 0 && p->num_frames > 0 &&
         p->seq_len % p->num_frames == 0 && p->ctx_len > 0 && p->tp_size >= 1 && p->tp_size <= 64 &&
         p->local_heads * 128 * p->tp_size == p->dim && p->ckv_tok_stride >= p->local_heads * 128 &&
         p->ckv_batch_stride >= p->ctx_len * p->ckv_tok_stride;
}

}  // namespace

int64_t block_workspace_bytes(int64_t batch, int64_t seq_len, int64_t dim, int64_t local_heads, int64_t ffn_local,
                              int64_t ctx_len, int tp_size) {
  if (batch <= 0 || seq_len <= 0 || dim <= 0 || local_heads <= 0 || ffn_local <= 0 || ctx_len <= 0 || tp_size < 1)
    return 0;
  return block_layout(batch, seq_len, dim, local_heads, ffn_local, ctx_len, tp_size).total;
}

int block_forward(const wanb200_block_params* p, cudaStream_t st) {
  if (!p) return set_error(WANB200_EINVAL, "block: null params");
  if (!shape_ok(p))
    return set_error(WANB200_EINVAL, "block: need dim % 512 == 0 (<= 4096), local_heads * 128 * tp_size == dim, "
                                     "ffn_local % 64 == 0, seq_len a multiple of num_frames, ctx_len > 0 and ck / cv "
                                     "strides covering [B, ctx_len, local_heads, 128]");
  if (!p->x || !p->x_out || p->x == p->x_out)
    return set_error(WANB200_EINVAL, "block: x and x_out must be distinct non-null buffers");
  if (!p->e0 || !p->cos || !p->sin || !p->ck || !p->cv)
    return set_error(WANB200_EINVAL, "block: null e0 / cos / sin / ck / cv");
  const wanb200_block_weights& w = p->w;
  const void* need[] = {w.modulation, w.w_qkv, w.b_qkv, w.g_q, w.g_k, w.w_o, w.b_o, w.ln3_w, w.ln3_b, w.w_cq,
                        w.b_cq, w.g_cq, w.w_co, w.b_co, w.w1, w.b1, w.w2, w.b2};
  for (const void* q : need)
    if (!q) return set_error(WANB200_EINVAL, "block: a weight pointer is null");
  if (p->tp_size > 1 && !p->all_reduce)
    return set_error(WANB200_EINVAL, "block: tp_size > 1 needs the all_reduce callback");
  const BlockLayout l =
      block_layout(p->batch, p->seq_len, p->dim, p->local_heads, p->ffn_local, p->ctx_len, p->tp_size);
  if (!p->workspace || (reinterpret_cast<uintptr_t>(p->workspace) & 255) || p->workspace_bytes < l.total)
    return set_error(WANB200_EINVAL, "block: needs a 256-byte aligned workspace of wanb200_block_workspace_bytes()");

  const int64_t B = p->batch, Lx = p->seq_len, C = p->dim, N = B * Lx, Hl = p->local_heads, Cl = Hl * 128;
  const int64_t Fl = p->ffn_local, tpf = Lx / p->num_frames;
  const bool tp = p->tp_size > 1;
  uint8_t* ws = static_cast<uint8_t*>(p->workspace);
  void* h = ws + l.h;
  void* qkv = ws + l.qkv;
  void* y = ws + l.y;
  void* cq = ws + l.cq;
  void* f = ws + l.f;
  float* ss = reinterpret_cast<float*>(ws + l.ss);
  float* ssr = reinterpret_cast<float*>(ws + l.ssr);
  float* x1 = reinterpret_cast<float*>(ws + l.x1);
  void* part = ws + l.part;
  void* attn_ws = ws + l.attn;
  const int64_t attn_ws_bytes = l.total - l.attn;
  int rc = 0;
  auto all_reduce = [&](void* buf, int64_t count, int dtype) -> int {
    if (!tp) return WANB200_OK;
    const int r = p->all_reduce(buf, count, dtype, p->all_reduce_ctx, st);
    return r ? set_error(WANB200_ECUDA, "block: the all_reduce callback failed") : WANB200_OK;
  };

  auto ln_mod = [&](const void* x, int xf32, int shift, int scale) {
    wanb200_ln_params q = {};
    q.x = x;
    q.x_f32 = xf32;
    q.out = h;
    q.rows = N;
    q.dim = C;
    q.eps = p->eps;
    q.mode = WANB200_LN_MODULATE;
    q.modulation = w.modulation;
    q.e0 = p->e0;
    q.e0_frame_stride = 6 * C;
    q.shift_idx = shift;
    q.scale_idx = scale;
    q.seq_len = Lx;
    q.tokens_per_frame = tpf;
    return layernorm(&q, st);
  };
  auto gemm = [&](const void* a, int64_t K, const void* wt, const void* bias, int64_t Nout, void* d, int epi) {
    wanb200_gemm_params g = {};
    g.a = a;
    g.lda = K;
    g.w = wt;
    g.ldw = K;
    g.d = d;
    g.ldd = Nout;
    g.M = N;
    g.N = Nout;
    g.K = K;
    g.epilogue = epi;
    g.bias = bias;
    g.seq_len = Lx;
    g.tokens_per_frame = tpf;
    return g;
  };
  auto attention = [&](const void* q, int64_t q_tok, const void* k, const void* v, int64_t kv_len, int64_t kv_tok,
                       int64_t kv_batch, void* o, int splits) {
    wanb200_attn_params a = {};
    a.q = q;
    a.q_tok_stride = q_tok;
    a.q_batch_stride = Lx * q_tok;
    a.k = k;
    a.k_tok_stride = kv_tok;
    a.k_batch_stride = kv_batch;
    a.v = v;
    a.v_tok_stride = kv_tok;
    a.v_batch_stride = kv_batch;
    a.o = o;
    a.o_tok_stride = Cl;
    a.o_batch_stride = Lx * Cl;
    a.batch = B;
    a.heads = Hl;
    a.q_len = Lx;
    a.kv_len = kv_len;
    a.head_dim = 128;
    a.softmax_scale = 0.08838834764831845f;  // 128^-1/2
    a.kv_splits = splits;
    a.workspace = attn_ws;
    a.workspace_bytes = attn_ws_bytes;
    return attn_fwd(&a, st);
  };
  auto residual_pass = [&](const void* res, int res_f32, const void* bias, const void* gate_mod, int gate_idx,
                           void* out, int out_f32) {
    wanb200_residual_params r = {};
    r.out = out;
    r.out_f32 = out_f32;
    r.residual = res;
    r.residual_f32 = res_f32;
    r.y = part;
    r.rows = N;
    r.dim = C;
    r.bias = bias;
    r.gate_mod = gate_mod;
    if (gate_mod) {
      r.gate_e0 = p->e0 + gate_idx * C;
      r.gate_frame_stride = 6 * C;
      r.seq_len = Lx;
      r.tokens_per_frame = tpf;
    }
    r.nsum = 1;
    return bias_gate_residual(&r, st);
  };
  // a row-parallel projection with its residual epilogue: fused into the GEMM on one GPU; under
  // TP the partial sums are all-reduced first and a residual pass applies bias / gate / residual
  auto projection = [&](const void* a, int64_t K, const void* wt, const void* bias, const void* res, int res_f32,
                        int gate_idx, void* out, int out_f32) -> int {
    const void* gate_mod = gate_idx >= 0 ? static_cast<const uint8_t*>(w.modulation) + gate_idx * C * 2 : nullptr;
    if (tp) {
      wanb200_gemm_params g = gemm(a, K, wt, nullptr, C, part, WANB200_EPI_NONE);
      int r = gemm_bf16(&g, st);
      if (!r) r = all_reduce(part, N * C, 1);
      if (!r) r = residual_pass(res, res_f32, bias, gate_mod, gate_idx, out, out_f32);
      return r;
    }
    wanb200_gemm_params g = gemm(a, K, wt, bias, C, out, gate_idx >= 0 ? WANB200_EPI_BIAS_GATE_RES : WANB200_EPI_BIAS_RES);
    g.residual = res;
    g.ldr = C;
    g.residual_f32 = res_f32;
    g.out_f32 = out_f32;
    if (gate_idx >= 0) {
      g.gate_mod = gate_mod;
      g.gate_e0 = p->e0 + gate_idx * C;
      g.gate_frame_stride = 6 * C;
    }
    return gemm_bf16(&g, st);
  };

  // Σx² of `nsec` sections of Cl columns: on one GPU the norm kernel forms it from the bf16 values
  // (ss NULL); under TP the SUMSQ GEMM's chunk partials ([N, nsec * Cl / 32]) are reduced per
  // section into ssr + sec0 * N and those sums all-reduced
  auto sumsq_tp = [&](int nsec, int64_t sec0) -> int {
    if (!tp) return WANB200_OK;
    wanb200_sumsq_reduce_params r = {};
    r.part = ss;
    r.rows = N;
    r.row_stride = nsec * (Cl / 32);
    r.nsections = nsec;
    r.part0[0] = 0;
    r.part0[1] = Cl / 32;
    r.parts = (int)(Cl / 32);
    r.out = ssr + sec0 * N;
    r.out_stride = N;
    int rc2 = sumsq_reduce(&r, st);
    return rc2 ? rc2 : all_reduce(ssr + sec0 * N, nsec * N, 0);
  };
  auto set_ss = [&](wanb200_qknorm_params& q, int nsec, int64_t sec0) {
    for (int s = 0; s < nsec; ++s) q.ss[s] = tp ? ssr + (sec0 + s) * N : nullptr;
    q.ss_parts = 1;
    q.ss_row_stride = 1;
  };

  // -- self-attention
  if ((rc = ln_mod(p->x, p->x_f32, 0, 1))) return rc;
  {
    wanb200_gemm_params g = gemm(h, C, w.w_qkv, w.b_qkv, 3 * Cl, qkv, tp ? WANB200_EPI_BIAS_SUMSQ : WANB200_EPI_BIAS);
    g.rowss = tp ? ss : nullptr;
    g.ss_cols = tp ? 2 * Cl : 0;
    if ((rc = gemm_bf16(&g, st))) return rc;
  }
  if ((rc = sumsq_tp(2, 0))) return rc;
  {
    wanb200_qknorm_params q = {};
    q.x = qkv;
    q.ld = 3 * Cl;
    q.rows = N;
    q.nsections = 2;
    q.col0[0] = 0;
    q.col0[1] = Cl;
    q.width = Cl;
    set_ss(q, 2, 0);
    q.gamma[0] = w.g_q;
    q.gamma[1] = w.g_k;
    q.inv_dim = 1.f / (float)C;
    q.eps = p->eps;
    q.rope = 1;
    q.cos = p->cos;
    q.sin = p->sin;
    q.seq_len = Lx;
    if ((rc = qk_norm_rope(&q, st))) return rc;
  }
  const uint8_t* qkv8 = static_cast<const uint8_t*>(qkv);
  if ((rc = attention(qkv, 3 * Cl, qkv8 + Cl * 2, qkv8 + 2 * Cl * 2, Lx, 3 * Cl, Lx * 3 * Cl, y, l.splits_self)))
    return rc;
  if ((rc = projection(y, Cl, w.w_o, w.b_o, p->x, p->x_f32, 2, x1, 1))) return rc;

  // -- cross-attention over the cached text K/V
  {
    wanb200_ln_params q = {};
    q.x = x1;
    q.x_f32 = 1;
    q.out = h;
    q.rows = N;
    q.dim = C;
    q.eps = p->eps;
    q.mode = WANB200_LN_AFFINE;
    q.weight = w.ln3_w;
    q.bias = w.ln3_b;
    if ((rc = layernorm(&q, st))) return rc;
  }
  {
    wanb200_gemm_params g = gemm(h, C, w.w_cq, w.b_cq, Cl, cq, tp ? WANB200_EPI_BIAS_SUMSQ : WANB200_EPI_BIAS);
    g.rowss = tp ? ss : nullptr;
    g.ss_cols = tp ? Cl : 0;
    if ((rc = gemm_bf16(&g, st))) return rc;
  }
  if ((rc = sumsq_tp(1, 2))) return rc;
  {
    wanb200_qknorm_params q = {};
    q.x = cq;
    q.ld = Cl;
    q.rows = N;
    q.nsections = 1;
    q.width = Cl;
    set_ss(q, 1, 2);
    q.gamma[0] = w.g_cq;
    q.inv_dim = 1.f / (float)C;
    q.eps = p->eps;
    if ((rc = qk_norm_rope(&q, st))) return rc;
  }
  if ((rc = attention(cq, Cl, p->ck, p->cv, p->ctx_len, p->ckv_tok_stride, p->ckv_batch_stride, y, l.splits_cross)))
    return rc;
  if ((rc = projection(y, Cl, w.w_co, w.b_co, x1, 1, -1, x1, 1))) return rc;

  // -- FFN
  if ((rc = ln_mod(x1, 1, 3, 4))) return rc;
  {
    wanb200_gemm_params g = gemm(h, C, w.w1, w.b1, Fl, f, WANB200_EPI_BIAS_GELU);
    if ((rc = gemm_bf16(&g, st))) return rc;
  }
  return projection(f, Fl, w.w2, w.b2, x1, 1, 5, p->x_out, p->out_f32);
}

}  // namespace wanb200
