"""The DiT block forward on the B200 kernels, behind the reference's per-block call signature.

`FastBlock.forward(x, e, cos, sin, ck, cv) -> x` is `_FastBlock.forward` of
models/fast_dit.py:270-311 (one WanAttentionBlock, batched CFG, per-frame modulation, TP by
heads with in-graph all-reduces).  `FastCrossKV.forward(context) -> (ck, cv)` is
`_FastCrossKV` (fast_dit.py:464-477), run once per generation.

Op sequence of one block (N = B*L tokens, C = 3072, C_l = C / TP, F_l = 14336 / TP):
   1  h   = LN1(x) * (1 + scale) + shift                    layernorm
   2  qkv = h W_qkv^T + b, Σq², Σk² per row and 32 columns  tcgen05 GEMM, SUMSQ epilogue
      [TP: sumsq_reduce, all-reduce Σq², Σk²]
   3  q,k = RoPE(x * rsqrt(Σ/C + eps) * γ)                   qk_norm_rope (in place)
   4  y   = softmax(q k^T / sqrt(d)) v                       flash attention
   5  x1  = x + (y W_o^T + b_o) * gate2                      GEMM, GATE_RES epilogue (x1 fp32)
      [TP: GEMM partial -> all-reduce -> bias_gate_residual]
   6  h   = LN3_affine(x1)
   7  qc  = h W_cq^T + b, Σqc²                              GEMM, SUMSQ  [TP: reduce, all-reduce Σ]
   8  qc  = qc * rsqrt(Σ/C + eps) * γ                        qk_norm_rope (no rotation)
   9  y   = attention(qc, ck, cv)                            flash attention over 512 keys
  10  x1 += y W_co^T + b_co                                  GEMM, RES epilogue [TP: AR path]
  11  h   = LN2(x1) * (1 + scale) + shift
  12  f   = gelu_tanh(h W_1^T + b_1)                         GEMM, GELU epilogue
  13  x1 += (f W_2^T + b_2) * gate5                          GEMM, GATE_RES  [TP: AR path]

The residual stream x1 is fp32 inside the block (the GEMM epilogues and norms read and write it in
fp32); x may come in as bf16 (the reference's dtype, rounded once at the block's output) or fp32
(FastWanDiT keeps it fp32 across all the blocks of a step).  Rounding the stream to bf16 after each
of a block's three updates is the dominant error of a bf16 step: over the 30 layers of config 2
it alone takes the step-0 prediction to ~5e-2 of the fp32 result; keeping it in fp32 leaves the
bf16 roundings of the GEMM and attention operands, ~1e-2.
"""
from __future__ import annotations

import ctypes
import itertools
import weakref

import torch
import torch.distributed as dist

from . import _lib as L
from . import ops
from .weights import BlockWeights

BF16 = torch.bfloat16


class Workspace:
    """Scratch activations of one block forward, allocated once per (device, token count)."""

    def __init__(self, n_tok: int, dim: int, local_dim: int, ffn_local: int, device, tp: bool):
        kw = dict(device=device, dtype=BF16)
        self.h = torch.empty(n_tok, dim, **kw)
        self.qkv = torch.empty(n_tok, 3 * local_dim, **kw)
        self.y = torch.empty(n_tok, local_dim, **kw)
        self.cq = torch.empty(n_tok, local_dim, **kw)
        self.f = torch.empty(n_tok, ffn_local, **kw)
        # TP: Σx² of q and k per row and 32 output columns (the SUMSQ GEMM's chunk partials,
        # [rows, 2P]; the cross-q GEMM writes [rows, P] into the same storage) and their
        # per-section sums, all-reduced (one GPU: the norm kernel forms Σx² itself)
        self.ssp = torch.empty(n_tok * 2 * local_dim // 32, device=device, dtype=torch.float32) if tp else None
        self.ss = torch.empty(3, n_tok, device=device, dtype=torch.float32) if tp else None
        self.part = torch.empty(n_tok, dim, **kw) if tp else None


_WS = {}


def workspace(n_tok, w: BlockWeights, device, tp: bool) -> Workspace:
    key = (str(device), n_tok, w.dim, w.local_dim, w.ffn_local, tp)
    ws = _WS.get(key)
    if ws is None:
        ws = _WS[key] = Workspace(n_tok, w.dim, w.local_dim, w.ffn_local, device, tp)
    return ws


def clear_workspaces():
    _WS.clear()


class FastBlock:
    """One WanAttentionBlock (models/fast_dit.py:260-311) on libwanb200.

    weights: BlockWeights of this TP rank; num_frames: latent frames F (the modulation row of
    token l is frame l // (L / F)); tp_group: torch.distributed group of the TP ranks (None or
    size 1 = single GPU).
    """

    def __init__(self, weights: BlockWeights, num_frames: int, tp_group=None, eps: float = 1e-6, sp=None,
                 attn_fp8: bool = False, tp_chunks: int = 4):
        """sp: a wanb200.comm.KVGather of the sequence-parallel group for Q-local self-attention
        (`WanSelfAttentionSP`, models/dit_attention_sp.py:25-152): x then holds the tokens
        sp.rank*S .. sp.rank*S + S - 1 of every batch element, every op runs on those rows, and
        only K/V are gathered from the group.  None = x holds whole sequences.
        attn_fp8: self-attention through the e4m3 variant (wanb200_attn_fwd_fp8).
        tp_chunks: row blocks of a row-parallel projection whose all-reduces overlap the next
        block's GEMM (TP only)."""
        self.w = weights
        self.num_frames = num_frames
        self.tp_group = tp_group
        self.tp = weights.tp_size > 1
        self.eps = eps
        self.sp = sp
        self.attn_fp8 = attn_fp8
        self.tp_chunks = max(1, int(tp_chunks))

    def _all_reduce(self, t):
        if self.tp:
            dist.all_reduce(t, group=self.tp_group)

    def _qk_proj(self, a, wmat, bias, out, ws, nsec, kind):
        """The projection ahead of a QK-norm (QKV: nsec 2, cross q: 1) and the Σx² operands of
        qk_norm_rope for its nsec sections of local_dim columns: on one GPU None (the norm kernel
        forms Σx² from the bf16 values, as `_tp_rms_qk` does, models/fast_dit.py:138-140); under TP
        the GEMM's chunk partials reduced per section and all-reduced over the group (141, 159)."""
        if not self.tp:
            ops.linear(a, wmat, bias, epilogue=L.EPI_BIAS, out=out, kind=kind)
            return [None] * nsec
        ops.linear(a, wmat, bias, epilogue=L.EPI_BIAS_SUMSQ, out=out, rowss=self._partials(ws, nsec),
                   ss_cols=nsec * self.w.local_dim, kind=kind)
        return self._sumsq(ws, nsec, 0 if nsec == 2 else 2)

    def _sumsq(self, ws, nsec, sec0):
        """TP: the partials of nsec sections reduced per section into ws.ss[sec0:] and all-reduced."""
        P = self.w.local_dim // 32
        part = self._partials(ws, nsec)
        out = ws.ss[sec0:sec0 + nsec]
        ops.sumsq_reduce(part, [s * P for s in range(nsec)], P, out)
        self._all_reduce(out)
        return [out[s] for s in range(nsec)]

    def _partials(self, ws, nsec):
        """ws.ssp as the [rows, nsec * P] output of a SUMSQ GEMM over nsec sections."""
        n = nsec * self.w.local_dim // 32
        return ws.ssp[:ws.h.shape[0] * n].view(ws.h.shape[0], n)

    def _row_parallel(self, a, wmat, part, kind):
        """part = all_reduce(a @ wmat^T) over the TP group: the partial sums of a row-parallel
        projection (`_row_linear`, models/fast_dit.py:126-131).  The rows go in tp_chunks blocks
        of whole 128-row GEMM tiles; block c's all-reduce runs on NCCL's stream while block c+1's
        GEMM runs on this one (the reference also chunks this all-reduce, fast_dit.py:88-99), and
        this stream waits for all of them before the bias / gate / residual pass reads part."""
        M = a.shape[0]
        n = max(1, min(self.tp_chunks, M // 1024))
        bounds = [0] + [min(M, (M * i // n + 127) // 128 * 128) for i in range(1, n)] + [M]
        works = []
        for r0, r1 in zip(bounds[:-1], bounds[1:]):
            if r1 > r0:
                ops.linear(a[r0:r1], wmat, None, epilogue=L.EPI_NONE, out=part[r0:r1], kind=kind)
                works.append(dist.all_reduce(part[r0:r1], group=self.tp_group, async_op=True))
        t0 = ops.region_begin(part)
        for wk in works:
            wk.wait()
        ops.region_end(part, t0, "tp_allreduce_exposed", 2.0 * part.numel())

    def forward(self, x, e, cos, sin, ck, cv):
        """x [B, L, C] bf16 or fp32 (the residual stream); e [1, F, 6, C] per-frame time projection
        (any float dtype); cos/sin [1, L, 1, 64] fp32; ck/cv [B, Lc, H_local, 128] bf16 -> new x
        [B, L, C] in x's dtype (fp32 inside the block either way)."""
        w, sp = self.w, self.sp
        B, Lx, C = x.shape  # Lx: rows per batch element held here (the shard length under sp)
        nf = self.num_frames
        L_seq = sp.L if sp is not None else Lx
        if L_seq % nf:
            raise ValueError(f"sequence length {L_seq} is not a multiple of {nf} frames")
        if sp is not None and (Lx != sp.S or B != sp.B):
            raise ValueError(f"x is [{B}, {Lx}, C]; the sequence-parallel group expects [{sp.B}, {sp.S}, C]")
        tpf = L_seq // nf
        N, Cl, nl = B * Lx, w.local_dim, w.local_heads
        row0 = sp.rank * sp.S if sp is not None else 0
        frames = (L_seq, tpf, row0, Lx) if sp is not None else (Lx, tpf)
        xf = x.reshape(N, C)
        if not xf.is_contiguous():
            xf = xf.contiguous()
        e0 = e.reshape(-1, 6, C)
        if e0.dtype != torch.float32 or not e0.is_contiguous():
            e0 = e0.float().contiguous()
        if e0.shape[0] != nf:
            raise ValueError(f"e has {e0.shape[0]} frames, expected {nf}")
        cos2 = cos.reshape(-1, cos.shape[-1])
        sin2 = sin.reshape(-1, sin.shape[-1])
        if cos2.shape[0] < row0 + Lx:
            raise ValueError(f"RoPE tables have {cos2.shape[0]} rows, need {row0 + Lx} (pad them to SP * S rows)")
        cos2, sin2 = cos2[row0:row0 + Lx], sin2[row0:row0 + Lx]
        if cos2.dtype != torch.float32 or not cos2.is_contiguous():
            cos2, sin2 = cos2.float().contiguous(), sin2.float().contiguous()
        ws = workspace(N, w, x.device, self.tp)
        mod = w.modulation

        # -- self-attention
        ops.layernorm_modulate(xf, mod, e0, 0, 1, frames, out=ws.h, eps=self.eps)
        ssq, ssk = self._qk_proj(ws.h, w.w_qkv, w.b_qkv, ws.qkv, ws, 2, "gemm_qkv")
        ops.qk_norm_rope(ws.qkv, [(0, ssq, w.g_q), (Cl, ssk, w.g_k)], Cl, C, eps=self.eps,
                         cos=cos2, sin=sin2, seq_len=Lx)
        q = ws.qkv[:, :Cl].view(B, Lx, nl, 128)
        y = ws.y.view(B, Lx, nl, 128)
        if sp is None:
            k = ws.qkv[:, Cl:2 * Cl].view(B, Lx, nl, 128)
            v = ws.qkv[:, 2 * Cl:].view(B, Lx, nl, 128)
            ops.attention(q, k, v, out=y, kind="attn_self", fp8=self.attn_fp8)
        elif sp.overlapped:
            # Q-local: the other ranks' K/V cross NVLink while this shard's queries attend the
            # shard's own keys; the remote keys follow and the partials of both are merged
            sp.start(ws.qkv[:, Cl:])
            n_loc, n_rem = sp.valid, sp.remote_len
            s_loc = ops.kv_splits(B, nl, Lx, n_loc) if n_loc else 0
            s_rem = ops.kv_splits(B, nl, Lx, n_rem) if n_rem else 0
            n = s_loc + s_rem
            if n_loc:
                k = ws.qkv[:, Cl:2 * Cl].view(B, Lx, nl, 128)[:, :n_loc]
                v = ws.qkv[:, 2 * Cl:].view(B, Lx, nl, 128)[:, :n_loc]
                ops.attention(q, k, v, out=y, kind="attn_self", kv_splits=s_loc, parts=(0, n, n_rem > 0),
                              fp8=self.attn_fp8)
            kv = sp.finish()
            if n_rem:
                k = kv[:, :, :Cl].unflatten(2, (nl, 128))
                v = kv[:, :, Cl:].unflatten(2, (nl, 128))
                ops.attention(q, k, v, out=y, kind="attn_self", kv_splits=s_rem, parts=(s_loc, n, False),
                              fp8=self.attn_fp8)
        else:  # Q-local over NCCL: gather the whole sequence's keys, then one attention
            kv = sp.gather(ws.qkv[:, Cl:])[:, :L_seq]
            k = kv[:, :, :Cl].unflatten(2, (nl, 128))
            v = kv[:, :, Cl:].unflatten(2, (nl, 128))
            ops.attention(q, k, v, out=y, kind="attn_self", fp8=self.attn_fp8)
        if xf.dtype not in (BF16, torch.float32):
            raise ValueError(f"x must be bf16 or fp32, not {xf.dtype}")
        x1 = torch.empty(N, C, device=x.device, dtype=torch.float32)  # the fp32 residual stream
        x_out = x1 if xf.dtype == torch.float32 else torch.empty(N, C, device=x.device, dtype=BF16)
        gate2 = (mod[2], e0[:, 2, :])
        if self.tp:
            self._row_parallel(ws.y, w.w_o, ws.part, "gemm_o")
            ops.bias_gate_residual(xf, ws.part, w.b_o, gate=gate2, frames=frames, out=x1)
        else:
            ops.linear(ws.y, w.w_o, w.b_o, epilogue=L.EPI_BIAS_GATE_RES, out=x1, residual=xf, gate=gate2,
                       frames=frames, kind="gemm_o")

        # -- cross-attention (ck/cv cached per generation)
        ops.layernorm_affine(x1, w.ln3_w, w.ln3_b, out=ws.h, eps=self.eps)
        (ssc,) = self._qk_proj(ws.h, w.w_cq, w.b_cq, ws.cq, ws, 1, "gemm_cross_q")
        ops.qk_norm_rope(ws.cq, [(0, ssc, w.g_cq)], Cl, C, eps=self.eps)
        ops.attention(ws.cq.view(B, Lx, nl, 128), ck, cv, out=ws.y.view(B, Lx, nl, 128), kind="attn_cross")
        if self.tp:
            self._row_parallel(ws.y, w.w_co, ws.part, "gemm_cross_o")
            ops.bias_gate_residual(x1, ws.part, w.b_co, out=x1)
        else:
            ops.linear(ws.y, w.w_co, w.b_co, epilogue=L.EPI_BIAS_RES, out=x1, residual=x1, kind="gemm_cross_o")

        # -- FFN
        ops.layernorm_modulate(x1, mod, e0, 3, 4, frames, out=ws.h, eps=self.eps)
        ops.linear(ws.h, w.w1, w.b1, epilogue=L.EPI_BIAS_GELU, out=ws.f, kind="gemm_ffn_up")
        gate5 = (mod[5], e0[:, 5, :])
        if self.tp:
            self._row_parallel(ws.f, w.w2, ws.part, "gemm_ffn_down")
            ops.bias_gate_residual(x1, ws.part, w.b2, gate=gate5, frames=frames, out=x_out)
        else:
            ops.linear(ws.f, w.w2, w.b2, epilogue=L.EPI_BIAS_GATE_RES, out=x_out, residual=x1, gate=gate5,
                       frames=frames, kind="gemm_ffn_down")
        return x_out.view(B, Lx, C)

    __call__ = forward

    # kernel launches per forward at the config-2 shapes (an estimate; the bench counts the
    # launches it makes)
    @property
    def launches(self) -> int:
        n = 13 if not self.tp else 18 + 3 * (self.tp_chunks - 1)
        if self.sp is not None and self.sp.overlapped:
            n += 3  # shard gather + peer barrier + the second attention piece
        return n


class FastCrossKV:
    """A block's cross-attention K (RMS-normed over all heads) and V from the text context,
    once per generation (models/fast_dit.py:464-477)."""

    def __init__(self, weights: BlockWeights, tp_group=None, eps: float = 1e-6):
        self.w, self.tp_group, self.eps = weights, tp_group, eps

    def forward(self, context):
        """context [B, Lc, C] bf16 -> ck, cv [B, Lc, H_x, 128] bf16 (views of one buffer); H_x is
        this rank's heads, or all heads when the weights keep the cross-attention whole."""
        w = self.w
        B, Lc, C = context.shape
        N, Cl, nh = B * Lc, w.cross_dim, w.cross_heads
        ctx = context.reshape(N, C).to(BF16).contiguous()
        if w.tp_size > 1 and not w.local_cross:  # k's Σx² over the group: partials, reduce, all-reduce
            part = torch.empty(N, Cl // 32, device=context.device, dtype=torch.float32)
            kv = ops.linear(ctx, w.w_ckv, w.b_ckv, epilogue=L.EPI_BIAS_SUMSQ, rowss=part, ss_cols=Cl,
                            kind="gemm_cross_kv")
            ss = torch.empty(N, device=context.device, dtype=torch.float32)
            ops.sumsq_reduce(part, [0], Cl // 32, ss)
            dist.all_reduce(ss, group=self.tp_group)
        else:  # the whole k row is here: the norm kernel forms its Σx²
            kv = ops.linear(ctx, w.w_ckv, w.b_ckv, epilogue=L.EPI_BIAS, kind="gemm_cross_kv")
            ss = None
        ops.qk_norm_rope(kv, [(0, ss, w.g_ck)], Cl, C, eps=self.eps)
        ck = kv[:, :Cl].view(B, Lc, nh, 128)
        cv = kv[:, Cl:].view(B, Lc, nh, 128)
        return ck, cv

    __call__ = forward


class SPWorkspace:
    """Scratch of the sequence-parallel block for (device, shard rows S, TP size T)."""

    def __init__(self, S: int, T: int, dim: int, local_dim: int, ffn_local: int, device):
        Np = S * T
        kw = dict(device=device, dtype=BF16)
        self.h_s = torch.empty(S, dim, **kw)
        self.hf = torch.empty(Np, dim, **kw)
        self.qkv = torch.empty(Np, 3 * local_dim, **kw)
        self.y = torch.zeros(Np, local_dim, **kw)  # rows past the real tokens stay zero
        self.part = torch.empty(Np, dim, **kw)
        self.part_s = torch.empty(S, dim, **kw)
        self.cq = torch.empty(S, dim, **kw)
        self.yc = torch.empty(S, dim, **kw)
        self.f = torch.empty(Np, ffn_local, **kw)
        self.ssp = torch.empty(Np, 2 * local_dim // 32, device=device, dtype=torch.float32)  # Σq², Σk² partials
        self.ss = torch.empty(2, Np, device=device, dtype=torch.float32)  # their sums, all-reduced



_SPWS = {}


class FastBlockSP:
    """One WanAttentionBlock with a token-sharded residual stream inside the TP group and local
    all-head cross-attention: `_FastBlockSP.forward(xs, e, oh, cos, sin, ck, cv)` of
    models/fast_dit.py:314-389 with `full_cross` (372-377), batch 1 (CFG-parallel).

    The residual xs [S, C] is rank r's shard (rows r*S .. r*S+S-1) of the flattened tokens,
    zero-padded to T*S rows.  Before the column-parallel QKV / FFN-up GEMMs the normed shard is
    all-gathered; after the row-parallel O / FFN-down GEMMs the partial sums are
    reduce-scattered back to the shard (the bytes of the all-reduce they replace), so the norms,
    gates and residual adds run on S rows.  Cross-attention runs on the shard with all 24 heads
    and whole weights (BlockWeights(local_cross=True)) and needs no collective.  The per-token
    modulation row comes from the global token index (row offset r*S) instead of the
    reference's one-hot matmul.
    """

    def __init__(self, weights: BlockWeights, seq_len: int, num_frames: int, tp_group, eps: float = 1e-6,
                 comm=None):
        """comm: a wanb200.comm.PeerComm of the group to run the all-gathers / reduce-scatters
        fused into the LayerNorm and GEMM kernels over NVLink peer memory; None = NCCL."""
        assert weights.local_cross, "the sequence-parallel block needs BlockWeights(local_cross=True)"
        self.w, self.L, self.num_frames, self.tp_group, self.eps = weights, seq_len, num_frames, tp_group, eps
        self.T, self.rank = weights.tp_size, weights.tp_rank
        self.comm = comm

    def _ln_gather(self, xs, mod, e0, shift, scale, frames, ws):
        """LN + modulation of the shard, all-gathered to [T*S, C]; returns the gathered buffer."""
        if self.comm is not None:
            ops.layernorm_modulate(xs, mod, e0, shift, scale, frames, out=None, eps=self.eps, push=self.comm.push)
            self.comm.barrier()
            return self.comm.hf
        ops.layernorm_modulate(xs, mod, e0, shift, scale, frames, out=ws.h_s, eps=self.eps)
        dist.all_gather_into_tensor(ws.hf, ws.h_s, group=self.tp_group)
        return ws.hf

    def _rowpar_residual(self, a, wmat, bias, residual, gate, frames, out, ws, kind):
        """out = residual + (reduce_scatter(a @ wmat^T) + bias) * gate (row-parallel projection)."""
        if self.comm is not None:
            ops.linear(a, wmat, None, epilogue=L.EPI_SCATTER, scatter=self.comm.scatter, kind=kind)
            self.comm.barrier()
            return ops.bias_gate_residual(residual, self.comm.inbox, bias, gate=gate, frames=frames, out=out,
                                          nsum=self.T)
        ops.linear(a, wmat, None, epilogue=L.EPI_NONE, out=ws.part, kind=kind)
        dist.reduce_scatter_tensor(ws.part_s, ws.part, group=self.tp_group)
        return ops.bias_gate_residual(residual, ws.part_s, bias, gate=gate, frames=frames, out=out)

    def _ws(self, S, device):
        w = self.w
        key = (str(device), S, self.T, w.dim, w.local_dim, w.ffn_local)
        ws = _SPWS.get(key)
        if ws is None:
            ws = _SPWS[key] = SPWorkspace(S, self.T, w.dim, w.local_dim, w.ffn_local, device)
        return ws

    def forward(self, xs, e, cos, sin, ck, cv):
        """xs [S, C] shard, bf16 or fp32 (the residual stream, fp32 inside the block); e [1, F, 6, C];
        cos/sin [1, L, 1, 64] fp32; ck/cv [1, Lc, 24, 128] -> new xs in xs's dtype."""
        w, Lx, nf, g = self.w, self.L, self.num_frames, self.tp_group
        S, C = xs.shape
        N, Cl, nl = Lx, w.local_dim, w.local_heads  # batch 1
        tpf = Lx // nf
        frames_s = (Lx, tpf, self.rank * S)
        e0 = e.reshape(-1, 6, C)
        if e0.dtype != torch.float32 or not e0.is_contiguous():
            e0 = e0.float().contiguous()
        cos2, sin2 = cos.reshape(Lx, -1), sin.reshape(Lx, -1)
        if cos2.dtype != torch.float32 or not cos2.is_contiguous():
            cos2, sin2 = cos2.float().contiguous(), sin2.float().contiguous()
        ws = self._ws(S, xs.device)
        mod = w.modulation

        # -- self-attention: LN on the shard, all-gather, column-parallel QKV on all tokens
        hf = self._ln_gather(xs, mod, e0, 0, 1, frames_s, ws)
        ops.linear(hf, w.w_qkv, w.b_qkv, epilogue=L.EPI_BIAS_SUMSQ, out=ws.qkv, rowss=ws.ssp, ss_cols=2 * Cl,
                   kind="gemm_qkv")
        P = Cl // 32
        ops.sumsq_reduce(ws.ssp, [0, P], P, ws.ss)
        dist.all_reduce(ws.ss, group=g)
        ops.qk_norm_rope(ws.qkv, [(0, ws.ss[0], w.g_q), (Cl, ws.ss[1], w.g_k)], Cl, C, eps=self.eps,
                         cos=cos2, sin=sin2, seq_len=Lx)
        q = ws.qkv[:N, :Cl].view(1, Lx, nl, 128)
        k = ws.qkv[:N, Cl:2 * Cl].view(1, Lx, nl, 128)
        v = ws.qkv[:N, 2 * Cl:].view(1, Lx, nl, 128)
        ops.attention(q, k, v, out=ws.y[:N].view(1, Lx, nl, 128), kind="attn_self")
        if xs.dtype not in (BF16, torch.float32):
            raise ValueError(f"xs must be bf16 or fp32, not {xs.dtype}")
        x1 = torch.empty(S, C, device=xs.device, dtype=torch.float32)  # the fp32 residual stream
        x_out = x1 if xs.dtype == torch.float32 else torch.empty(S, C, device=xs.device, dtype=BF16)
        self._rowpar_residual(ws.y, w.w_o, w.b_o, xs, (mod[2], e0[:, 2, :]), frames_s, x1, ws, "gemm_o")

        # -- cross-attention on the shard, all heads, no collective
        ops.layernorm_affine(x1, w.ln3_w, w.ln3_b, out=ws.h_s, eps=self.eps)
        ops.linear(ws.h_s, w.w_cq, w.b_cq, epilogue=L.EPI_BIAS, out=ws.cq, kind="gemm_cross_q")
        ops.qk_norm_rope(ws.cq, [(0, None, w.g_cq)], C, C, eps=self.eps)  # all heads here: Σx² formed in the norm
        H = w.cross_heads
        ops.attention(ws.cq.view(1, S, H, 128), ck, cv, out=ws.yc.view(1, S, H, 128), kind="attn_cross")
        ops.linear(ws.yc, w.w_co, w.b_co, epilogue=L.EPI_BIAS_RES, out=x1, residual=x1, kind="gemm_cross_o")

        # -- FFN: LN on the shard, all-gather, column/row-parallel GEMMs, reduce-scatter
        hf = self._ln_gather(x1, mod, e0, 3, 4, frames_s, ws)
        ops.linear(hf, w.w1, w.b1, epilogue=L.EPI_BIAS_GELU, out=ws.f, kind="gemm_ffn_up")
        self._rowpar_residual(ws.f, w.w2, w.b2, x1, (mod[5], e0[:, 5, :]), frames_s, x_out, ws, "gemm_ffn_down")
        return x_out

    __call__ = forward

    @property
    def launches(self) -> int:
        return 16



# ---------------------------------------------------------------------------- C entry
_C_WORKSPACES = {}


def block_forward_c(block: FastBlock, x, e, cos, sin, ck, cv, out_dtype=None):
    """The same block through the library's one-call entry point (wanb200_block_forward): every
    launch of the block queued by C on the current stream.  x [B, L, C] bf16 or fp32; returns
    [B, L, C] in out_dtype (default x's dtype).  With TP the C side calls back into
    torch.distributed.all_reduce on the group's buffers (views of the workspace)."""
    if block.sp is not None:
        raise ValueError("block_forward_c covers the whole-sequence block (sp=None)")
    w = block.w
    B, Lx, C = x.shape
    N = B * Lx
    lib = L.load()
    xf = x.reshape(N, C).contiguous()
    out_dtype = out_dtype or x.dtype
    out = torch.empty(N, C, device=x.device, dtype=out_dtype)
    e0 = e.reshape(-1, 6, C).float().contiguous()
    cos2 = cos.reshape(-1, cos.shape[-1])[:Lx].float().contiguous()
    sin2 = sin.reshape(-1, sin.shape[-1])[:Lx].float().contiguous()
    tp = w.tp_size
    nbytes = lib.wanb200_block_workspace_bytes(B, Lx, C, w.local_heads, w.ffn_local, ck.shape[1], tp)
    key = (str(x.device), nbytes)
    ws = _C_WORKSPACES.get(key)
    if ws is None:
        _C_WORKSPACES.clear()
        ws = _C_WORKSPACES[key] = torch.empty(nbytes + 256, dtype=torch.uint8, device=x.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    p = L.BlockParams()
    p.x, p.x_f32, p.x_out, p.out_f32 = xf.data_ptr(), int(xf.dtype == torch.float32), out.data_ptr(), \
        int(out_dtype == torch.float32)
    p.batch, p.seq_len, p.dim, p.local_heads, p.ffn_local = B, Lx, C, w.local_heads, w.ffn_local
    p.num_frames, p.eps = block.num_frames, block.eps
    p.e0, p.cos, p.sin = e0.data_ptr(), cos2.data_ptr(), sin2.data_ptr()
    p.ck, p.cv, p.ctx_len = ck.data_ptr(), cv.data_ptr(), ck.shape[1]
    p.ckv_tok_stride, p.ckv_batch_stride = ck.stride(1), ck.stride(0)
    for f in ("modulation", "w_qkv", "b_qkv", "g_q", "g_k", "w_o", "b_o", "ln3_w", "ln3_b", "w_cq", "b_cq", "g_cq",
              "w_co", "b_co", "w1", "b1", "w2", "b2"):
        setattr(p.w, f, getattr(w, f).data_ptr())
    p.workspace, p.workspace_bytes, p.tp_size = base, nbytes, tp
    if tp > 1:
        u8 = ws

        def all_reduce(buf, count, dtype, ctx, stream):
            try:
                off = buf - ws.data_ptr()
                el = 4 if dtype == 0 else 2
                t = u8[off:off + count * el].view(torch.float32 if dtype == 0 else BF16)
                dist.all_reduce(t, group=block.tp_group)
                return 0
            except Exception:  # reported to the C side as a failed callback
                return 1

        p.all_reduce = L.ALLREDUCE_FN(all_reduce)
    L.check(ops._launch(x, "block", 0.0, lambda: lib.wanb200_block_forward(ctypes.byref(p), ops._stream(x))),
            "wanb200_block_forward")
    return out.view(B, Lx, C)


# ---------------------------------------------------------------------------- torch.library op
# The per-block compiled unit of the reference (`_FastBlock.forward` / `_FastBlockSP.forward`,
# models/fast_dit.py:270, 349, compiled whole at 586 / 646-649) as one custom op, so a step built
# from these blocks traces under torch.compile(fullgraph=True) / make_fx as one opaque node per
# block.  The block's weights and collectives are not tensors of the op: a block object is
# registered once and named by an integer handle (held weakly; it lives as long as its owner).
_BLOCKS = weakref.WeakValueDictionary()
_NEXT_HANDLE = itertools.count(1)


def register_block(block) -> int:
    """Handle of a FastBlock / FastBlockSP for torch.ops.wanb200.block."""
    h = next(_NEXT_HANDLE)
    _BLOCKS[h] = block
    return h


@torch.library.custom_op("wanb200::block", mutates_args=())
def block_op(x: torch.Tensor, e: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, ck: torch.Tensor,
             cv: torch.Tensor, handle: int) -> torch.Tensor:
    """x -> the block's new residual stream (a new tensor of x's shape; no input is modified)."""
    blk = _BLOCKS.get(handle)
    if blk is None:
        raise KeyError(f"wanb200::block: no live block with handle {handle}")
    return blk.forward(x, e, cos, sin, ck, cv)


@block_op.register_fake
def _(x, e, cos, sin, ck, cv, handle):
    return torch.empty_like(x)
