"""CPU fp32 restatement of the tensor-parallel block decomposition — TEST INFRASTRUCTURE ONLY.

The reference shards the block by heads (models/tp_utils.py:378-458) and all-reduces
  * the QK-norm sum of squares (fast_dit.py:141, `_tp_rms_qk`) and the cross-q one (159),
  * the row-parallel partial sums after the self out-projection (293), the cross
    out-projection (305) and the FFN down-projection (310), adding the full bias afterwards
    (`_row_linear`, 126-131).
`block_fwd_tp` runs one rank's share of that on the CPU in fp32, from the rank's
`wanb200.BlockWeights` slices, with a caller-supplied `all_reduce` (gloo in the tests), in the
same op order as `wanb200.block.FastBlock`'s TP branch.  Summed over ranks it must equal the
unsharded `dit_ref.block_fwd`.  `block_fwd_sp` restates the token-sharded residual layout
(`_FastBlockSP`) and `block_fwd_qsp` the Q-local sequence-parallel one (local queries, K/V
all-gathered, TP inside) the same way.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .dit_ref import EPS, attn, per_frame, rope


def block_fwd_tp(w, x, e0, cos, sin, ck, cv, nf: int, all_reduce):
    """w: this rank's BlockWeights (any device; used as fp32 CPU); x [B, L, C] fp32 (full);
    e0 [1, F, 6, C]; ck/cv [B, Lc, n_local, d] of this rank's heads -> x [B, L, C]."""
    f = {k: getattr(w, k).float().cpu() for k in ("modulation", "w_qkv", "b_qkv", "g_q", "g_k", "w_o", "b_o", "ln3_w",
                                                   "ln3_b", "w_cq", "b_cq", "g_cq", "w_co", "b_co", "w1", "b1",
                                                   "w2", "b2")}
    B, L, C = x.shape
    Cl, nl = w.local_dim, w.local_heads
    em = f["modulation"].reshape(1, 6, C).unsqueeze(0) + e0  # [1, F, 6, C]
    e = [t.squeeze(2) for t in em.chunk(6, dim=2)]

    def mod(h, shift, scale):
        return (per_frame(h, nf) * (1 + scale.unsqueeze(2)) + shift.unsqueeze(2)).view(B, L, C)

    def gate(y, g):
        return (per_frame(y, nf) * g.unsqueeze(2)).view(B, L, C)

    h = mod(F.layer_norm(x, (C,), eps=EPS), e[0], e[1])
    qkv = F.linear(h, f["w_qkv"], f["b_qkv"])
    q, k, v = qkv[..., :Cl], qkv[..., Cl:2 * Cl], qkv[..., 2 * Cl:]
    ss = torch.stack([q.pow(2).sum(-1), k.pow(2).sum(-1)])
    all_reduce(ss)
    q = q * torch.rsqrt(ss[0] / C + EPS).unsqueeze(-1) * f["g_q"]
    k = k * torch.rsqrt(ss[1] / C + EPS).unsqueeze(-1) * f["g_k"]
    q = rope(q.reshape(B, L, nl, 128), cos, sin)
    k = rope(k.reshape(B, L, nl, 128), cos, sin)
    y = attn(q, k, v.reshape(B, L, nl, 128)).reshape(B, L, Cl)
    part = F.linear(y, f["w_o"])
    all_reduce(part)
    x = x + gate(part + f["b_o"], e[2])
    h = F.layer_norm(x, (C,), f["ln3_w"], f["ln3_b"], eps=EPS)
    qc = F.linear(h, f["w_cq"], f["b_cq"])
    ssc = qc.pow(2).sum(-1)
    all_reduce(ssc)
    qc = (qc * torch.rsqrt(ssc / C + EPS).unsqueeze(-1) * f["g_cq"]).reshape(B, L, nl, 128)
    y = attn(qc, ck, cv).reshape(B, L, Cl)
    part = F.linear(y, f["w_co"])
    all_reduce(part)
    x = x + part + f["b_co"]
    h = mod(F.layer_norm(x, (C,), eps=EPS), e[3], e[4])
    part = F.linear(F.gelu(F.linear(h, f["w1"], f["b1"]), approximate="tanh"), f["w2"])
    all_reduce(part)
    return x + gate(part + f["b2"], e[5])


def block_fwd_sp(w, xs, e0, cos, sin, ck, cv, seq_len: int, nf: int, rank: int, world: int, all_gather,
                 reduce_scatter, all_reduce):
    """One rank's share of the sequence-parallel block (`_FastBlockSP` with local all-head
    cross-attention, models/fast_dit.py:314-389), batch 1, fp32 CPU, in the op order of
    `wanb200.block.FastBlockSP`.  xs [S, C] is the rank's shard of the zero-padded tokens;
    ck/cv [1, Lc, H, d] all heads; w built with local_cross=True.  Returns the new shard."""
    f = {k: getattr(w, k).float().cpu() for k in ("modulation", "w_qkv", "b_qkv", "g_q", "g_k", "w_o", "b_o", "ln3_w",
                                                   "ln3_b", "w_cq", "b_cq", "g_cq", "w_co", "b_co", "w1", "b1",
                                                   "w2", "b2")}
    S, C = xs.shape
    Cl, nl, H = w.local_dim, w.local_heads, w.cross_heads
    L = seq_len
    tpf = L // nf
    frame = ((torch.arange(S) + rank * S) % L) // tpf  # per-row frame of the shard
    em = f["modulation"].reshape(1, 6, C) + e0[0]       # [F, 6, C]
    et = em[frame]                                      # [S, 6, C]

    h = F.layer_norm(xs, (C,), eps=EPS) * (1 + et[:, 1]) + et[:, 0]
    hf = all_gather(h)                                  # [T*S, C]
    qkv = F.linear(hf, f["w_qkv"], f["b_qkv"])
    q, k, v = qkv[:, :Cl], qkv[:, Cl:2 * Cl], qkv[:, 2 * Cl:]
    ss = torch.stack([q.pow(2).sum(-1), k.pow(2).sum(-1)])
    all_reduce(ss)
    q = q * torch.rsqrt(ss[0] / C + EPS).unsqueeze(-1) * f["g_q"]
    k = k * torch.rsqrt(ss[1] / C + EPS).unsqueeze(-1) * f["g_k"]
    q = rope(q[:L].reshape(1, L, nl, 128), cos, sin)
    k = rope(k[:L].reshape(1, L, nl, 128), cos, sin)
    y = attn(q, k, v[:L].reshape(1, L, nl, 128)).reshape(L, Cl)
    y = torch.cat([y, y.new_zeros(hf.shape[0] - L, Cl)])
    part = reduce_scatter(F.linear(y, f["w_o"]))       # [S, C]
    xs = xs + (part + f["b_o"]) * et[:, 2]
    h = F.layer_norm(xs, (C,), f["ln3_w"], f["ln3_b"], eps=EPS)
    qc = F.linear(h, f["w_cq"], f["b_cq"])
    qc = qc * torch.rsqrt(qc.pow(2).mean(-1, keepdim=True) + EPS) * f["g_cq"]
    yc = attn(qc.reshape(1, S, H, 128), ck, cv).reshape(S, C)
    xs = xs + F.linear(yc, f["w_co"], f["b_co"])
    h = F.layer_norm(xs, (C,), eps=EPS) * (1 + et[:, 4]) + et[:, 3]
    hf = all_gather(h)
    part = reduce_scatter(F.linear(F.gelu(F.linear(hf, f["w1"], f["b1"]), approximate="tanh"), f["w2"]))
    return xs + (part + f["b2"]) * et[:, 5]


def block_fwd_qsp(w, xs, e0, cos, sin, ck, cv, seq_len: int, nf: int, rank: int, sp: int, gather_kv, all_reduce):
    """One rank's share of the Q-local sequence-parallel block (`WanSelfAttentionSP`,
    models/dit_attention_sp.py:25-152, for the whole block) with TP inside, fp32 CPU, in the op
    order of `wanb200.block.FastBlock` with a KVGather.  xs [B, S, C] holds tokens
    rank*S .. rank*S + S - 1 of every batch element (the last shard zero-padded); cos/sin
    [1, sp*S, 1, 64] (zero-padded); ck/cv [B, Lc, n_local, d]; gather_kv([B, S, W]) ->
    [B, sp*S, W] concatenates the shards of the SP group; all_reduce sums over the TP group."""
    f = {k: getattr(w, k).float().cpu() for k in ("modulation", "w_qkv", "b_qkv", "g_q", "g_k", "w_o", "b_o", "ln3_w",
                                                   "ln3_b", "w_cq", "b_cq", "g_cq", "w_co", "b_co", "w1", "b1",
                                                   "w2", "b2")}
    B, S, C = xs.shape
    Cl, nl = w.local_dim, w.local_heads
    L = seq_len
    tpf = L // nf
    frame = ((torch.arange(S) + rank * S) % L) // tpf   # frame of each shard row (padding wraps)
    et = (f["modulation"].reshape(1, 6, C) + e0[0])[frame]  # [S, 6, C]
    c, s = cos[:, rank * S:(rank + 1) * S], sin[:, rank * S:(rank + 1) * S]

    h = F.layer_norm(xs, (C,), eps=EPS) * (1 + et[:, 1]) + et[:, 0]
    qkv = F.linear(h, f["w_qkv"], f["b_qkv"])
    q, k, v = qkv[..., :Cl], qkv[..., Cl:2 * Cl], qkv[..., 2 * Cl:]
    ss = torch.stack([q.pow(2).sum(-1), k.pow(2).sum(-1)])
    all_reduce(ss)
    q = rope((q * torch.rsqrt(ss[0] / C + EPS).unsqueeze(-1) * f["g_q"]).reshape(B, S, nl, 128), c, s)
    k = rope((k * torch.rsqrt(ss[1] / C + EPS).unsqueeze(-1) * f["g_k"]).reshape(B, S, nl, 128), c, s)
    kv = gather_kv(torch.cat([k.reshape(B, S, Cl), v], dim=-1))[:, :L]  # [B, L, 2*Cl]
    y = attn(q, kv[..., :Cl].reshape(B, L, nl, 128), kv[..., Cl:].reshape(B, L, nl, 128)).reshape(B, S, Cl)
    part = F.linear(y, f["w_o"])
    all_reduce(part)
    xs = xs + (part + f["b_o"]) * et[:, 2]
    h = F.layer_norm(xs, (C,), f["ln3_w"], f["ln3_b"], eps=EPS)
    qc = F.linear(h, f["w_cq"], f["b_cq"])
    ssc = qc.pow(2).sum(-1)
    all_reduce(ssc)
    qc = (qc * torch.rsqrt(ssc / C + EPS).unsqueeze(-1) * f["g_cq"]).reshape(B, S, nl, 128)
    part = F.linear(attn(qc, ck, cv).reshape(B, S, Cl), f["w_co"])
    all_reduce(part)
    xs = xs + part + f["b_co"]
    h = F.layer_norm(xs, (C,), eps=EPS) * (1 + et[:, 4]) + et[:, 3]
    part = F.linear(F.gelu(F.linear(h, f["w1"], f["b1"]), approximate="tanh"), f["w2"])
    all_reduce(part)
    return xs + (part + f["b2"]) * et[:, 5]
