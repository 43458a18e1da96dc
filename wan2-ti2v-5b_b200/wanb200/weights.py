"""Model description, seeded synthetic weights, and the device-side packing of one block.

Parameters use the HF checkpoint names of Wan2.2-TI2V-5B (`blocks.{i}.self_attn.q.weight`, ...,
`time_embedding.0.weight`, `head.head.weight`; wan/modules/model.py:292-404), so a real
checkpoint's state dict drops in where the seeded one is used here.

`BlockWeights` slices one block for a tensor-parallel rank the way the reference's
`shard_model_tp` does (models/tp_utils.py:378-458): Q/K/V, cross-Q/K/V and FFN-up by output
rows (heads), O / cross-O / FFN-down by input columns, QK-norm gammas by heads, row-parallel
biases kept whole (added once, after the all-reduce).  Q, K and V are concatenated into one
[3*C_local, C] matrix so the block runs a single QKV GEMM.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

BF16 = torch.bfloat16


@dataclass(frozen=True)
class WanSpec:
    """Shape of a WanModel (wan/configs/wan_ti2v_5B.py:19-27 for TI2V-5B)."""
    dim: int = 3072
    ffn_dim: int = 14336
    num_heads: int = 24
    num_layers: int = 30
    freq_dim: int = 256
    text_dim: int = 4096
    in_dim: int = 48
    out_dim: int = 48
    patch_size: tuple = (1, 2, 2)
    text_len: int = 512
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


TI2V_5B = WanSpec()


def _block_shapes(spec: WanSpec):
    C, F = spec.dim, spec.ffn_dim
    shapes = {"modulation": (1, 6, C), "norm3.weight": (C,), "norm3.bias": (C,),
              "ffn.0.weight": (F, C), "ffn.0.bias": (F,), "ffn.2.weight": (C, F), "ffn.2.bias": (C,)}
    for a in ("self_attn", "cross_attn"):
        for p in ("q", "k", "v", "o"):
            shapes[f"{a}.{p}.weight"] = (C, C)
            shapes[f"{a}.{p}.bias"] = (C,)
        shapes[f"{a}.norm_q.weight"] = (C,)
        shapes[f"{a}.norm_k.weight"] = (C,)
    return shapes


def _fill(name: str, shape, gen, device, dim: int):
    """Seeded init used for synthetic runs: weights and biases N(0, 0.02), norm gains
    1 + N(0, 0.1), modulation N(0, 1)/sqrt(dim) (its init scale, model.py:246)."""
    r = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if "norm" in name and name.endswith("weight"):
        r = 1.0 + 0.1 * r
    elif name.endswith("modulation"):
        r = r / dim ** 0.5
    else:
        r = 0.02 * r
    return r.to(BF16)


def random_block_state(spec: WanSpec, seed: int, device="cpu") -> dict:
    gen = torch.Generator(device=device).manual_seed(seed)
    return {k: _fill(k, s, gen, device, spec.dim) for k, s in sorted(_block_shapes(spec).items())}


def model_shapes(spec: WanSpec, num_layers=None) -> dict:
    """Every DiT parameter the fast path reads, by checkpoint key, with its shape."""
    C = spec.dim
    p = spec.patch_size
    shapes = {
        "patch_embedding.weight": (C, spec.in_dim) + tuple(p), "patch_embedding.bias": (C,),
        "text_embedding.0.weight": (C, spec.text_dim), "text_embedding.0.bias": (C,),
        "text_embedding.2.weight": (C, C), "text_embedding.2.bias": (C,),
        "time_embedding.0.weight": (C, spec.freq_dim), "time_embedding.0.bias": (C,),
        "time_embedding.2.weight": (C, C), "time_embedding.2.bias": (C,),
        "time_projection.1.weight": (6 * C, C), "time_projection.1.bias": (6 * C,),
        "head.modulation": (1, 2, C), "head.head.weight": (p[0] * p[1] * p[2] * spec.out_dim, C),
        "head.head.bias": (p[0] * p[1] * p[2] * spec.out_dim,),
    }
    for i in range(spec.num_layers if num_layers is None else num_layers):
        for k, sh in sorted(_block_shapes(spec).items()):
            shapes[f"blocks.{i}.{k}"] = sh
    return shapes


def random_model_state(spec: WanSpec, seed: int, device="cpu", num_layers=None) -> dict:
    """Whole-model seeded state dict (bf16) with the checkpoint's key names."""
    gen = torch.Generator(device=device).manual_seed(seed)
    return {k: _fill(k, s, gen, device, spec.dim) for k, s in model_shapes(spec, num_layers).items()}


def block_state(sd: dict, i: int) -> dict:
    pre = f"blocks.{i}."
    return {k[len(pre):]: v for k, v in sd.items() if k.startswith(pre)}


class BlockWeights:
    """One block's parameters on `device` in bf16, sliced for TP rank `tp_rank` of `tp_size`."""

    def __init__(self, sd: dict, num_heads: int, device, tp_rank: int = 0, tp_size: int = 1,
                 local_cross: bool = False):
        """local_cross: keep the cross-attention weights whole (all heads) on every rank, for the
        sequence-parallel block whose cross-attention runs on the rank's token shard without
        collectives (the reference's `full_cross`, models/fast_dit.py:372-377)."""
        C = sd["self_attn.q.weight"].shape[1]
        assert num_heads % tp_size == 0, f"{num_heads} heads do not split over {tp_size} ranks"
        d = C // num_heads
        assert d == 128, "the attention kernels are built for head_dim 128"
        nl = num_heads // tp_size
        Cl = nl * d
        F = sd["ffn.0.weight"].shape[0]
        assert F % tp_size == 0
        Fl = F // tp_size
        hs = slice(tp_rank * Cl, (tp_rank + 1) * Cl)
        fs = slice(tp_rank * Fl, (tp_rank + 1) * Fl)

        def g(k, sl=None, col=False):
            t = sd[k]
            if sl is not None:
                t = t[:, sl] if col else t[sl]
            return t.to(device=device, dtype=BF16).contiguous()

        self.dim, self.num_heads, self.local_heads, self.local_dim = C, num_heads, nl, Cl
        self.ffn_local = Fl
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.modulation = g("modulation").reshape(6, C).contiguous()
        sa, ca = "self_attn", "cross_attn"
        self.w_qkv = torch.cat([g(f"{sa}.{p}.weight", hs) for p in "qkv"]).contiguous()
        self.b_qkv = torch.cat([g(f"{sa}.{p}.bias", hs) for p in "qkv"]).contiguous()
        self.g_q, self.g_k = g(f"{sa}.norm_q.weight", hs), g(f"{sa}.norm_k.weight", hs)
        self.w_o, self.b_o = g(f"{sa}.o.weight", hs, col=True), g(f"{sa}.o.bias")
        self.ln3_w, self.ln3_b = g("norm3.weight"), g("norm3.bias")
        self.local_cross = local_cross
        cs = None if local_cross else hs
        self.cross_heads = num_heads if local_cross else nl
        self.cross_dim = C if local_cross else Cl
        self.w_cq, self.b_cq, self.g_cq = g(f"{ca}.q.weight", cs), g(f"{ca}.q.bias", cs), g(f"{ca}.norm_q.weight", cs)
        self.w_ckv = torch.cat([g(f"{ca}.k.weight", cs), g(f"{ca}.v.weight", cs)]).contiguous()
        self.b_ckv = torch.cat([g(f"{ca}.k.bias", cs), g(f"{ca}.v.bias", cs)]).contiguous()
        self.g_ck = g(f"{ca}.norm_k.weight", cs)
        self.w_co, self.b_co = g(f"{ca}.o.weight", cs, col=True), g(f"{ca}.o.bias")
        self.w1, self.b1 = g("ffn.0.weight", fs), g("ffn.0.bias", fs)
        self.w2, self.b2 = g("ffn.2.weight", fs, col=True), g("ffn.2.bias")
