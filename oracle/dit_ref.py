"""CPU fp32 oracle for the Wan2.2-TI2V-5B DiT denoise path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this module; only
`tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` use it, and only as the checker (or as the timed CPU baseline), never as a
code path of the B200 implementation.

It restates, in float32 PyTorch on the CPU, the reference's own "upstream math, no bf16"
oracle (yahavb/wan2-ti2v-5b `scripts/validate/ref_fp32.py`), plus the pieces that script
borrows from `models/fast_dit.py` and `wan/modules/model.py`.  Every function names the
reference lines it follows.  Parameters are plain dicts of fp32 tensors keyed exactly like
the HF checkpoint (`self_attn.q.weight`, `ffn.0.bias`, ... per block;
`blocks.{i}.…`, `time_embedding.0.weight`, ... per model), so the same dict layout feeds
the device implementation.

Pinned: `tests/golden/make_golden.py` imports the reference itself (with import shims) and
stores its outputs on small seeded cases; `tests/test_oracle.py` checks this module against
those fixtures.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

EPS = 1e-6  # WanLayerNorm / WanRMSNorm eps for TI2V-5B (wan/configs/wan_ti2v_5B.py:27)


# ---------------------------------------------------------------------------- RoPE
def rope_params(max_seq_len: int, dim: int, theta: float = 10000.0) -> torch.Tensor:
    """Angle table [max_seq_len, dim//2], fp32 (wan/modules/rope_neuron.py:14-24)."""
    inv = 1.0 / torch.pow(theta, torch.arange(0, dim, 2).float().div(dim))
    return torch.outer(torch.arange(max_seq_len).float(), inv)


def model_freqs(head_dim: int, max_seq_len: int = 1024) -> torch.Tensor:
    """WanModel.freqs: frame / height / width angle tables side by side (model.py:395-403)."""
    d = head_dim
    return torch.cat([rope_params(max_seq_len, d - 4 * (d // 6)),
                      rope_params(max_seq_len, 2 * (d // 6)),
                      rope_params(max_seq_len, 2 * (d // 6))], dim=1)


def rope_tables(freqs: torch.Tensor, grid, head_dim: int):
    """cos/sin [1, L, 1, d/2] for a (F, H, W) token grid (fast_dit.py:548-558).

    Pair c of token (f, h, w) gets angle freqs[f|h|w, c] with the pairs split
    (c - 2*(c//3), c//3, c//3) between frame, height and width (22/21/21 for d=128).
    """
    f, h, w = grid
    c = head_dim // 2
    fr = freqs.float().split([c - 2 * (c // 3), c // 3, c // 3], dim=1)
    ang = torch.cat([
        fr[0][:f].view(f, 1, 1, -1).expand(f, h, w, -1),
        fr[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
        fr[2][:w].view(1, 1, w, -1).expand(f, h, w, -1),
    ], dim=-1).reshape(1, f * h * w, 1, c)
    return torch.cos(ang), torch.sin(ang)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation (x0, x1) -> (x0 c - x1 s, x0 s + x1 c) (fast_dit.py:163-169)."""
    B, L, n, d = x.shape
    xp = x.float().reshape(B, L, n, d // 2, 2)
    xr, xi = xp[..., 0], xp[..., 1]
    return torch.stack([xr * cos - xi * sin, xr * sin + xi * cos], dim=-1).reshape(B, L, n, d)


# ---------------------------------------------------------------------------- primitives
def rms(x, weight, eps=EPS):
    """RMSNorm over the last dim, fp32 (ref_fp32.py:20-21)."""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight


def lin(x, weight, bias=None):
    """nn.Linear (ref_fp32.py:24-25)."""
    return F.linear(x, weight, bias)


def attn(q, k, v):
    """Exact softmax(q k^T / sqrt(d)) v on [B, L, n, d] (ref_fp32.py:28-29)."""
    return F.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)


def per_frame(t, nf):
    """[B, L, C] -> [B, F, L/F, C] so a per-frame [1, F, C] row broadcasts (ref_fp32.py:32-34)."""
    B, L, C = t.shape
    return t.view(B, nf, L // nf, C)


# ---------------------------------------------------------------------------- one block
def block_fwd(p: dict, x, e0, cos, sin, ck, cv, nf: int, num_heads: int):
    """One WanAttentionBlock forward in fp32 (ref_fp32.py:37-59).

    p: block params keyed like the checkpoint (`modulation`, `self_attn.q.weight`, ...,
    `norm3.weight`, `ffn.0.weight`, ...).  x [B, L, C]; e0 [1, F, 6, C] per-frame time
    projection; cos/sin [1, L, 1, d/2]; ck/cv [B, Lc, n, d] cross K/V (see cross_kv).
    """
    B, L, C = x.shape
    n = num_heads
    d = C // n
    e = [t.squeeze(2) for t in (p["modulation"].unsqueeze(0) + e0).chunk(6, dim=2)]

    def mod(h, shift, scale):
        return (per_frame(h, nf) * (1 + scale.unsqueeze(2)) + shift.unsqueeze(2)).view(B, L, C)

    def gate(y, g):
        return (per_frame(y, nf) * g.unsqueeze(2)).view(B, L, C)

    def P(name):
        return p[name + ".weight"], p.get(name + ".bias")

    h = mod(F.layer_norm(x, (C,), eps=EPS), e[0], e[1])
    q = rope(rms(lin(h, *P("self_attn.q")), p["self_attn.norm_q.weight"]).view(B, L, n, d), cos, sin)
    k = rope(rms(lin(h, *P("self_attn.k")), p["self_attn.norm_k.weight"]).view(B, L, n, d), cos, sin)
    v = lin(h, *P("self_attn.v")).view(B, L, n, d)
    x = x + gate(lin(attn(q, k, v).reshape(B, L, C), *P("self_attn.o")), e[2])
    h = F.layer_norm(x, (C,), p["norm3.weight"], p["norm3.bias"], eps=EPS)
    q = rms(lin(h, *P("cross_attn.q")), p["cross_attn.norm_q.weight"]).view(B, L, n, d)
    x = x + lin(attn(q, ck, cv).reshape(B, L, C), *P("cross_attn.o"))
    h = mod(F.layer_norm(x, (C,), eps=EPS), e[3], e[4])
    y = lin(F.gelu(lin(h, *P("ffn.0")), approximate="tanh"), *P("ffn.2"))
    return x + gate(y, e[5])


def cross_kv(p: dict, context, num_heads: int):
    """Per-block cross-attention K (RMS-normed) and V from the text context (ref_fp32.py:85-86)."""
    B, Lc, C = context.shape
    d = C // num_heads
    k = rms(lin(context, p["cross_attn.k.weight"], p["cross_attn.k.bias"]), p["cross_attn.norm_k.weight"])
    v = lin(context, p["cross_attn.v.weight"], p["cross_attn.v.bias"])
    return k.view(B, Lc, num_heads, d), v.view(B, Lc, num_heads, d)


# ---------------------------------------------------------------------------- whole step
def sinusoidal_embedding_1d(dim: int, position: torch.Tensor) -> torch.Tensor:
    """[len(position), dim] float64 sinusoid (wan/modules/model.py:15-25)."""
    half = dim // 2
    position = position.type(torch.float64)
    sinusoid = torch.outer(position, torch.pow(10000, -torch.arange(half).to(position).div(half)))
    return torch.cat([torch.cos(sinusoid), torch.sin(sinusoid)], dim=1)


def time_embed(mp: dict, t: float, nf: int, freq_dim: int):
    """Per-frame time embedding, frame 0 (the image frame) at t=0 (ref_fp32.py:77-80).

    Returns e [1, F, C] and e0 [1, F, 6, C].
    """
    t_frames = torch.full((nf,), float(t), dtype=torch.float64)
    t_frames[0] = 0.0
    s = sinusoidal_embedding_1d(freq_dim, t_frames).float().unsqueeze(0)
    e = lin(F.silu(lin(s, mp["time_embedding.0.weight"], mp["time_embedding.0.bias"])),
            mp["time_embedding.2.weight"], mp["time_embedding.2.bias"])
    e0 = lin(F.silu(e), mp["time_projection.1.weight"], mp["time_projection.1.bias"])
    return e, e0.unflatten(2, (6, e.shape[-1]))


def text_embed(mp: dict, ctx):
    """text_embedding = Linear, GELU(tanh), Linear (model.py:378-380)."""
    h = F.gelu(lin(ctx, mp["text_embedding.0.weight"], mp["text_embedding.0.bias"]), approximate="tanh")
    return lin(h, mp["text_embedding.2.weight"], mp["text_embedding.2.bias"])


def patch_embed(mp: dict, latent, patch=(1, 2, 2)):
    """Conv3d patchify of a [C_in, F, H, W] latent -> tokens [1, L, C] (ref_fp32.py:82)."""
    x = F.conv3d(latent.unsqueeze(0), mp["patch_embedding.weight"], mp["patch_embedding.bias"], stride=patch)
    return x.flatten(2).transpose(1, 2)


def head(mp: dict, x, e, grid, patch=(1, 2, 2), out_dim=48):
    """Head: LN + 2-way modulation + Linear, then unpatchify to [B, c, F, H, W] (ref_fp32.py:90-98)."""
    nf = grid[0]
    m = [t.squeeze(2) for t in (mp["head.modulation"].unsqueeze(0) + e.unsqueeze(2)).chunk(2, dim=2)]
    B, L, C = x.shape
    y = lin((per_frame(F.layer_norm(x, (C,), eps=EPS), nf) * (1 + m[1].unsqueeze(2))
             + m[0].unsqueeze(2)).view(B, L, C), mp["head.head.weight"], mp["head.head.bias"])
    f, h, w = grid
    p, q, r = patch
    c = out_dim
    return y.view(B, f, h, w, p, q, r, c).permute(0, 7, 1, 4, 2, 5, 3, 6).reshape(B, c, f * p, h * q, w * r)


def block_params(mp: dict, i: int) -> dict:
    pre = f"blocks.{i}."
    return {k[len(pre):]: v for k, v in mp.items() if k.startswith(pre)}


def step(mp: dict, cfg: dict, latent, t, ctx, ctx_null, guide: float = 5.0, layers=None):
    """Step-0 CFG noise prediction through all blocks (ref_fp32.py:62-99).

    cfg: {"num_heads", "num_layers", "freq_dim", "patch", "out_dim"}.  latent [C_in, F, H, W];
    ctx / ctx_null [Lc, text_dim].  `layers` limits the block loop (for bounded CPU samples).
    mp may hold its tensors on any device and in any float dtype: the embedding / head params
    are copied to fp32 CPU tensors once and each block's params just before the block runs, so
    a full-size model needs one block's fp32 params on the host at a time.
    """
    C_in, nf, H, W = latent.shape
    p = tuple(cfg.get("patch", (1, 2, 2)))
    grid = (nf // p[0], H // p[1], W // p[2])
    n = cfg["num_heads"]

    def f32(d):
        return {k: v.detach().to("cpu", torch.float32) for k, v in d.items()}

    emb = f32({k: v for k, v in mp.items() if not k.startswith("blocks.")})
    dim = emb["patch_embedding.weight"].shape[0]
    d = dim // n
    cos, sin = rope_tables(model_freqs(d), grid, d)
    e, e0 = time_embed(emb, t, grid[0], cfg["freq_dim"])
    context = text_embed(emb, torch.stack([ctx, ctx_null], 0).float().cpu())
    x = patch_embed(emb, latent.float().cpu(), p).expand(2, -1, -1).contiguous()
    nl = cfg["num_layers"] if layers is None else layers
    for i in range(nl):
        bp = f32(block_params(mp, i))
        ck, cv = cross_kv(bp, context, n)
        x = block_fwd(bp, x, e0, cos, sin, ck, cv, grid[0], n)
        del bp
    y = head(emb, x, e, grid, p, cfg.get("out_dim", 48))
    return y[1] + guide * (y[0] - y[1])


def rel_rms(a, b) -> float:
    """||a - b||_2 / ||b||_2, the reference's error score (ref_fp32.py:108)."""
    a, b = a.double(), b.double()
    return float(((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt()).item())
