"""Kernel parity on a B200: each libwanb200 entry point against a plain PyTorch fp32 reference
of the same op, at ragged sizes.  Tolerances are relative RMS errors (bf16 output rounding is
~2^-9 relative, i.e. about 2e-3 RMS)."""
import math

import pytest
import torch

from wanb200 import _lib as L
from wanb200 import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.fixture(autouse=True)
def _no_device_error():
    L.device_error(reset=True)
    yield
    assert L.device_error(reset=True) == 0, "a kernel reported a device-side timeout"


def randn(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(torch.bfloat16)


# ---------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 192), (1000, 384, 3072), (77, 1152, 384),
                                   (2160, 3072, 3072)])
def test_gemm_bias(M, N, K):
    a, w, b = randn(M, K, seed=1), randn(N, K, scale=0.05, seed=2), randn(N, scale=0.1, seed=3)
    out = ops.linear(a, w, b, epilogue=L.EPI_BIAS)
    ref = a.float() @ w.float().t() + b.float()
    assert rel(out, ref) < 4e-3


def test_gemm_none_and_strided_views():
    M, N, K = 513, 768, 256
    big = randn(M, 2 * K, seed=4)
    a = big[:, K:]  # row stride 2K
    w = randn(N, K, scale=0.05, seed=5)
    out = torch.zeros(M, N + 64, dtype=torch.bfloat16, device=DEV)
    ops.linear(a, w, None, epilogue=L.EPI_NONE, out=out[:, :N])
    ref = a.float() @ w.float().t()
    assert rel(out[:, :N], ref) < 4e-3
    assert torch.count_nonzero(out[:, N:]) == 0


def test_gemm_gelu():
    M, N, K = 700, 1792, 3072
    a, w, b = randn(M, K, seed=6), randn(N, K, scale=0.02, seed=7), randn(N, scale=0.1, seed=8)
    out = ops.linear(a, w, b, epilogue=L.EPI_BIAS_GELU)
    ref = torch.nn.functional.gelu(a.float() @ w.float().t() + b.float(), approximate="tanh")
    assert rel(out, ref) < 4e-3


@pytest.mark.parametrize("inplace", [False, True])
def test_gemm_gate_residual(inplace):
    Lx, nf, B = 360, 6, 2
    M, N, K = B * Lx, 512, 384
    a, w, b = randn(M, K, seed=9), randn(N, K, scale=0.05, seed=10), randn(N, scale=0.1, seed=11)
    res = randn(M, N, seed=12)
    mod = randn(6, N, scale=0.1, seed=13)
    e0 = torch.randn(nf, 6, N, device=DEV) * 0.1
    gate = (mod[2], e0[:, 2, :])
    res0 = res.clone()
    out = res if inplace else None
    out = ops.linear(a, w, b, epilogue=L.EPI_BIAS_GATE_RES, residual=res, gate=gate, frames=(Lx, Lx // nf), out=out)
    g = (mod[2].float() + e0[:, 2, :]).repeat_interleave(Lx // nf, 0).repeat(B, 1)
    ref = res0.float() + (a.float() @ w.float().t() + b.float()) * g
    assert rel(out, ref) < 4e-3


@pytest.mark.parametrize("tile_n", [64, 96, 128, 160, 192, 224, 256, 0])
def test_gemm_tile_widths(tile_n):
    """Every tile width along N (ragged last column tile included) gives the same product, and
    every 32-column chunk's sum of squares lands in its own slot."""
    M, K, Cl = 300, 192, 224
    N = 3 * Cl  # 672: not a multiple of most tile widths
    a, w, b = randn(M, K, seed=51), randn(N, K, scale=0.05, seed=52), randn(N, scale=0.1, seed=53)
    ss = torch.full((M, 2 * Cl // 32), float("nan"), device=DEV)  # every entry must be written
    out = ops.linear(a, w, b, epilogue=L.EPI_BIAS_SUMSQ, rowss=ss, ss_cols=2 * Cl, tile_n=tile_n)
    ref = a.float() @ w.float().t() + b.float()
    assert rel(out, ref) < 4e-3
    ref_parts = ref[:, :2 * Cl].reshape(M, 2 * Cl // 32, 32).pow(2).sum(2)
    assert rel(ss, ref_parts) < 1e-3


def test_gemm_gate_residual_on_a_sequence_shard():
    """rows_per_seq / row_offset: a [2, S] buffer holding tokens 40 .. 40+S-1 of each sequence."""
    Lx, nf, S, off = 180, 6, 70, 40
    M, N, K = 2 * S, 256, 128
    a, w, b = randn(M, K, seed=54), randn(N, K, scale=0.05, seed=55), randn(N, scale=0.1, seed=56)
    res = randn(M, N, seed=57)
    mod = randn(6, N, scale=0.1, seed=58)
    e0 = torch.randn(nf, 6, N, device=DEV) * 0.1
    out = ops.linear(a, w, b, epilogue=L.EPI_BIAS_GATE_RES, residual=res, gate=(mod[2], e0[:, 2, :]),
                     frames=(Lx, Lx // nf, off, S), tile_n=128)
    frame = ((torch.arange(M, device=DEV) % S) + off) // (Lx // nf)
    g = mod[2].float() + e0[frame, 2, :]
    ref = res.float() + (a.float() @ w.float().t() + b.float()) * g
    assert rel(out, ref) < 4e-3


def test_gemm_residual():
    M, N, K = 333, 256, 128
    a, w, b, res = randn(M, K, seed=14), randn(N, K, scale=0.05, seed=15), randn(N, seed=16), randn(M, N, seed=17)
    out = ops.linear(a, w, b, epilogue=L.EPI_BIAS_RES, residual=res)
    assert rel(out, res.float() + a.float() @ w.float().t() + b.float()) < 4e-3


@pytest.mark.parametrize("Cl", [384, 3072])
def test_gemm_sumsq_sections(Cl):
    M, K = 517, 256
    N = 3 * Cl
    a, w, b = randn(M, K, seed=18), randn(N, K, scale=0.05, seed=19), randn(N, scale=0.1, seed=20)
    P = Cl // 32
    ss = torch.full((M, 2 * P), float("nan"), device=DEV)
    out = ops.linear(a, w, b, epilogue=L.EPI_BIAS_SUMSQ, rowss=ss, ss_cols=2 * Cl)
    ref = a.float() @ w.float().t() + b.float()
    assert rel(out, ref) < 4e-3
    ref_ss = torch.stack([ref[:, :Cl].pow(2).sum(1), ref[:, Cl:2 * Cl].pow(2).sum(1)])
    # the per-section sums the TP path all-reduces (sumsq_reduce adds a row's partials in order)
    red = torch.empty(2, M, device=DEV)
    ops.sumsq_reduce(ss, [0, P], P, red)
    assert rel(red, ref_ss) < 1e-3
    assert rel(red, ss.view(M, 2, P).sum(2).t()) < 1e-6
    # bit-reproducible: the same launch again gives the same partials and sums (no atomics)
    ss2 = torch.empty_like(ss)
    out2 = ops.linear(a, w, b, epilogue=L.EPI_BIAS_SUMSQ, rowss=ss2, ss_cols=2 * Cl)
    red2 = torch.empty(2, M, device=DEV)
    ops.sumsq_reduce(ss2, [0, P], P, red2)
    assert torch.equal(ss, ss2) and torch.equal(red, red2) and torch.equal(out, out2)


# ---------------------------------------------------------------------------- attention
def sdpa_ref(q, k, v, scale=None):
    return torch.nn.functional.scaled_dot_product_attention(
        q.float().transpose(1, 2), k.float().transpose(1, 2), v.float().transpose(1, 2), scale=scale).transpose(1, 2)


@pytest.mark.parametrize("B,H,Lq,Lk", [(1, 1, 128, 128), (2, 3, 200, 77), (2, 3, 1, 1), (1, 2, 127, 129),
                                       (2, 2, 1080, 1080), (2, 3, 1000, 512), (1, 1, 300, 4100)])
def test_attention_vs_sdpa(B, H, Lq, Lk):
    q, k, v = randn(B, Lq, H, 128, seed=21), randn(B, Lk, H, 128, seed=22), randn(B, Lk, H, 128, seed=23)
    o = ops.attention(q, k, v)
    assert rel(o, sdpa_ref(q, k, v)) < 1e-2


@pytest.mark.parametrize("B,H,Lq,Lk,splits", [(1, 6, 1000, 7854, 3), (2, 3, 300, 1080, 2), (1, 2, 200, 77, 1),
                                              (1, 4, 257, 513, 3), (2, 2, 128, 1100, 3)])
def test_attention_split_kv(B, H, Lq, Lk, splits):
    """Split-KV: each CTA covers a contiguous range of key tiles, writes unnormalised partials,
    and the merge kernel combines them (ragged last split included)."""
    q, k, v = randn(B, Lq, H, 128, seed=41), randn(B, Lk, H, 128, seed=42), randn(B, Lk, H, 128, seed=43)
    o = ops.attention(q, k, v, kv_splits=splits)
    ref = sdpa_ref(q, k, v)
    assert rel(o, ref) < 1e-2
    o1 = ops.attention(q, k, v, kv_splits=1)
    assert rel(o, o1.float()) < 1e-2


def test_attention_split_choice():
    """The library's split count: none for short key ranges (cross-attention over 512 keys) or
    grids that already fill the SMs in many waves; a split for few-wave grids over long keys."""
    lib = L.load()
    assert lib.wanb200_attn_kv_splits(1, 24, 7854, 512) == 1     # cross-attention, batch 1
    assert lib.wanb200_attn_kv_splits(2, 24, 7854, 7854) == 1    # config-2 self-attention
    assert lib.wanb200_attn_kv_splits(1, 24, 1964, 7854) > 1     # Q-local shard of 4
    assert lib.wanb200_attn_kv_splits(1, 6, 7854, 7854) > 1      # TP 4, batch 1


@pytest.mark.parametrize("cut,s1,s2", [(600, 1, 2), (1, 1, 1), (1499, 2, 1)])
def test_attention_key_set_in_pieces(cut, s1, s2):
    """Partial slots: the keys [0, cut) and [cut, Lk) in two launches that share a workspace,
    the second merging all slots, equal one attention over all keys."""
    B, H, Lq, Lk = 2, 3, 700, 1500
    q, k, v = randn(B, Lq, H, 128, seed=61), randn(B, Lk, H, 128, seed=62), randn(B, Lk, H, 128, seed=63)
    o = torch.empty_like(q)
    n = s1 + s2
    ops.attention(q, k[:, :cut], v[:, :cut], out=o, kv_splits=s1, parts=(0, n, True))
    ops.attention(q, k[:, cut:], v[:, cut:], out=o, kv_splits=s2, parts=(s1, n, False))
    assert rel(o, sdpa_ref(q, k, v)) < 1e-2


@pytest.mark.parametrize("B,H,Lq,Lk,splits", [(1, 2, 128, 128, 1), (2, 3, 300, 1080, None), (1, 2, 127, 129, 1),
                                              (2, 2, 1000, 512, 1), (1, 6, 1000, 2100, 3), (1, 1, 129, 4100, 2)])
def test_attention_fp8_vs_sdpa_and_bf16(B, H, Lq, Lk, splits):
    """The e4m3 variant (q, k per 128-token-block scales, v per head, P in e4m3) against fp32
    SDPA: within the e4m3 rounding (3 mantissa bits), far above the bf16 path's error but
    averaged over the keys; ragged q / k tails and split-KV included."""
    q, k, v = randn(B, Lq, H, 128, seed=71), randn(B, Lk, H, 128, seed=72), randn(B, Lk, H, 128, seed=73)
    ref = sdpa_ref(q, k, v)
    o8 = ops.attention(q, k, v, kv_splits=splits, fp8=True)
    o16 = ops.attention(q, k, v, kv_splits=splits)
    e8, e16 = rel(o8, ref), rel(o16, ref)
    print(f"fp8 rel-RMS {e8:.4f} (bf16 {e16:.4f})")
    assert e8 < 6e-2
    assert e16 < 1e-2


def test_attention_fp8_scaled_inputs():
    """Per-block scales: q blocks of magnitude 1..64 and k blocks of 1..1/8 (softmax kept as flat
    as in the other cases) give the same accuracy as unscaled inputs; and scaling q by 64 and k
    by 1/32 with the softmax scale compensated gives the same e4m3 codes, so the same result."""
    B, H, L = 1, 2, 512
    q, k, v = randn(B, L, H, 128, seed=74), randn(B, L, H, 128, seed=75), randn(B, L, H, 128, seed=76)
    mag = torch.tensor([1.0, 4.0, 16.0, 64.0], device=DEV).repeat_interleave(128)[None, :, None, None]
    qs = (q.float() * mag).to(torch.bfloat16)
    ks = (k.float() / mag.flip(1).sqrt()).to(torch.bfloat16)
    sc = 1.0 / (64.0 * math.sqrt(128.0))
    err = rel(ops.attention(qs, ks, v, softmax_scale=sc, fp8=True), sdpa_ref(qs, ks, v, scale=sc))
    print(f"fp8 rel-RMS with block magnitudes 1..64: {err:.4f}")
    assert err < 6e-2
    o = ops.attention(q, k, v, softmax_scale=0.1, fp8=True)
    o2 = ops.attention((q.float() * 64).to(torch.bfloat16), (k.float() / 32).to(torch.bfloat16), v,
                       softmax_scale=0.1 / 2, fp8=True)
    assert rel(o2, o.float()) < 1e-3


def test_attention_split_kv_rejects_empty_split():
    q = randn(1, 128, 1, 128, seed=44)
    k = randn(1, 300, 1, 128, seed=45)  # 3 key tiles
    with pytest.raises(L.WanB200Error, match="kv_splits"):
        ops.attention(q, k, k, kv_splits=4)


def test_attention_fused_qkv_layout_and_scaled_scores():
    """q, k, v as column slices of one [B*L, 3*H*128] buffer (the QKV GEMM output); RMS-normed
    inputs with a gain of 3 so the scores are large (softmax far from uniform)."""
    B, Lx, H = 2, 1080, 3
    qkv = randn(B * Lx, 3 * H * 128, seed=24).float()
    qkv[:, :2 * H * 128] *= 3.0
    qkv = qkv.to(torch.bfloat16)
    q = qkv[:, :H * 128].view(B, Lx, H, 128)
    k = qkv[:, H * 128:2 * H * 128].view(B, Lx, H, 128)
    v = qkv[:, 2 * H * 128:].view(B, Lx, H, 128)
    o = ops.attention(q, k, v)
    assert rel(o, sdpa_ref(q, k, v)) < 1e-2


def test_attention_op_registered():
    q = randn(1, 256, 2, 128, seed=25)
    o = torch.ops.wanb200.attn(q, q, q, 1.0 / math.sqrt(128))
    assert rel(o, sdpa_ref(q, q, q)) < 1e-2


# ---------------------------------------------------------------------------- norms
def test_layernorm_modulate_and_affine():
    B, Lx, nf, C = 2, 1080, 6, 3072
    x = randn(B * Lx, C, seed=26)
    mod = randn(6, C, scale=0.1, seed=27)
    e0 = torch.randn(nf, 6, C, device=DEV) * 0.1
    h = ops.layernorm_modulate(x, mod, e0, 0, 1, (Lx, Lx // nf))
    ln = torch.nn.functional.layer_norm(x.float(), (C,), eps=1e-6)
    sh = (mod[0].float() + e0[:, 0]).repeat_interleave(Lx // nf, 0).repeat(B, 1)
    sc = (mod[1].float() + e0[:, 1]).repeat_interleave(Lx // nf, 0).repeat(B, 1)
    assert rel(h, ln * (1 + sc) + sh) < 4e-3
    wgt, bia = randn(C, seed=28), randn(C, seed=29)
    h2 = ops.layernorm_affine(x, wgt, bia)
    ref2 = torch.nn.functional.layer_norm(x.float(), (C,), wgt.float(), bia.float(), eps=1e-6)
    assert rel(h2, ref2) < 4e-3


def test_layernorm_small_dim():
    x = randn(37, 256, seed=30)
    wgt, bia = randn(256, seed=31), randn(256, seed=32)
    h = ops.layernorm_affine(x, wgt, bia)
    assert rel(h, torch.nn.functional.layer_norm(x.float(), (256,), wgt.float(), bia.float(), eps=1e-6)) < 4e-3


@pytest.mark.parametrize("form", ["sums", "partials", "self"])
def test_qk_norm_rope_vs_oracle(form):
    """The sums of squares as finished per-row sums (the TP path), as a GEMM's 32-column chunk
    partials, or formed by the kernel from the section's own bf16 values (one GPU)."""
    from oracle import dit_ref as R
    grid = (3, 5, 7)
    Lx = 105
    B, H = 2, 3
    Cl = H * 128
    M = B * Lx
    qkv = randn(M, 3 * Cl, seed=33)
    ref_in = qkv.float().clone()
    ss = torch.stack([ref_in[:, :Cl].pow(2).sum(1), ref_in[:, Cl:2 * Cl].pow(2).sum(1)]) * 8.0  # "global" dim 8x
    gd = 8 * Cl
    if form == "sums":
        ssq, ssk = ss[0], ss[1]
    elif form == "self":  # the section is the whole global dim
        ssq = ssk = None
        ss, gd = ss / 8.0, Cl
    else:
        parts = ref_in[:, :2 * Cl].reshape(M, 2 * Cl // 32, 32).pow(2).sum(2) * 8.0  # [M, 2P]
        ssq, ssk = parts[:, :Cl // 32], parts[:, Cl // 32:]
    gq, gk = randn(Cl, scale=0.1, seed=34).float().add(1).to(torch.bfloat16), randn(Cl, seed=35)
    cos, sin = R.rope_tables(R.model_freqs(128), grid, 128)
    ops.qk_norm_rope(qkv, [(0, ssq, gq), (Cl, ssk, gk)], Cl, gd, cos=cos.reshape(Lx, 64).to(DEV),
                     sin=sin.reshape(Lx, 64).to(DEV), seq_len=Lx)
    for sec, g in ((0, gq), (1, gk)):
        x = ref_in[:, sec * Cl:(sec + 1) * Cl]
        y = x * torch.rsqrt(ss[sec][:, None] / gd + 1e-6) * g.float()
        y = R.rope(y.view(B, Lx, H, 128).cpu(), cos, sin).reshape(B * Lx, Cl)
        assert rel(qkv[:, sec * Cl:(sec + 1) * Cl].cpu(), y) < 4e-3
    assert torch.equal(qkv[:, 2 * Cl:], ref_in[:, 2 * Cl:].to(torch.bfloat16))


def test_bias_gate_residual():
    B, Lx, nf, C = 2, 120, 4, 768
    res, y, b = randn(B * Lx, C, seed=36), randn(B * Lx, C, seed=37), randn(C, seed=38)
    mod = randn(6, C, scale=0.1, seed=39)
    e0 = torch.randn(nf, 6, C, device=DEV) * 0.1
    out = ops.bias_gate_residual(res, y, b, gate=(mod[5], e0[:, 5, :]), frames=(Lx, Lx // nf))
    g = (mod[5].float() + e0[:, 5]).repeat_interleave(Lx // nf, 0).repeat(B, 1)
    assert rel(out, res.float() + (y.float() + b.float()) * g) < 4e-3
    out2 = ops.bias_gate_residual(res, y, b)
    assert rel(out2, res.float() + y.float() + b.float()) < 4e-3


# ---------------------------------------------------------------------------- fp32 residual stream
F32 = torch.float32


@pytest.mark.parametrize("res_dt,out_dt,inplace", [(F32, F32, False), (F32, F32, True), (torch.bfloat16, F32, False),
                                                   (F32, torch.bfloat16, False)])
def test_gemm_gate_residual_fp32_stream(res_dt, out_dt, inplace):
    """GATE_RES with an fp32 residual and / or an fp32 output: the sum is formed in fp32 and stored
    without rounding (fp32 out: error of the bf16 GEMM operands only, far below bf16 output rounding)."""
    Lx, nf, B = 360, 6, 2
    M, N, K = B * Lx, 512, 384
    a, w, b = randn(M, K, seed=61), randn(N, K, scale=0.05, seed=62), randn(N, scale=0.1, seed=63)
    res = (torch.randn(M, N, generator=torch.Generator(device=DEV).manual_seed(64), device=DEV) * 3).to(res_dt)
    mod = randn(6, N, scale=0.1, seed=65)
    e0 = torch.randn(nf, 6, N, device=DEV) * 0.1
    res0 = res.clone()
    out = res if inplace else torch.empty(M, N, device=DEV, dtype=out_dt)
    ops.linear(a, w, b, epilogue=L.EPI_BIAS_GATE_RES, residual=res, gate=(mod[2], e0[:, 2, :]),
               frames=(Lx, Lx // nf), out=out)
    g = (mod[2].float() + e0[:, 2, :]).repeat_interleave(Lx // nf, 0).repeat(B, 1)
    y = (a.float() @ w.float().t() + b.float()) * g
    ref = res0.float() + y
    assert out.dtype == out_dt
    if out_dt == F32:  # the residual part is exact: only the GEMM's fp32 accumulation differs
        assert rel(out - res0.float(), y) < 1e-5
    assert rel(out, ref) < (1e-6 if out_dt == F32 else 4e-3)


def test_gemm_residual_fp32_stream():
    M, N, K = 333, 256, 128
    a, w, b = randn(M, K, seed=66), randn(N, K, scale=0.05, seed=67), randn(N, seed=68)
    res = torch.randn(M, N, device=DEV) * 5
    res0 = res.clone()
    out = ops.linear(a, w, b, epilogue=L.EPI_BIAS_RES, residual=res, out=res)  # in place, fp32
    assert out is res and out.dtype == F32
    assert rel(out, res0 + a.float() @ w.float().t() + b.float()) < 1e-6


@pytest.mark.parametrize("epi", [L.EPI_BIAS_GATE_RES, L.EPI_BIAS_RES])
def test_gemm_fp32_stream_row_segment_epilogue(epi):
    """The fp32 residual update in place at tile width 256 (the accumulator chunk staged in shared
    memory, row-segment residual loads and stores) and 224 / 192 / 128 (one row per lane): the same
    values as each other and as the fp32 reference, with a ragged last row block, a partial last
    column tile and a sequence-shard frame map."""
    Lx, nf, S, off = 540, 6, 300, 120
    M, N, K = 2 * S, 672, 256
    a, w, b = randn(M, K, seed=71), randn(N, K, scale=0.05, seed=72), randn(N, scale=0.1, seed=73)
    res0 = torch.randn(M, N, generator=torch.Generator(device=DEV).manual_seed(74), device=DEV) * 3
    mod = randn(6, N, scale=0.1, seed=75)
    e0 = torch.randn(nf, 6, N, device=DEV) * 0.1
    kw = dict(gate=(mod[2], e0[:, 2, :]), frames=(Lx, Lx // nf, off, S)) if epi == L.EPI_BIAS_GATE_RES else {}
    y = a.float() @ w.float().t() + b.float()
    if epi == L.EPI_BIAS_GATE_RES:
        frame = ((torch.arange(M, device=DEV) % S) + off) // (Lx // nf)
        y = y * (mod[2].float() + e0[frame, 2, :])
    outs = {}
    for tn in (256, 224, 192, 128):
        res = res0.clone()
        out = ops.linear(a, w, b, epilogue=epi, residual=res, out=res, tile_n=tn, **kw)
        assert out is res
        assert rel(res - res0, y) < 1e-5, tn
        outs[tn] = res
    for tn in (224, 192, 128):
        assert rel(outs[tn], outs[256]) < 1e-6, tn


def test_layernorm_reads_the_fp32_stream():
    B, Lx, nf, C = 2, 540, 6, 3072
    x = torch.randn(B * Lx, C, device=DEV) * 4 + 1
    mod = randn(6, C, scale=0.1, seed=69)
    e0 = torch.randn(nf, 6, C, device=DEV) * 0.1
    h = ops.layernorm_modulate(x, mod, e0, 3, 4, (Lx, Lx // nf))
    ln = torch.nn.functional.layer_norm(x, (C,), eps=1e-6)
    sh = (mod[3].float() + e0[:, 3]).repeat_interleave(Lx // nf, 0).repeat(B, 1)
    sc = (mod[4].float() + e0[:, 4]).repeat_interleave(Lx // nf, 0).repeat(B, 1)
    assert h.dtype == torch.bfloat16 and rel(h, ln * (1 + sc) + sh) < 4e-3
    wgt, bia = randn(C, seed=70), randn(C, seed=71)
    h2 = ops.layernorm_affine(x, wgt, bia)
    assert rel(h2, torch.nn.functional.layer_norm(x, (C,), wgt.float(), bia.float(), eps=1e-6)) < 4e-3
    x3 = torch.randn(37, 768, device=DEV)  # one warp per row (dim % 512 != 0)
    h3 = ops.layernorm_affine(x3, wgt[:768], bia[:768])
    assert rel(h3, torch.nn.functional.layer_norm(x3, (768,), wgt[:768].float(), bia[:768].float(), eps=1e-6)) < 4e-3


def test_bias_gate_residual_fp32_stream():
    B, Lx, nf, C = 2, 120, 4, 768
    res, y, b = torch.randn(B * Lx, C, device=DEV) * 3, randn(B * Lx, C, seed=72), randn(C, seed=73)
    mod = randn(6, C, scale=0.1, seed=74)
    e0 = torch.randn(nf, 6, C, device=DEV) * 0.1
    g = (mod[5].float() + e0[:, 5]).repeat_interleave(Lx // nf, 0).repeat(B, 1)
    ref = res + (y.float() + b.float()) * g
    out = ops.bias_gate_residual(res, y, b, gate=(mod[5], e0[:, 5, :]), frames=(Lx, Lx // nf))
    assert out.dtype == F32 and rel(out, ref) < 1e-6
    out16 = torch.empty(B * Lx, C, device=DEV, dtype=torch.bfloat16)
    ops.bias_gate_residual(res, y, b, gate=(mod[5], e0[:, 5, :]), frames=(Lx, Lx // nf), out=out16)
    assert rel(out16, ref) < 4e-3
