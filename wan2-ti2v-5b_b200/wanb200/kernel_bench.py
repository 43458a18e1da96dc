"""Single-kernel timing at the block's shapes (CUDA events, inputs larger than L2).

    python -m wanb200.kernel_bench gemm --M 15708 --N 14336 --K 3072 --epi gelu [--iters 20]
    python -m wanb200.kernel_bench attn --B 2 --H 24 --Lq 7854 --Lk 7854 [--iters 20]
    python -m wanb200.kernel_bench ln --M 15708 --C 3072 [--f32]
    python -m wanb200.kernel_bench qknorm --M 15708 --C 3072
    python -m wanb200.kernel_bench gemm --M 15708 --N 3072 --K 3072 --epi gate_res --f32

(run from wan2-ti2v-5b_b200/ or with it on sys.path).  Prints one JSON line with the mean
time per launch and the algorithmic TFLOP/s or GB/s.  Used for sweeps and as the small-case
command under ncu.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _lib as L
from . import ops

EPIS = {"none": L.EPI_NONE, "bias": L.EPI_BIAS, "gelu": L.EPI_BIAS_GELU, "gate_res": L.EPI_BIAS_GATE_RES,
        "res": L.EPI_BIAS_RES, "sumsq": L.EPI_BIAS_SUMSQ}


def _time(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(a):
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(a.M, a.K, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(a.N, a.K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    b = torch.zeros(a.N, device=dev, dtype=torch.bfloat16)
    out = torch.empty(a.M, a.N, device=dev, dtype=torch.bfloat16)
    epi = EPIS[a.epi]
    kw = {}
    if epi in (L.EPI_BIAS_GATE_RES, L.EPI_BIAS_RES):
        kw["residual"] = torch.zeros(a.M, a.N, device=dev, dtype=torch.float32 if a.f32 else torch.bfloat16)
        if a.f32:  # the fp32 residual stream, updated in place as in the block
            out = kw["residual"]
    if epi == L.EPI_BIAS_GATE_RES:
        kw["gate"] = (torch.zeros(a.N, device=dev, dtype=torch.bfloat16), torch.ones(21, 6 * a.N, device=dev)[:, :a.N])
        kw["frames"] = (a.M, max(1, a.M // 21))
    if epi == L.EPI_BIAS_SUMSQ:
        kw["rowss"] = torch.empty(a.M, 2 * (a.N // 3) // 32, device=dev)  # q and k chunk partials
        kw["ss_cols"] = 2 * (a.N // 3)
    ms = _time(lambda: ops.linear(x, w, b if epi else None, epilogue=epi, out=out, tile_n=a.tile_n, **kw), a.iters)
    return {"kernel": "gemm", "M": a.M, "N": a.N, "K": a.K, "epi": a.epi, "f32_residual": a.f32,
            "tile_n": a.tile_n, "ms": ms,
            "tflops": 2 * a.M * a.N * a.K / ms / 1e9}


def bench_attn(a):
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(a.B, a.Lq, a.H, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(a.B, a.Lk, a.H, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(a.B, a.Lk, a.H, 128, generator=g, device=dev).to(torch.bfloat16)
    o = torch.empty_like(q)
    if a.local:  # the Q-local SP pattern: the shard's own a.local keys, then the rest, merged
        n_rem = a.Lk - a.local
        s_loc = a.kv_splits or ops.kv_splits(a.B, a.H, a.Lq, a.local)
        s_rem = a.kv_splits_rem or ops.kv_splits(a.B, a.H, a.Lq, n_rem)
        n = s_loc + s_rem

        def fn():
            ops.attention(q, k[:, :a.local], v[:, :a.local], out=o, kv_splits=s_loc, parts=(0, n, True))
            ops.attention(q, k[:, a.local:], v[:, a.local:], out=o, kv_splits=s_rem, parts=(s_loc, n, False))
        ms = _time(fn, a.iters)
        return {"kernel": "attn_sp", "B": a.B, "H": a.H, "Lq": a.Lq, "Lk": a.Lk, "local": a.local, "s_loc": s_loc,
                "s_rem": s_rem, "ms": ms, "tflops": 4 * a.B * a.H * a.Lq * a.Lk * 128 / ms / 1e9}
    ms = _time(lambda: ops.attention(q, k, v, out=o, fp8=a.fp8, kv_splits=a.kv_splits or None), a.iters)
    return {"kernel": "attn_fp8" if a.fp8 else "attn", "B": a.B, "H": a.H, "Lq": a.Lq, "Lk": a.Lk,
            "kv_splits": a.kv_splits, "ms": ms, "tflops": 4 * a.B * a.H * a.Lq * a.Lk * 128 / ms / 1e9}


def bench_ln(a):
    dev = "cuda"
    x = torch.randn(a.M, a.C, device=dev)
    if not a.f32:
        x = x.to(torch.bfloat16)
    mod = torch.zeros(6, a.C, device=dev, dtype=torch.bfloat16)
    e0 = torch.zeros(21, 6, a.C, device=dev)
    out = torch.empty(a.M, a.C, device=dev, dtype=torch.bfloat16)
    ms = _time(lambda: ops.layernorm_modulate(x, mod, e0, 0, 1, (a.M, max(1, a.M // 21)), out=out), a.iters)
    return {"kernel": "layernorm_modulate", "M": a.M, "C": a.C, "x_f32": a.f32, "ms": ms,
            "gbs": (x.element_size() + 2) * a.M * a.C / ms / 1e6}


def bench_qknorm(a):
    """q and k sections of a [M, 3C] QKV buffer normed and rotated in place, B = 2 sequences of M / 2
    tokens; the sums of squares formed by the kernel (--ss self, one GPU), or given as a GEMM's
    32-column chunk partials or as finished sums (the TP path)."""
    dev = "cuda"
    C, M = a.C, a.M
    qkv = torch.randn(M, 3 * C, device=dev).to(torch.bfloat16)
    part = torch.rand(M, 2 * C // 32, device=dev) * 32
    g = torch.ones(C, device=dev, dtype=torch.bfloat16)
    Lx = max(1, M // 2)
    ang = torch.rand(Lx, 64, device=dev)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    P = C // 32
    if a.ss == "sums":  # finished per-row sums (the TP path, after the all-reduce)
        ss = part[:, :2].t().contiguous()
        fn = lambda: ops.qk_norm_rope(qkv, [(0, ss[0], g), (C, ss[1], g)], C, C, cos=cos, sin=sin, seq_len=Lx)
        P = 1
    elif a.ss == "self":
        fn = lambda: ops.qk_norm_rope(qkv, [(0, None, g), (C, None, g)], C, C, cos=cos, sin=sin, seq_len=Lx)
        P = 0
    else:
        fn = lambda: ops.qk_norm_rope(qkv, [(0, part[:, :P], g), (C, part[:, P:], g)], C, C, cos=cos, sin=sin,
                                      seq_len=Lx)
    ms = _time(fn, a.iters)
    nbytes = 2 * (4 * M * C + 4 * M * P)
    return {"kernel": "qk_norm_rope", "M": M, "C": C, "ss": a.ss, "ms": ms, "gbs": nbytes / ms / 1e6}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kind", choices=["gemm", "attn", "ln", "qknorm"])
    ap.add_argument("--M", type=int, default=15708)
    ap.add_argument("--N", type=int, default=14336)
    ap.add_argument("--K", type=int, default=3072)
    ap.add_argument("--C", type=int, default=3072)
    ap.add_argument("--epi", default="gelu", choices=sorted(EPIS))
    ap.add_argument("--B", type=int, default=2)
    ap.add_argument("--H", type=int, default=24)
    ap.add_argument("--Lq", type=int, default=7854)
    ap.add_argument("--Lk", type=int, default=7854)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--tile-n", type=int, default=0, help="gemm tile width along N (0 = the library's choice)")
    ap.add_argument("--kv-splits", type=int, default=0, help="attn: key splits (0 = the library's choice)")
    ap.add_argument("--local", type=int, default=0, help="attn: the Q-local SP pattern with this many local keys")
    ap.add_argument("--kv-splits-rem", type=int, default=0, help="attn --local: splits of the remote keys")
    ap.add_argument("--fp8", action="store_true", help="attn: the e4m3 variant (quantisation included in the time)")
    ap.add_argument("--f32", action="store_true", help="gemm residual epilogues / ln: the fp32 residual stream")
    ap.add_argument("--ss", default="self", choices=["self", "partials", "sums"], help="qknorm: where the sums of squares come from")
    a = ap.parse_args()
    torch.cuda.set_device(0)
    r = {"gemm": bench_gemm, "attn": bench_attn, "ln": bench_ln, "qknorm": bench_qknorm}[a.kind](a)
    r["device_error"] = L.device_error(reset=True)
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
