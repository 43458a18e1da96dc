"""Torch-facing wrappers of the libwanb200 entry points.

Each function takes CUDA tensors, checks dtype / layout on the host, fills the C parameter
struct and launches on the current torch stream.  There is no eager fallback: a missing
library or a non-CUDA tensor raises.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib as L

BF16 = torch.bfloat16


class KernelTimer:
    """Optional per-launch CUDA-event timing of the ops below, by kernel class.

    While installed with `set_timer`, every op records an event pair on the launching stream
    and its algorithmic work (FLOPs for tensor-core kernels, bytes for HBM-bound ones).
    `summary()` synchronizes and returns {kind: (launches, total_ms, total_work)}.
    """

    def __init__(self):
        self.records = []

    def begin(self, t):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(t.device))
        return ev

    def end(self, t, start, kind, work):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(t.device))
        self.records.append((kind, start, ev, work))

    def summary(self):
        torch.cuda.synchronize()
        out = {}
        for kind, s, e, work in self.records:
            n, ms, w = out.get(kind, (0, 0.0, 0.0))
            out[kind] = (n + 1, ms + s.elapsed_time(e), w + work)
        return out


_timer = None
launch_count = 0


def set_timer(timer):
    global _timer
    _timer = timer


def _launch(t, kind, work, fn):
    global launch_count
    launch_count += 1
    if _timer is None:
        return fn()
    s = _timer.begin(t)
    rc = fn()
    _timer.end(t, s, kind, work)
    return rc


def region_begin(t):
    """Start of a timed region on t's current stream (None when no KernelTimer is installed)."""
    return _timer.begin(t) if _timer is not None else None


def region_end(t, start, kind, work):
    """End of a region started by region_begin: recorded under `kind` with `work` (bytes)."""
    if _timer is not None and start is not None:
        _timer.end(t, start, kind, work)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need(cond: bool, msg: str):
    if not cond:
        raise ValueError(msg)


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise L.WanB200Error("libwanb200 ops need CUDA tensors (no CPU fallback)")


def _p(t):
    return None if t is None else t.data_ptr()


def _set_frames(p, frames):
    """frames = (seq_len, tokens_per_frame[, row_offset[, rows_per_seq]]): row r holds token
    t = (r % rows_per_seq if rows_per_seq else r) + row_offset of its sequence and belongs to
    latent frame (t % seq_len) // tokens_per_frame."""
    p.seq_len, p.tokens_per_frame = frames[0], frames[1]
    p.row_offset = frames[2] if len(frames) > 2 else 0
    p.rows_per_seq = frames[3] if len(frames) > 3 else 0


def _rows(t: torch.Tensor, name: str):
    _need(t.dim() == 2 and t.stride(1) == 1, f"{name} must be 2-D with unit column stride")
    return t.stride(0)


# ---------------------------------------------------------------------------- GEMM
def linear(a, w, bias=None, *, epilogue=L.EPI_BIAS, out=None, residual=None, gate=None, frames=None,
           rowss=None, ss_cols=0, kind="gemm", scatter=None, tile_n=0):
    """out[M, N] = epilogue(a[M, K] @ w[N, K]^T) on tcgen05 (see include/wanb200.h).

    tile_n: width of the output tile along N (0 = the library's choice; 64..256, multiple of 32).

    gate: (gate_mod [N] bf16, gate_e0 [F, N] fp32 view with unit column stride) for EPI_BIAS_GATE_RES.
    frames: (seq_len, tokens_per_frame) mapping a row to its latent frame.
    rowss: fp32 [M, ss_cols / 32] for EPI_BIAS_SUMSQ: rowss[r, k] receives row r's sum of squares
    over output columns 32k .. 32k+31 (written, not accumulated; see qk_norm_rope / sumsq_reduce).
    residual / out may be fp32 for the residual epilogues (the fp32 residual stream).
    """
    _cuda(a, w, bias, out, residual, rowss)
    _need(a.dtype == BF16 and w.dtype == BF16, "linear: a and w must be bf16")
    lda, ldw = _rows(a, "a"), _rows(w, "w")
    M, K = a.shape
    N = w.shape[0]
    _need(w.shape[1] == K, f"linear: a is [*, {K}] but w is {tuple(w.shape)}")
    if out is None and scatter is None:
        out = torch.empty(M, N, dtype=BF16, device=a.device)
    ldd = _rows(out, "out") if out is not None else N  # scatter: rows land in the peers' inboxes
    for name, t in (("out", out), ("residual", residual)):
        _need(t is None or t.dtype in (BF16, torch.float32), f"linear: {name} must be bf16 or fp32")
    p = L.GemmParams()
    p.out_f32 = int(out is not None and out.dtype == torch.float32)
    p.residual_f32 = int(residual is not None and residual.dtype == torch.float32)
    p.a, p.lda, p.w, p.ldw, p.d, p.ldd = _p(a), lda, _p(w), ldw, _p(out), ldd
    p.M, p.N, p.K, p.epilogue = M, N, K, epilogue
    p.tile_n = tile_n
    p.bias = _p(bias)
    if residual is not None:
        p.residual, p.ldr = _p(residual), _rows(residual, "residual")
    if gate is not None:
        gm, ge = gate
        _need(gm.dtype == BF16 and ge.dtype == torch.float32 and ge.stride(-1) == 1, "linear: bad gate tensors")
        p.gate_mod, p.gate_e0, p.gate_frame_stride = _p(gm), _p(ge), ge.stride(0)
    if frames is not None:
        _set_frames(p, frames)
    if rowss is not None:
        _need(rowss.dtype == torch.float32 and rowss.is_contiguous() and rowss.numel() >= (ss_cols // 32) * M,
              "linear: rowss must be contiguous fp32 [M, ss_cols / 32]")
        p.rowss, p.ss_cols = _p(rowss), ss_cols
    if scatter is not None:  # (peer inbox pointers, this rank, rows per shard)
        ptrs, src, shard_rows = scatter
        _need(epilogue == L.EPI_SCATTER and 1 <= len(ptrs) <= L.MAX_PEERS, "linear: bad scatter")
        for i, q in enumerate(ptrs):
            p.peer_out[i] = q
        p.npeers, p.src_rank, p.shard_rows = len(ptrs), src, shard_rows
    lib = L.load()
    L.check(_launch(a, kind, 2.0 * M * N * K, lambda: lib.wanb200_gemm_bf16(ctypes.byref(p), _stream(a))),
            "wanb200_gemm_bf16")
    return out


# ---------------------------------------------------------------------------- attention
_WORKSPACES = {}


def _workspace(device, nbytes):
    """A per-device scratch buffer of at least nbytes (grown on demand, reused by every launch on
    the stream; launches on one stream are ordered, so reuse is safe)."""
    key = str(device)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = _WORKSPACES[key] = torch.empty(nbytes, dtype=torch.uint8, device=device)
    return ws


def kv_splits(batch, heads, q_len, kv_len) -> int:
    """The library's split-KV count for an attention of this shape (wanb200_attn_kv_splits)."""
    return L.load().wanb200_attn_kv_splits(batch, heads, q_len, kv_len)


_FP8_WORKSPACES = {}


def attention(q, k, v, out=None, softmax_scale=None, kind="attn", kv_splits=None, parts=None, fp8=False):
    """o = softmax(q k^T * scale) v on [B, L, H, 128] tensors (head stride 128, unit d stride).
    kv_splits: None = the library's choice for the grid size, 1 = no split.
    parts: (slot0, nslots, defer_combine) when the key set comes in pieces: this launch writes
    partial slots slot0.. of a workspace of nslots slots, and merges all of them into `out`
    unless defer_combine (wanb200_attn_params).
    fp8: the e4m3 variant (wanb200_attn_fwd_fp8): q, k, v are quantised with per-block scales
    inside the call; the result differs from the bf16 path by the e4m3 rounding."""
    _cuda(q, k, v, out)
    for name, t in (("q", q), ("k", k), ("v", v)):
        _need(t.dtype == BF16 and t.dim() == 4 and t.shape[-1] == 128 and t.stride(3) == 1 and t.stride(2) == 128,
              f"attention: {name} must be bf16 [B, L, H, 128] with head stride 128")
    B, Lq, H, D = q.shape
    _need(k.shape[0] == B and k.shape[2] == H and v.shape == k.shape, "attention: q/k/v shape mismatch")
    if out is None:
        out = torch.empty(B, Lq, H, D, dtype=BF16, device=q.device)
    _need(out.stride(3) == 1 and out.stride(2) == 128, "attention: out must have head stride 128")
    p = L.AttnParams()
    p.q, p.q_tok_stride, p.q_batch_stride = _p(q), q.stride(1), q.stride(0)
    p.k, p.k_tok_stride, p.k_batch_stride = _p(k), k.stride(1), k.stride(0)
    p.v, p.v_tok_stride, p.v_batch_stride = _p(v), v.stride(1), v.stride(0)
    p.o, p.o_tok_stride, p.o_batch_stride = _p(out), out.stride(1), out.stride(0)
    p.batch, p.heads, p.q_len, p.kv_len, p.head_dim = B, H, Lq, k.shape[1], D
    p.softmax_scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    lib = L.load()
    splits = kv_splits if kv_splits is not None else lib.wanb200_attn_kv_splits(B, H, Lq, k.shape[1])
    p.kv_splits = splits
    slots = splits
    if parts is not None:
        p.part_slot0, p.part_nslots, p.defer_combine = parts[0], parts[1], int(bool(parts[2]))
        slots = parts[1]
    if slots > 1:
        nbytes = lib.wanb200_attn_workspace_bytes(B, H, Lq, slots)
        p.workspace, p.workspace_bytes = _workspace(q.device, nbytes).data_ptr(), nbytes
    flops = 4.0 * B * H * Lq * k.shape[1] * D
    if fp8:
        f = L.AttnFp8Params()
        f.attn = p
        nb = lib.wanb200_attn_fp8_workspace_bytes(B, H, Lq, k.shape[1])
        key = str(q.device)
        ws = _FP8_WORKSPACES.get(key)
        if ws is None or ws.numel() < nb:
            ws = _FP8_WORKSPACES[key] = torch.empty(nb, dtype=torch.uint8, device=q.device)
        f.fp8_workspace, f.fp8_workspace_bytes = ws.data_ptr(), nb
        L.check(_launch(q, kind, flops, lambda: lib.wanb200_attn_fwd_fp8(ctypes.byref(f), _stream(q))),
                "wanb200_attn_fwd_fp8")
        return out
    L.check(_launch(q, kind, flops, lambda: lib.wanb200_attn_fwd(ctypes.byref(p), _stream(q))), "wanb200_attn_fwd")
    return out


# ---------------------------------------------------------------------------- norms
def _set_push(p, push):
    """push = (peer buffer pointers, first row): also store the output rows into every peer buffer
    at rows first_row.. (the all-gather fused into the norm)."""
    if push is not None:
        ptrs, row0 = push
        _need(1 <= len(ptrs) <= L.MAX_PEERS, "layernorm: bad push")
        for i, q in enumerate(ptrs):
            p.push_out[i] = q
        p.npush, p.push_row0 = len(ptrs), row0


def _ln_input(x):
    _need(x.dtype in (BF16, torch.float32) and x.is_contiguous() and x.dim() == 2,
          "layernorm: x must be contiguous bf16 or fp32 [M, C]")


def layernorm_modulate(x, modulation, e0, shift_idx, scale_idx, frames, out=None, eps=1e-6, push=None,
                       one_row=False):
    """LN(x) * (1 + scale[f]) + shift[f] -> bf16; x [M, C] bf16 or fp32 (the fp32 residual
    stream), modulation [6, C] bf16, e0 [F, 6, C] fp32.  one_row: the head's modulation
    (modulation [2, C], e0 [F, C]: shift and scale both add the frame's time-embedding row)."""
    _cuda(x, modulation, e0, out)
    _ln_input(x)
    _need(e0.dtype == torch.float32 and e0.is_contiguous() and modulation.dtype == BF16, "layernorm: bad mod tensors")
    M, C = x.shape
    if out is None and push is None:
        out = torch.empty(M, C, dtype=BF16, device=x.device)
    p = L.LnParams()
    p.x_f32 = int(x.dtype == torch.float32)
    p.e0_one_row = int(one_row)
    _set_push(p, push)
    p.x, p.out, p.rows, p.dim, p.eps, p.mode = _p(x), _p(out), M, C, eps, L.LN_MODULATE
    p.modulation, p.e0, p.e0_frame_stride = _p(modulation), _p(e0), (C if one_row else 6 * C)
    p.shift_idx, p.scale_idx = shift_idx, scale_idx
    _set_frames(p, frames)
    lib = L.load()
    L.check(_launch(x, "layernorm", (x.element_size() + 2.0) * M * C,
                    lambda: lib.wanb200_layernorm(ctypes.byref(p), _stream(x))), "wanb200_layernorm")
    return out


def layernorm_affine(x, weight, bias, out=None, eps=1e-6):
    """LN(x) * weight + bias -> bf16; x [M, C] bf16 or fp32."""
    _cuda(x, weight, bias, out)
    _ln_input(x)
    M, C = x.shape
    if out is None:
        out = torch.empty(M, C, dtype=BF16, device=x.device)
    p = L.LnParams()
    p.x_f32 = int(x.dtype == torch.float32)
    p.x, p.out, p.rows, p.dim, p.eps, p.mode = _p(x), _p(out), M, C, eps, L.LN_AFFINE
    p.weight, p.bias = _p(weight), _p(bias)
    lib = L.load()
    L.check(_launch(x, "layernorm", (x.element_size() + 2.0) * M * C,
                    lambda: lib.wanb200_layernorm(ctypes.byref(p), _stream(x))), "wanb200_layernorm")
    return out


def qk_norm_rope(x, sections, width, global_dim, eps=1e-6, cos=None, sin=None, seq_len=0):
    """In place on x [M, ld]: for each (col0, ss, gamma [width] bf16) section,
    x[:, col0:col0+width] = RoPE(x * rsqrt(S/global_dim + eps) * gamma) (RoPE if cos given).

    ss is None (the kernel forms S from the section's own bf16 values: one GPU, the section is the
    whole global dim), [M] fp32 (finished sums S, e.g. after the TP all-reduce) or an [M, P] fp32
    view with unit column stride: P partial sums per row (the SUMSQ GEMM's 32-column chunks, e.g.
    a column slice of its [M, 2P] output) that the kernel adds in a fixed order.  Every section
    takes the same form."""
    _cuda(x, cos, sin)
    ld = _rows(x, "x")
    p = L.QkNormParams()
    p.x, p.ld, p.rows, p.nsections, p.width = _p(x), ld, x.shape[0], len(sections), width
    M = x.shape[0]
    forms = set()
    for i, (c0, ss, g) in enumerate(sections):
        _cuda(ss, g)
        _need(g.dtype == BF16 and (ss is None or ss.dtype == torch.float32), "qk_norm_rope: ss fp32, gamma bf16")
        if ss is None:
            forms.add((0, 0))
        elif ss.dim() == 1:
            _need(ss.numel() >= M and ss.stride(0) == 1, "qk_norm_rope: ss must hold a sum per row")
            forms.add((1, 1))
        else:
            _need(ss.dim() == 2 and ss.shape[0] >= M and ss.stride(1) == 1, "qk_norm_rope: ss partials must be [M, P]")
            forms.add((ss.shape[1], ss.stride(0)))
        p.col0[i], p.ss[i], p.gamma[i] = c0, _p(ss), _p(g)
    _need(len(forms) == 1, "qk_norm_rope: every section's ss must have the same partial count and row stride")
    p.ss_parts, p.ss_row_stride = forms.pop()
    if p.ss_parts == 0:
        p.ss_parts = 1
    p.inv_dim, p.eps = 1.0 / global_dim, eps
    if cos is not None:
        _need(cos.dtype == torch.float32 and cos.is_contiguous() and sin.is_contiguous(), "qk_norm_rope: bad tables")
        p.rope, p.cos, p.sin, p.seq_len = 1, _p(cos), _p(sin), seq_len
    lib = L.load()
    nbytes = 4.0 * M * width * len(sections) + (0.0 if sections[0][1] is None else 4.0 * M * p.ss_parts * len(sections))
    L.check(_launch(x, "qk_norm_rope", nbytes, lambda: lib.wanb200_qk_norm_rope(ctypes.byref(p), _stream(x))),
            "wanb200_qk_norm_rope")
    return x


def sumsq_reduce(part, part0, parts, out):
    """out[s, r] = part[r, part0[s]] + ... + part[r, part0[s] + parts - 1] (added in that order) for
    the one or two sections s, part [M, P] fp32 (the SUMSQ GEMM's chunk partials): the per-rank
    sums of squares ahead of the TP all-reduce.  out: [sections, M] or [M] for one section."""
    _cuda(part, out)
    _need(part.dtype == torch.float32 and part.dim() == 2 and part.stride(1) == 1, "sumsq_reduce: part [M, P] fp32")
    _need(out.dtype == torch.float32 and out.stride(-1) == 1 and 1 <= len(part0) <= 2, "sumsq_reduce: bad out")
    M = part.shape[0]
    out2 = out if out.dim() == 2 else out.view(1, -1)
    _need(out2.shape[0] == len(part0) and out2.shape[1] >= M, "sumsq_reduce: out must be [sections, M]")
    _need(all(0 <= q and q + parts <= part.shape[1] for q in part0), "sumsq_reduce: partials out of range")
    p = L.SumsqReduceParams()
    p.part, p.rows, p.row_stride, p.nsections, p.parts, p.out = _p(part), M, part.stride(0), len(part0), parts, _p(out2)
    p.out_stride = out2.stride(0) if out2.shape[0] > 1 else M
    for i, q in enumerate(part0):
        p.part0[i] = q
    lib = L.load()
    L.check(_launch(part, "sumsq_reduce", 4.0 * M * (parts + 1) * len(part0),
                    lambda: lib.wanb200_sumsq_reduce(ctypes.byref(p), _stream(part))), "wanb200_sumsq_reduce")
    return out


def bias_gate_residual(residual, y, bias, gate=None, frames=None, out=None, nsum=1):
    """out = residual + (y + bias) * gate[f]  (or residual + y + bias without gate).
    nsum > 1: y is [nsum * M, C] (the inbox of a fused reduce-scatter) and its nsum slices of M
    rows are summed first.  residual / out: bf16 or fp32 (the fp32 residual stream); y bf16."""
    _cuda(residual, y, bias, out)
    M, C = residual.shape
    _need(residual.is_contiguous() and y.is_contiguous() and tuple(y.shape) == (nsum * M, C),
          "bias_gate_residual: layout")
    if out is None:
        out = torch.empty_like(residual)
    _need(out.is_contiguous() and tuple(out.shape) == (M, C), "bias_gate_residual: out layout")
    for name, t in (("out", out), ("residual", residual)):
        _need(t.dtype in (BF16, torch.float32), f"bias_gate_residual: {name} must be bf16 or fp32")
    p = L.ResidualParams()
    p.residual_f32, p.out_f32 = int(residual.dtype == torch.float32), int(out.dtype == torch.float32)
    p.out, p.residual, p.y, p.rows, p.dim, p.bias = _p(out), _p(residual), _p(y), M, C, _p(bias)
    p.nsum, p.y_slice_stride = nsum, M * C
    if gate is not None:
        gm, ge = gate
        p.gate_mod, p.gate_e0, p.gate_frame_stride = _p(gm), _p(ge), ge.stride(0)
        _set_frames(p, frames)
    lib = L.load()
    L.check(_launch(residual, "bias_gate_residual", (residual.element_size() + 2.0 * nsum + out.element_size()) * M * C,
                    lambda: lib.wanb200_bias_gate_residual(ctypes.byref(p), _stream(residual))),
            "wanb200_bias_gate_residual")
    return out


# ---------------------------------------------------------------------------- embeddings / head
def patchify(latent, patch, batch, out=None):
    """The Conv3d patchify of latent [C, F, H, W] (fp32 or bf16) -> [batch, L, C*pf*ph*pw] bf16,
    the same rows in every batch copy (wanb200_patchify)."""
    _cuda(latent, out)
    _need(latent.dim() == 4 and latent.is_contiguous() and latent.dtype in (torch.float32, BF16),
          "patchify: latent must be contiguous fp32 / bf16 [C, F, H, W]")
    Cc, Fr, H, W = latent.shape
    pf, ph, pw = patch
    L_ = (Fr // pf) * (H // ph) * (W // pw)
    if out is None:
        out = torch.empty(batch, L_, Cc * pf * ph * pw, dtype=BF16, device=latent.device)
    p = L.PatchifyParams()
    p.latent, p.latent_f32 = latent.data_ptr(), int(latent.dtype == torch.float32)
    p.channels, p.frames, p.height, p.width = Cc, Fr, H, W
    p.pf, p.ph, p.pw, p.batch, p.out = pf, ph, pw, batch, out.data_ptr()
    lib = L.load()
    L.check(_launch(latent, "patchify", float(latent.numel() * latent.element_size() + out.numel() * 2),
                    lambda: lib.wanb200_patchify(ctypes.byref(p), _stream(latent))), "wanb200_patchify")
    return out


def unpatchify_cfg(y, grid, patch, channels, mode, guide, out_dtype=BF16):
    """Head output y [B, L, pf*ph*pw*C] fp32 -> [C, F*pf, H*ph, W*pw] with the CFG combine
    (mode L.CFG_COMBINE: B = 2, uncond + guide (cond - uncond); L.CFG_SCALE: guide * y[0])."""
    _cuda(y)
    _need(y.dtype == torch.float32 and y.is_contiguous(), "unpatchify: y must be contiguous fp32")
    f, h, w = grid
    pf, ph, pw = patch
    out = torch.empty(channels, f * pf, h * ph, w * pw, dtype=out_dtype, device=y.device)
    p = L.UnpatchifyParams()
    p.y, p.batch, p.frames, p.height, p.width = y.data_ptr(), y.shape[0], f, h, w
    p.pf, p.ph, p.pw, p.channels, p.mode, p.guide = pf, ph, pw, channels, mode, guide
    p.out, p.out_f32 = out.data_ptr(), int(out_dtype == torch.float32)
    lib = L.load()
    L.check(_launch(y, "unpatchify", float(y.numel() * 4 + out.numel() * out.element_size()),
                    lambda: lib.wanb200_unpatchify_cfg(ctypes.byref(p), _stream(y))), "wanb200_unpatchify_cfg")
    return out


class _OnDevice:
    """Stands in for a tensor in `_launch` where an op has none: only `.device` is read."""

    def __init__(self, device):
        self.device = torch.device(device)


def peer_barrier(flag_ptrs, rank, epoch, device):
    """Barrier of the TP group over NVLink peer memory (include/wanb200.h, wanb200_peer_barrier)."""
    arr = (ctypes.c_void_p * len(flag_ptrs))(*flag_ptrs)
    lib = L.load()
    st = torch.cuda.current_stream(device).cuda_stream
    L.check(_launch(_OnDevice(device), "peer_barrier", 0.0,
                    lambda: lib.wanb200_peer_barrier(arr, rank, len(flag_ptrs), epoch, st)), "wanb200_peer_barrier")


def shard_gather(src, batch, shard_rows, valid_rows, dst_ptrs, dst_ld, dst_batch_stride, dst_rows, device):
    """Push this rank's shard rows into gathered buffers (include/wanb200.h,
    wanb200_shard_gather).  src: [batch * shard_rows, width] bf16 view with unit column stride
    (e.g. the k|v columns of the QKV buffer); dst_ptrs: device addresses of the gathered buffers
    (peer-mapped), all with row stride dst_ld and batch stride dst_batch_stride elements;
    dst_rows[i]: the row of dst_ptrs[i] that receives shard row 0."""
    _cuda(src)
    _need(src.dtype == BF16, "shard_gather: src must be bf16")
    _need(src.shape[0] >= batch * shard_rows, "shard_gather: src has fewer than batch * shard_rows rows")
    p = L.ShardGatherParams()
    p.src, p.src_ld = src.data_ptr(), _rows(src, "src")
    p.batch, p.shard_rows, p.valid_rows, p.width = batch, shard_rows, valid_rows, src.shape[1]
    for i, ptr in enumerate(dst_ptrs):
        p.dst[i] = ptr
    p.ndst = len(dst_ptrs)
    p.dst_ld, p.dst_batch_stride = dst_ld, dst_batch_stride
    for i, r in enumerate(dst_rows):
        p.dst_row0[i] = r
    lib = L.load()
    nbytes = 2.0 * batch * valid_rows * src.shape[1] * (1 + len(dst_ptrs))  # local read + one write per rank
    L.check(_launch(src, "kv_gather", nbytes, lambda: lib.wanb200_shard_gather(ctypes.byref(p), _stream(src))),
            "wanb200_shard_gather")


# ---------------------------------------------------------------------------- torch.library ops
# The attention seam of the reference (`fn(q, k, v) -> o`, models/fast_dit.py:186-255) as a
# custom op with a fake kernel, so the device path can sit under torch.compile / CUDA graphs.
@torch.library.custom_op("wanb200::attn", mutates_args=())
def attn_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    return attention(q, k, v, softmax_scale=softmax_scale)


@attn_op.register_fake
def _(q, k, v, softmax_scale):
    return torch.empty(q.shape[0], q.shape[1], q.shape[2], q.shape[3], dtype=q.dtype, device=q.device)


# The cross-attention seam (`_nki_cross` / `_cte` over the cached text K/V, fast_dit.py:244-255):
# q [B, L, H, 128] against ck / cv [B, Lc, H, 128].
@torch.library.custom_op("wanb200::cross_attn", mutates_args=())
def cross_attn_op(q: torch.Tensor, ck: torch.Tensor, cv: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    return attention(q, ck, cv, softmax_scale=softmax_scale, kind="attn_cross")


@cross_attn_op.register_fake
def _(q, ck, cv, softmax_scale):
    return torch.empty(q.shape[0], q.shape[1], q.shape[2], q.shape[3], dtype=q.dtype, device=q.device)
