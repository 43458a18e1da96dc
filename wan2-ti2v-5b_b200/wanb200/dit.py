"""FastWanDiT on the B200 kernels: the denoise-step driver around the 30 block ops.

Mirrors `FastWanDiT` of models/fast_dit.py:561-697:
    fast = FastWanDiT(model, grid=(F, H/2, W/2), guide_scale=5.0, device=dev)
    fast.set_context(ctx_cond, ctx_null)     # [1, 512, 4096] each, once per prompt
    noise_pred = fast(latent, t)             # latent [48, F, H, W], t scalar -> [48, F, H, W]

`model` is either a reference `WanModel` (any object with `.state_dict()` and the WanModel
config attributes) or a `(WanSpec, state_dict)` pair.

Layouts (as the reference's):
  * batched CFG (`cfg_group=None`): cond and uncond run as a batch of 2 through every block;
  * CFG-parallel (`cfg_group=0/1`, inference_neuron_ti2v.py:241-274): this rank's group runs
    only the cond (0) or uncond (1) branch at batch 1, and the head sums w * pred over
    `pair_group` (the same TP rank of the other group), w = g or 1 - g (fast_dit.py:508-524);
  * TP inside a group (`tp_group` of size T > 1): each rank holds 24/T heads and 1/T of the
    FFN, and the block ops all-reduce over the group (`shard_model_tp`, tp_utils.py:378-458).

The time / text / patch embeddings and the head (about 1% of the step) run on the library's
kernels too (tcgen05 GEMMs, the LayerNorm, patchify / unpatchify gathers), in the reference's
bf16 dtype flow, so a step launches nothing but the library's kernels (plus the NCCL collectives
of the multi-GPU layouts).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib as L
from . import ops
from . import block as _block_mod
from .block import FastBlock, FastBlockSP, FastCrossKV, register_block
from .weights import BlockWeights, WanSpec, block_state

BF16 = torch.bfloat16


def rope_params(max_seq_len: int, dim: int, theta: float = 10000.0) -> torch.Tensor:
    """[max_seq_len, dim/2] angles (wan/modules/rope_neuron.py:14-24)."""
    inv = 1.0 / torch.pow(theta, torch.arange(0, dim, 2).float().div(dim))
    return torch.outer(torch.arange(max_seq_len).float(), inv)


def model_freqs(head_dim: int) -> torch.Tensor:
    d = head_dim
    return torch.cat([rope_params(1024, d - 4 * (d // 6)), rope_params(1024, 2 * (d // 6)),
                      rope_params(1024, 2 * (d // 6))], dim=1)


def rope_tables(grid, head_dim: int, device):
    """cos/sin [1, L, 1, d/2] fp32 for a (F, H, W) token grid (models/fast_dit.py:548-558)."""
    f, h, w = grid
    c = head_dim // 2
    fr = model_freqs(head_dim).split([c - 2 * (c // 3), c // 3, c // 3], dim=1)
    ang = torch.cat([fr[0][:f].view(f, 1, 1, -1).expand(f, h, w, -1),
                     fr[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
                     fr[2][:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(1, f * h * w, 1, c)
    return torch.cos(ang).to(device), torch.sin(ang).to(device)


def sinusoidal_embedding_1d(dim: int, position: torch.Tensor) -> torch.Tensor:
    """(wan/modules/model.py:15-25) in float64."""
    half = dim // 2
    position = position.type(torch.float64)
    s = torch.outer(position, torch.pow(10000, -torch.arange(half).to(position).div(half)))
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


def _spec_and_state(model):
    if isinstance(model, tuple):
        return model
    sd = model.state_dict()
    spec = WanSpec(dim=model.dim, ffn_dim=model.ffn_dim, num_heads=model.num_heads, num_layers=len(model.blocks),
                   freq_dim=model.freq_dim, text_dim=model.text_dim, in_dim=model.in_dim, out_dim=model.out_dim,
                   patch_size=tuple(model.patch_size), text_len=model.text_len, eps=model.eps)
    return spec, sd


class FastWanDiT:
    def __init__(self, model, grid, guide_scale, device, cfg_group=None, pair_group=None, tp_group=None,
                 num_layers=None, seq_parallel=None, comm="peer", sp_group=None, attn_fp8=False):
        """seq_parallel: token-sharded residual inside the TP group with local all-head
        cross-attention (`_FastBlockSP`, fast_dit.py:314-389); default on for CFG-parallel with
        TP > 1 (batch 1) and no sp_group, the reference's best layout.
        sp_group: Q-local sequence parallelism (`WanSelfAttentionSP`, dit_attention_sp.py:25-152)
        over this group: each rank runs every block on ceil(L / SP) tokens of each batch element
        and gathers only the normed, rotated K/V of the group (TP inside, by tp_group, as usual);
        the head runs on the token shard and its 4*48-wide output is gathered.
        comm: how the sequence-parallel collectives run: "peer" = fused into the kernels /
        pushed over NVLink peer memory (wanb200.comm), "nccl" = torch.distributed collectives.
        attn_fp8: self-attention in e4m3 (the optional FP8 variant; not with
        seq_parallel)."""
        spec, sd = _spec_and_state(model)
        self.spec = spec
        self.grid = tuple(int(g) for g in grid)
        self.num_frames = self.grid[0]
        self.seq_len = self.grid[0] * self.grid[1] * self.grid[2]
        self.guide_scale = float(guide_scale)
        self.device = torch.device(device)
        self.tp_group = tp_group
        if cfg_group not in (None, 0, 1):
            raise ValueError("cfg_group must be None, 0 (cond) or 1 (uncond)")
        self.cfg_group, self.pair_group = cfg_group, pair_group
        self.batch = 2 if cfg_group is None else 1
        self.cfg_w = None if cfg_group is None else (self.guide_scale if cfg_group == 0 else 1.0 - self.guide_scale)
        tp = dist.get_world_size(tp_group) if (tp_group is not None and dist.is_initialized()) else 1
        rank = dist.get_rank(tp_group) if tp > 1 else 0
        self.tp_size, self.tp_rank = tp, rank
        self.cos, self.sin = rope_tables(self.grid, spec.head_dim, self.device)
        nl = spec.num_layers if num_layers is None else num_layers

        self.ew = self._embedding_weights(sd)
        spn = dist.get_world_size(sp_group) if (sp_group is not None and dist.is_initialized()) else 1
        self.sp_size = spn
        self.sp_rank = dist.get_rank(sp_group) if spn > 1 else 0
        self.sp_group = sp_group if spn > 1 else None
        if seq_parallel is None:
            seq_parallel = cfg_group is not None and tp > 1 and spn == 1
        if seq_parallel and (self.batch != 1 or tp == 1 or spn > 1):
            raise ValueError("seq_parallel needs CFG-parallel (batch 1), a TP group of size > 1 and no sp_group")
        if seq_parallel and attn_fp8:
            raise ValueError("attn_fp8 is available with the tp / sp layouts, not with seq_parallel")
        self.sp = seq_parallel
        self.kv_gather = None
        if spn > 1:
            from .comm import KVGather
            self.kv_gather = KVGather(sp_group, self.batch, self.seq_len, 2 * spec.dim // tp, self.device, comm)
            S = self.kv_gather.S
            pad = spn * S - self.seq_len
            if pad:  # the padded rows of the last shard rotate by zeros (they are never read back)
                self.cos = torch.cat([self.cos, self.cos.new_zeros(1, pad, 1, self.cos.shape[-1])], dim=1)
                self.sin = torch.cat([self.sin, self.sin.new_zeros(1, pad, 1, self.sin.shape[-1])], dim=1)
        self.block_weights = [BlockWeights(block_state(sd, i), spec.num_heads, self.device, rank, tp,
                                           local_cross=seq_parallel) for i in range(nl)]
        self.comm = None
        if seq_parallel:
            if comm == "peer":
                from .comm import PeerComm
                S = -(-self.batch * self.seq_len // tp)
                self.comm = PeerComm(tp_group, S, spec.dim, self.device)
            elif comm != "nccl":
                raise ValueError("comm must be 'peer' or 'nccl'")
            self.blocks = [FastBlockSP(w, self.seq_len, self.num_frames, tp_group, spec.eps, comm=self.comm)
                           for w in self.block_weights]
        else:
            self.blocks = [FastBlock(w, self.num_frames, tp_group, spec.eps, sp=self.kv_gather, attn_fp8=attn_fp8)
                           for w in self.block_weights]
        self.cross_kv = [FastCrossKV(w, tp_group, spec.eps) for w in self.block_weights]
        self.context = None
        self._err_probe = L.DeviceErrorProbe(self.device)
        self._sin_ring, self._sin_slot = None, 0
        self._handles = [register_block(b) for b in self.blocks]  # names for torch.ops.wanb200.block

    @classmethod
    def from_checkpoint(cls, path, grid, guide_scale, device, **kwargs):
        """Build from a Wan2.2 checkpoint directory (config.json + diffusion_pytorch_model
        safetensors, as `WanModel.from_pretrained` reads it; wanb200.checkpoint).  kwargs as for
        the constructor; num_layers also limits which blocks are read."""
        from .checkpoint import load_wan_checkpoint
        return cls(load_wan_checkpoint(path, num_layers=kwargs.get("num_layers")), grid, guide_scale, device,
                   **kwargs)

    # ------------------------------------------------------------------ embeddings and head
    # On the library's kernels, in the reference's bf16 dtype flow (fast_dit.py:658-687, 480-537):
    # the text / time / patch embeddings and the head Linear are tcgen05 GEMMs (fp32 outputs for
    # the residual stream and the modulation rows), the patchify / unpatchify + CFG combine are
    # gather kernels and the head norm is the LayerNorm kernel with the head's modulation.
    def _embedding_weights(self, sd):
        """bf16 copies of the embedding and head parameters in the [out, in] layouts the GEMMs read."""
        C = self.spec.dim

        def g(k, shape=None):
            t = sd[k].to(device=self.device, dtype=BF16)
            return (t.reshape(shape) if shape is not None else t).contiguous()

        return {"patch_w": g("patch_embedding.weight", (C, -1)), "patch_b": g("patch_embedding.bias"),
                "text0_w": g("text_embedding.0.weight"), "text0_b": g("text_embedding.0.bias"),
                "text2_w": g("text_embedding.2.weight"), "text2_b": g("text_embedding.2.bias"),
                "time0_w": g("time_embedding.0.weight"), "time0_b": g("time_embedding.0.bias"),
                "time2_w": g("time_embedding.2.weight"), "time2_b": g("time_embedding.2.bias"),
                "proj_w": g("time_projection.1.weight"), "proj_b": g("time_projection.1.bias"),
                "head_mod": g("head.modulation", (2, C)), "head_w": g("head.head.weight"),
                "head_b": g("head.head.bias")}

    def set_context(self, ctx_cond, ctx_null):
        """Text embedding + every block's cross K/V, once per prompt (fast_dit.py:658-664):
        Linear -> GELU(tanh) -> Linear in bf16, as `_FastText` runs it."""
        ew = self.ew
        cond = ctx_cond.reshape(1, -1, ctx_cond.shape[-1])
        null = ctx_null.reshape(1, -1, ctx_null.shape[-1])
        if self.cfg_group is None:
            ctx = torch.cat([cond, null])
        else:
            ctx = cond if self.cfg_group == 0 else null
        B, Lc, Dt = ctx.shape
        ctx = ctx.to(self.device, BF16).reshape(B * Lc, Dt).contiguous()
        h = ops.linear(ctx, ew["text0_w"], ew["text0_b"], epilogue=L.EPI_BIAS_GELU, kind="gemm_text")
        context = ops.linear(h, ew["text2_w"], ew["text2_b"], epilogue=L.EPI_BIAS, kind="gemm_text")
        self.context = [kv(context.view(B, Lc, -1)) for kv in self.cross_kv]

    def _sinusoid_host(self, t):
        """The per-frame sinusoid of timestep t in bf16 on the host (float64 arithmetic, frame 0
        at t = 0, as `_time_embed` computes it, fast_dit.py:677-684)."""
        tf = torch.full((self.num_frames,), float(t), dtype=torch.float64)
        tf[0] = 0.0
        return sinusoidal_embedding_1d(self.spec.freq_dim, tf).to(BF16)

    def _sinusoid(self, t):
        """The per-frame sinusoid of timestep t in bf16 on the device, through a two-slot
        page-locked ring so that the copy is asynchronous."""
        s = self._sinusoid_host(t)
        if self._sin_ring is None:
            self._sin_ring = [[torch.empty_like(s).pin_memory(), torch.empty_like(s, device=self.device), None]
                              for _ in range(2)]
        self._sin_slot ^= 1
        host, dev, ev = self._sin_ring[self._sin_slot]
        if ev is not None:
            ev.synchronize()  # the copy from this slot two steps ago has been read
        host.copy_(s)
        dev.copy_(host, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._sin_ring[self._sin_slot][2] = ev
        return dev

    def time_embed(self, t):
        """Per-frame embedding, frame 0 (the image frame) at t=0 (fast_dit.py:677-687):
        time_embedding = Linear, SiLU, Linear; time_projection = SiLU, Linear.  Returns
        e [F, C] fp32 (the head's modulation rows) and e0 [F, 6, C] fp32 (the blocks')."""
        return self.time_embed_from(self._sinusoid(t))

    def time_embed_from(self, s):
        """time_embed from the sinusoid s [F, freq_dim] bf16 already on the device."""
        ew, F_, C = self.ew, self.num_frames, self.spec.dim
        a1 = ops.linear(s, ew["time0_w"], ew["time0_b"], epilogue=L.EPI_BIAS_SILU, kind="gemm_time")
        e = torch.empty(F_, C, device=self.device, dtype=torch.float32)
        ops.linear(a1, ew["time2_w"], ew["time2_b"], epilogue=L.EPI_BIAS, out=e, kind="gemm_time")
        se = ops.linear(a1, ew["time2_w"], ew["time2_b"], epilogue=L.EPI_BIAS_SILU, kind="gemm_time")
        e0 = torch.empty(F_, 6 * C, device=self.device, dtype=torch.float32)
        ops.linear(se, ew["proj_w"], ew["proj_b"], epilogue=L.EPI_BIAS, out=e0, kind="gemm_time")
        return e, e0.view(F_, 6, C)

    def patch(self, latent):
        """Conv3d patchify (stride = kernel) + the patch-embedding GEMM -> x [B, L, C] fp32, the
        residual stream the blocks carry in fp32 through the step (the latent is rounded to bf16
        on the way in, as `_FastPatch` feeds it, fast_dit.py:690)."""
        ew = self.ew
        lat = latent.to(self.device)
        if lat.dtype not in (torch.float32, BF16):
            lat = lat.float()
        pt = ops.patchify(lat.contiguous(), self.spec.patch_size, self.batch)
        B, Lx, K = pt.shape
        x = torch.empty(B * Lx, self.spec.dim, device=self.device, dtype=torch.float32)
        ops.linear(pt.view(B * Lx, K), ew["patch_w"], ew["patch_b"], epilogue=L.EPI_BIAS, out=x, kind="gemm_patch")
        return x.view(B, Lx, self.spec.dim)

    def head_tokens(self, x, e, row0=0):
        """LN + 2-way modulation + Linear of `_FastHead` (fast_dit.py:480-505) per token:
        x [B, n, C] holds tokens row0 .. row0 + n - 1 of each sequence -> [B, n, 4*48] fp32."""
        ew = self.ew
        B, n, C = x.shape
        tpf = self.seq_len // self.num_frames
        h = ops.layernorm_modulate(x.reshape(B * n, C).contiguous(), ew["head_mod"], e.reshape(-1, C).contiguous(),
                                   0, 1, (self.seq_len, tpf, row0, n), eps=self.spec.eps, one_row=True)
        y = torch.empty(B * n, ew["head_w"].shape[0], device=x.device, dtype=torch.float32)
        ops.linear(h, ew["head_w"], ew["head_b"], epilogue=L.EPI_BIAS, out=y, kind="gemm_head")
        return y.view(B, n, -1)

    def head(self, x, e):
        """LN + 2-way modulation + Linear, unpatchify, CFG combine (fast_dit.py:480-505)."""
        return self.combine(self.head_tokens(x, e))

    def combine(self, y):
        """Unpatchify [B, L, 4*48] and combine the CFG branches -> [48, F, H, W] bf16, the dtype
        `_FastHead` / `_FastHeadCfgPar` return (fast_dit.py:503-505, 522-524); the combine runs
        in fp32 and rounds once."""
        y = y.contiguous()
        if self.cfg_group is None:
            return ops.unpatchify_cfg(y, self.grid, self.spec.patch_size, self.spec.out_dim, L.CFG_COMBINE,
                                      self.guide_scale)
        # CFG-parallel: uncond + g (cond - uncond) = g * cond + (1 - g) * uncond, summed over the pair
        out = ops.unpatchify_cfg(y, self.grid, self.spec.patch_size, self.spec.out_dim, L.CFG_SCALE, self.cfg_w,
                                 out_dtype=torch.float32)
        if self.pair_group is not None:
            dist.all_reduce(out, group=self.pair_group)
        return out.to(BF16)

    # ------------------------------------------------------------------ step
    def forward_blocks(self, x, e0):
        for blk, (ck, cv) in zip(self.blocks, self.context):
            x = blk(x, e0, self.cos, self.sin, ck, cv)
        return x

    def forward_blocks_op(self, x, e0):
        """forward_blocks through the torch.ops.wanb200.block custom op (one opaque node per block,
        with a fake kernel), for callers that trace the step with torch.compile / make_fx."""
        for h, (ck, cv) in zip(self._handles, self.context):
            x = torch.ops.wanb200.block(x, e0, self.cos, self.sin, ck, cv, h)
        return x

    def shard(self, x):
        """[B, L, C] -> this rank's [S, C] rows of the flattened tokens, zero-padded to T*S."""
        B, Lx, C = x.shape
        N, T = B * Lx, self.tp_size
        S = -(-N // T)
        flat = x.reshape(N, C)
        if S * T != N:
            flat = torch.cat([flat, flat.new_zeros(S * T - N, C)])
        return flat[self.tp_rank * S:(self.tp_rank + 1) * S].contiguous()

    def unshard(self, xs):
        """All-gather the token shards back to [B, L, C]."""
        S, C = xs.shape
        full = torch.empty(S * self.tp_size, C, dtype=xs.dtype, device=xs.device)
        dist.all_gather_into_tensor(full, xs, group=self.tp_group)
        return full[:self.batch * self.seq_len].view(self.batch, self.seq_len, C)

    def shard_q(self, x):
        """[B, L, C] -> this rank's Q-local shard [B, S, C] (tokens sp_rank*S .., zero-padded)."""
        B, Lx, C = x.shape
        S = self.kv_gather.S
        r0 = self.sp_rank * S
        xs = x.new_zeros(B, S, C)
        n = max(0, min(S, Lx - r0))
        xs[:, :n] = x[:, r0:r0 + n]
        return xs

    def gather_q(self, ys):
        """All-gather the per-shard head outputs [B, S, D] of the SP group -> [B, L, D]."""
        B, S, D = ys.shape
        full = torch.empty(self.sp_size, B, S, D, dtype=ys.dtype, device=ys.device)
        dist.all_gather_into_tensor(full, ys.contiguous(), group=self.sp_group)
        return full.permute(1, 0, 2, 3).reshape(B, self.sp_size * S, D)[:, :self.seq_len]

    def __call__(self, latent, t):
        """One CFG noise prediction: latent [C, F, H, W], timestep t -> [C, F, H, W] bf16.

        Every call queues a read of the device error word behind its launches and checks the
        last read that has landed (a step or two late, without synchronizing), raising
        WanB200Error if a kernel's bounded wait expired; `check_device_errors()` checks now."""
        if self.context is None:
            raise RuntimeError("call set_context() first")
        L.raise_on_device_error(self._err_probe.poll(), "FastWanDiT")
        e, e0 = self.time_embed(t)
        x = self.patch(latent)
        if self.kv_gather is not None:
            xs = self.forward_blocks(self.shard_q(x), e0)
            out = self.combine(self.gather_q(self.head_tokens(xs, e, self.sp_rank * self.kv_gather.S)))
        elif self.sp:
            x = self.unshard(self.forward_blocks(self.shard(x), e0))
            out = self.head(x, e)
        else:
            out = self.head(self.forward_blocks(x, e0), e)
        self._err_probe.post()
        return out

    def check_device_errors(self, raise_error: bool = True) -> int:
        """Wait for the work queued so far and read the device error word: 0, or (raise_error)
        WanB200Error for a bounded wait that expired inside a kernel."""
        code = self._err_probe.wait()
        if raise_error:
            L.raise_on_device_error(code, "FastWanDiT")
        return code

    @property
    def launches_per_step(self) -> int:
        return sum(b.launches for b in self.blocks)

    def capture(self, latent_like) -> "CapturedStep":
        """The whole noise prediction (time and patch embeddings, every block, head, CFG combine)
        captured as one CUDA graph for latents shaped like `latent_like`; single GPU only.  Call
        it after set_context(); it runs the step once to warm up, then captures it."""
        return CapturedStep(self, latent_like)


class CapturedStep:
    """One CFG noise prediction of a single-GPU FastWanDiT, captured as a CUDA graph.

    The graph holds every launch of `FastWanDiT.__call__`: the time-embedding GEMMs (read from a
    static sinusoid buffer), patchify and the patch-embedding GEMM (from a static latent buffer),
    the blocks, the head and the CFG combine (into a static output).  A call computes the sinusoid
    of t on the host, copies it (through page-locked memory) and the latent into the static
    buffers on the current stream, replays the graph and returns a copy of the output: one graph
    launch per step instead of ~400 kernel launches issued from Python.  The kernels and their
    order are the eager step's, so the output is the same bit for bit.  The reference compiles its
    whole step for its device for the same reason (`torch.compile(backend="neuron")` of the
    block stack, fast_dit.py:586, 646-649).

    The cross K/V that set_context() made are baked into the graph by address: after a later
    set_context() a call raises (capture again).  So are the blocks' shared scratch buffers and the
    attention workspaces, which the object keeps alive.  The multi-GPU layouts are refused: their NCCL
    collectives and peer barriers take host-side epochs that a replay would not advance.
    """

    def __init__(self, model: FastWanDiT, latent_like):
        if (model.cfg_group is not None or model.tp_size > 1 or model.sp or model.kv_gather is not None
                or model.pair_group is not None):
            raise ValueError("CapturedStep: single-GPU layout only (no CFG / TP / SP groups)")
        if model.context is None:
            raise RuntimeError("call set_context() first")
        dev = model.device
        self.model = model
        self._ctx = model.context
        self.latent = torch.empty(tuple(latent_like.shape), dtype=latent_like.dtype, device=dev)
        self.latent.copy_(latent_like)
        s = model._sinusoid_host(0.0)
        self._sin_host = torch.empty_like(s).pin_memory()
        self._sin = s.to(dev)
        self._sin_copied = None  # event after the last copy out of _sin_host
        # warm-up outside the capture: every lazy setup (kernel attributes, workspaces) happens here
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._body()
        # the graph reads and writes the shared scratch buffers by address: hold them, so that a
        # later clear_workspaces() or a grown workspace cannot hand their memory to other tensors
        self._keep = (list(_block_mod._WS.values()), list(ops._WORKSPACES.values()),
                      list(ops._FP8_WORKSPACES.values()))

    def _body(self):
        m = self.model
        e, e0 = m.time_embed_from(self._sin)
        return m.head(m.forward_blocks(m.patch(self.latent), e0), e)

    def __call__(self, latent, t):
        """latent [C, F, H, W] (device, or page-locked host memory), timestep t -> [C, F, H, W] bf16."""
        m = self.model
        if m.context is not self._ctx:
            raise RuntimeError("set_context() replaced the cross K/V after the capture: capture again")
        if tuple(latent.shape) != tuple(self.latent.shape):
            raise ValueError(f"latent shape {tuple(latent.shape)} differs from the captured {tuple(self.latent.shape)}")
        L.raise_on_device_error(m._err_probe.poll(), "CapturedStep")
        s = m._sinusoid_host(t)
        if self._sin_copied is not None:
            self._sin_copied.synchronize()  # the previous call's copy has read the page-locked buffer
        self._sin_host.copy_(s)
        stream = torch.cuda.current_stream(m.device)
        self._sin.copy_(self._sin_host, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self._sin_copied = ev
        self.latent.copy_(latent, non_blocking=True)
        self.graph.replay()
        out = self.out.clone()
        m._err_probe.post()
        return out

    def check_device_errors(self, raise_error: bool = True) -> int:
        """FastWanDiT.check_device_errors of the captured model (the denoise loop ends with it)."""
        return self.model.check_device_errors(raise_error)


def block_flops(n_tok: int, seq_len: int, dim: int = 3072, ffn: int = 14336, heads: int = 24, ctx_len: int = 512,
                batch: int = 2) -> dict:
    """Algorithmic FLOPs of one block (the roofline basis): GEMMs N(12C^2 + 4 C F), self-attention
    4 B H L^2 d, cross-attention 4 B H L Lc d."""
    d = dim // heads
    gemm = 2 * n_tok * (6 * dim * dim + 2 * dim * ffn)
    return {"gemm": gemm, "self_attn": 4 * batch * heads * seq_len * seq_len * d,
            "cross_attn": 4 * batch * heads * seq_len * ctx_len * d}
