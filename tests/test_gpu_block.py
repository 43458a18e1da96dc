"""Block- and step-level parity on a B200 against the CPU fp32 oracle (itself pinned to the
reference by tests/golden).  rel-RMS <= 2e-2 per block and <= 5e-2 at
the step-0 noise prediction."""
import os

import pytest
import torch

from oracle import dit_ref as R
from wanb200 import _lib as L
from wanb200 import BlockWeights, FastBlock, FastCrossKV, FastWanDiT, WanSpec, random_block_state
from wanb200.dit import rope_tables

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLD = os.path.join(os.path.dirname(__file__), "golden")
BLOCK_TOL = 2e-2
STEP_TOL = 5e-2


@pytest.fixture(autouse=True)
def _no_device_error():
    L.device_error(reset=True)
    yield
    assert L.device_error(reset=True) == 0


def fp32(sd):
    return {k: v.float() for k, v in sd.items()}


def test_block_matches_reference_golden():
    """The small golden block (dim 256, 2 heads) from the reference's own ref_fp32.block_fwd."""
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    g = torch.load(os.path.join(GOLD, "block_small.pt"), weights_only=False)
    bsd = R.block_params(mg["state_dict"], 0)
    w = BlockWeights(bsd, g["num_heads"], DEV)
    blk = FastBlock(w, g["grid"][0])
    ck, cv = FastCrossKV(w)(g["context"].to(DEV, torch.bfloat16))
    x = g["x"].to(DEV, torch.bfloat16)
    y = blk(x, g["e0"].to(DEV), g["cos"].to(DEV), g["sin"].to(DEV), ck, cv)
    err = R.rel_rms(y.float().cpu(), g["y"])
    assert err < BLOCK_TOL, err
    # the cross K/V on the device against the reference's
    assert R.rel_rms(ck.float().cpu(), g["ck"]) < 1e-2 and R.rel_rms(cv.float().cpu(), g["cv"]) < 1e-2


def test_step_matches_reference_golden():
    """Two-layer model step-0 noise prediction vs the reference's ref_fp32.main() output."""
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    cfg = mg["cfg"]
    spec = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"], num_layers=cfg["num_layers"],
                   freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"], in_dim=cfg["in_dim"], out_dim=cfg["out_dim"],
                   text_len=cfg["text_len"])
    lat = mg["latent"]
    grid = (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2)
    fast = FastWanDiT((spec, mg["state_dict"]), grid, mg["guide"], DEV)
    fast.set_context(mg["ctx"].to(DEV), mg["ctx_null"].to(DEV))
    pred = fast(lat.to(DEV), mg["t"])
    err = R.rel_rms(pred.float().cpu(), mg["noise_pred"])
    assert err < STEP_TOL, err
    # bit-reproducible run to run (the reference compares md5s of its outputs across runs): no
    # atomics anywhere on the path, every reduction in a fixed order
    pred2 = fast(lat.to(DEV), mg["t"])
    assert torch.equal(pred, pred2)


def _config0_inputs(seed=0, L_grid=(6, 12, 15), B=2, Lc=512):
    spec = WanSpec()
    sd = random_block_state(spec, seed)
    g = torch.Generator().manual_seed(seed + 1)
    Lx = L_grid[0] * L_grid[1] * L_grid[2]
    x = torch.randn(B, Lx, spec.dim, generator=g).to(torch.bfloat16).float()
    e0 = torch.randn(1, L_grid[0], 6, spec.dim, generator=g) * 0.1
    context = torch.randn(B, Lc, spec.dim, generator=g).to(torch.bfloat16).float()
    return spec, sd, x, e0, context


def test_block_config0_vs_oracle():
    """Config 0 of the benchmark: one block, dim 3072, 24 heads, B=2, L=1080 (6x12x15), 512 context
    tokens, seeded N(0, 0.02) weights -- device vs the fp32 CPU oracle."""
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    grid = (6, 12, 15)
    spec, sd, x, e0, context = _config0_inputs(L_grid=grid)
    cos, sin = R.rope_tables(R.model_freqs(128), grid, 128)
    p32 = fp32(sd)
    ck, cv = R.cross_kv(p32, context, spec.num_heads)
    y_ref = R.block_fwd(p32, x, e0, cos, sin, ck, cv, grid[0], spec.num_heads)

    w = BlockWeights(sd, spec.num_heads, DEV)
    ckd, cvd = FastCrossKV(w)(context.to(DEV, torch.bfloat16))
    cosd, sind = rope_tables(grid, 128, DEV)
    y = FastBlock(w, grid[0])(x.to(DEV, torch.bfloat16), e0.to(DEV), cosd, sind, ckd, cvd)
    err = R.rel_rms(y.float().cpu(), y_ref)
    upd = R.rel_rms((y.float().cpu() - x), (y_ref - x))
    print(f"config0 block rel-RMS output {err:.2e}, update {upd:.2e}")
    assert err < BLOCK_TOL
    assert upd < 5e-2


def test_block_is_deterministic_and_functional():
    grid = (2, 8, 8)
    spec, sd, x, e0, context = _config0_inputs(seed=3, L_grid=grid, Lc=64)
    w = BlockWeights(sd, spec.num_heads, DEV)
    ck, cv = FastCrossKV(w)(context.to(DEV, torch.bfloat16))
    cos, sin = rope_tables(grid, 128, DEV)
    blk = FastBlock(w, grid[0])
    xd = x.to(DEV, torch.bfloat16)
    x0 = xd.clone()
    y1 = blk(xd, e0.to(DEV), cos, sin, ck, cv).clone()
    y2 = blk(xd, e0.to(DEV), cos, sin, ck, cv)
    assert torch.equal(xd, x0), "the block must not modify its input"
    assert torch.equal(y1, y2), "two runs of the block must agree bit for bit"


def test_block_with_fp8_attention_config0():
    """The optional FP8 variant (config 3) at the block level: self-attention in e4m3
    (per-block scales) against the fp32 oracle and against the bf16 device block.  The output
    stays within the block tolerance; the attention's e4m3 rounding shows in the update."""
    grid = (6, 12, 15)
    spec, sd, x, e0, context = _config0_inputs(L_grid=grid)
    cos, sin = R.rope_tables(R.model_freqs(128), grid, 128)
    p32 = fp32(sd)
    ck, cv = R.cross_kv(p32, context, spec.num_heads)
    y_ref = R.block_fwd(p32, x, e0, cos, sin, ck, cv, grid[0], spec.num_heads)
    w = BlockWeights(sd, spec.num_heads, DEV)
    ckd, cvd = FastCrossKV(w)(context.to(DEV, torch.bfloat16))
    cosd, sind = rope_tables(grid, 128, DEV)
    xd = x.to(DEV, torch.bfloat16)
    y8 = FastBlock(w, grid[0], attn_fp8=True)(xd, e0.to(DEV), cosd, sind, ckd, cvd).float().cpu()
    y16 = FastBlock(w, grid[0])(xd, e0.to(DEV), cosd, sind, ckd, cvd).float().cpu()
    err, upd = R.rel_rms(y8, y_ref), R.rel_rms(y8 - x, y_ref - x)
    upd16 = R.rel_rms(y16 - x, y_ref - x)
    print(f"config0 block, fp8 self-attention: output {err:.2e}, update {upd:.2e} (bf16 update {upd16:.2e})")
    assert err < BLOCK_TOL
    assert upd < 1e-1


def test_step_with_fp8_attention_matches_reference_golden():
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    cfg = mg["cfg"]
    spec = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"], num_layers=cfg["num_layers"],
                   freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"], in_dim=cfg["in_dim"], out_dim=cfg["out_dim"],
                   text_len=cfg["text_len"])
    lat = mg["latent"]
    grid = (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2)
    fast = FastWanDiT((spec, mg["state_dict"]), grid, mg["guide"], DEV, attn_fp8=True)
    fast.set_context(mg["ctx"].to(DEV), mg["ctx_null"].to(DEV))
    err = R.rel_rms(fast(lat.to(DEV), mg["t"]).float().cpu(), mg["noise_pred"])
    print(f"golden step with fp8 self-attention: rel-RMS {err:.3e}")
    assert err < STEP_TOL


def test_denoise_loop_matches_oracle_loop():
    """The denoise loop (the structure of the 27280-token workload) on the golden 2-layer model: three UniPC
    steps with the image frame pinned, the DiT on the device vs the fp32 oracle step on the CPU
    driving the same sampler (itself bit-identical to the reference's scheduler on the CPU)."""
    from wanb200.unipc import FlowUniPC, denoise
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    cfg = mg["cfg"]
    spec = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"], num_layers=cfg["num_layers"],
                   freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"], in_dim=cfg["in_dim"], out_dim=cfg["out_dim"],
                   text_len=cfg["text_len"])
    lat = mg["latent"].float()
    img = torch.randn(lat.shape[0], 1, lat.shape[2], lat.shape[3], generator=torch.Generator().manual_seed(9))
    grid = (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2)
    fast = FastWanDiT((spec, mg["state_dict"]), grid, mg["guide"], DEV)
    fast.set_context(mg["ctx"].to(DEV), mg["ctx_null"].to(DEV))
    out = denoise(fast, lat.to(DEV), 3, 5.0, img.to(DEV)).float().cpu()

    mp = fp32(mg["state_dict"])
    ocfg = {"num_heads": cfg["num_heads"], "num_layers": cfg["num_layers"], "freq_dim": cfg["freq_dim"],
            "patch": cfg["patch"], "out_dim": cfg["out_dim"]}
    ref = denoise(lambda x, t: R.step(mp, ocfg, x, t, mg["ctx"].float(), mg["ctx_null"].float(), mg["guide"]),
                  lat.clone(), 3, 5.0, img, sampler=FlowUniPC())
    err = R.rel_rms(out, ref)
    print(f"3-step denoise loop vs oracle loop: rel-RMS {err:.3e}")
    assert torch.equal(out[:, :1], img)
    assert err < STEP_TOL


def test_block_config2_full_size_vs_oracle():
    """One block at the benchmark's full size (config 2: dim 3072, 24 heads, B=2, L=7854 on the
    21x17x22 grid, 512 context tokens) against the fp32 CPU oracle (ref_fp32.block_fwd)."""
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    grid = (21, 17, 22)
    spec, sd, x, e0, context = _config0_inputs(seed=4, L_grid=grid)
    cos, sin = R.rope_tables(R.model_freqs(128), grid, 128)
    p32 = fp32(sd)
    ck, cv = R.cross_kv(p32, context, spec.num_heads)
    y_ref = R.block_fwd(p32, x, e0, cos, sin, ck, cv, grid[0], spec.num_heads)
    w = BlockWeights(sd, spec.num_heads, DEV)
    ckd, cvd = FastCrossKV(w)(context.to(DEV, torch.bfloat16))
    cosd, sind = rope_tables(grid, 128, DEV)
    y = FastBlock(w, grid[0])(x.to(DEV, torch.bfloat16), e0.to(DEV), cosd, sind, ckd, cvd).float().cpu()
    err, upd = R.rel_rms(y, y_ref), R.rel_rms(y - x, y_ref - x)
    print(f"config2 block (L=7854) rel-RMS output {err:.2e}, update {upd:.2e}")
    assert err < BLOCK_TOL
    assert upd < 5e-2


def test_step_30_layers_full_width_vs_oracle():
    """A whole step-0 noise prediction of the TI2V-5B architecture (30 layers, dim 3072, 24 heads,
    ffn 14336, text dim 4096, seeded weights) at 1080 tokens (6x12x15 grid, latent [48, 6, 24, 30])
    against the fp32 CPU oracle chained over all 30 blocks (ref_fp32.main restated): the
    north-star's step-0 tolerance over the whole depth of the model."""
    from wanb200 import TI2V_5B, random_model_state
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    spec = TI2V_5B
    sd = random_model_state(spec, seed=11, device=DEV)
    g = torch.Generator().manual_seed(12)
    lat = torch.randn(48, 6, 24, 30, generator=g)
    ctx, ctx_null = torch.randn(512, 4096, generator=g), torch.randn(512, 4096, generator=g)
    fast = FastWanDiT((spec, sd), (6, 12, 15), 5.0, DEV)
    fast.set_context(ctx.to(DEV), ctx_null.to(DEV))
    pred = fast(lat.to(DEV), 999.0)
    assert pred.dtype == torch.bfloat16 and tuple(pred.shape) == (48, 6, 24, 30)
    assert fast.check_device_errors() == 0
    cfg = {"num_heads": 24, "num_layers": 30, "freq_dim": 256, "patch": (1, 2, 2), "out_dim": 48}
    with torch.no_grad():
        ref = R.step(sd, cfg, lat, 999.0, ctx, ctx_null, 5.0)
    err = R.rel_rms(pred.float().cpu(), ref)
    print(f"30-layer dim-3072 step-0 (L=1080) rel-RMS vs oracle {err:.3e}")
    assert err < STEP_TOL


def test_block_op_traces_under_torch_compile_fullgraph():
    """torch.ops.wanb200.block / cross_attn are custom ops with fake kernels: a step built from
    them compiles with fullgraph=True (no graph break) and gives the eager result."""
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    cfg = mg["cfg"]
    spec = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"], num_layers=cfg["num_layers"],
                   freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"], in_dim=cfg["in_dim"], out_dim=cfg["out_dim"],
                   text_len=cfg["text_len"])
    lat = mg["latent"]
    grid = (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2)
    fast = FastWanDiT((spec, mg["state_dict"]), grid, mg["guide"], DEV)
    fast.set_context(mg["ctx"].to(DEV), mg["ctx_null"].to(DEV))
    _, e0 = fast.time_embed(mg["t"])
    x = fast.patch(lat.to(DEV))
    eager = fast.forward_blocks(x, e0)
    torch._dynamo.reset()
    compiled = torch.compile(fast.forward_blocks_op, backend="eager", fullgraph=True)
    got = compiled(x, e0)
    assert torch.equal(got, eager)
    ck, cv = fast.context[0]
    q = torch.randn(2, 40, ck.shape[2], 128, device=DEV).to(torch.bfloat16)
    o = torch.compile(lambda a: torch.ops.wanb200.cross_attn(a, ck, cv, 128 ** -0.5), backend="eager",
                      fullgraph=True)(q)
    ref = R.attn(q.float(), ck.float(), cv.float())
    assert R.rel_rms(o.float(), ref) < 1e-2


def test_bounded_wait_expiry_reaches_the_step_driver():
    """A bounded wait that expires inside a kernel surfaces as WanB200Error from the product path.
    The expiry is made the safe way: a two-rank peer barrier run by one rank on this GPU alone
    waits for a flag that nothing sets, gives up after its 2 s deadline, records the code in the
    device error word and returns (no fault, no hang).  FastWanDiT then refuses to go on."""
    from wanb200 import ops
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    cfg = mg["cfg"]
    spec = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"], num_layers=cfg["num_layers"],
                   freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"], in_dim=cfg["in_dim"], out_dim=cfg["out_dim"],
                   text_len=cfg["text_len"])
    lat = mg["latent"].to(DEV)
    grid = (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2)
    fast = FastWanDiT((spec, mg["state_dict"]), grid, mg["guide"], DEV)
    fast.set_context(mg["ctx"].to(DEV), mg["ctx_null"].to(DEV))
    fast(lat, mg["t"])
    assert fast.check_device_errors() == 0
    dev = torch.device(DEV)

    def expire():  # rank 1 of the two never arrives: the wait gives up after 2 s
        flags = [torch.zeros(2, dtype=torch.int32, device=DEV) for _ in range(2)]
        ops.peer_barrier([f.data_ptr() for f in flags], 0, 1, dev)
        return flags

    keep = expire()
    with pytest.raises(L.WanB200Error, match="device error word 401"):
        fast.check_device_errors()
    with pytest.raises(L.WanB200Error, match="device error word 401"):
        fast(lat, mg["t"])  # a step refuses to run on top of a reported expiry
    assert L.device_error(reset=True) == 401
    assert fast.check_device_errors() == 0
    # without any synchronous check: a step queued behind the expiry posts the word, and the
    # next step reports it
    keep = expire()
    fast(lat, mg["t"])
    torch.cuda.synchronize()
    with pytest.raises(L.WanB200Error, match="device error word 401"):
        fast(lat, mg["t"])
    del keep
    assert L.device_error(reset=True) == 401
    assert fast.check_device_errors() == 0


def test_block_forward_c_entry_matches_the_python_block_op():
    """wanb200_block_forward (the whole block as one C call) against FastBlock.forward on the
    config-0 block: the same kernels in the same order, so they agree bit for bit; and against the
    fp32 oracle, with bf16 and fp32 residual streams."""
    from wanb200.block import block_forward_c
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    grid = (6, 12, 15)
    spec, sd, x, e0, context = _config0_inputs(seed=5, L_grid=grid)
    cos, sin = R.rope_tables(R.model_freqs(128), grid, 128)
    p32 = fp32(sd)
    ck, cv = R.cross_kv(p32, context, spec.num_heads)
    y_ref = R.block_fwd(p32, x, e0, cos, sin, ck, cv, grid[0], spec.num_heads)
    w = BlockWeights(sd, spec.num_heads, DEV)
    ckd, cvd = FastCrossKV(w)(context.to(DEV, torch.bfloat16))
    cosd, sind = rope_tables(grid, 128, DEV)
    blk = FastBlock(w, grid[0])
    xd = x.to(DEV, torch.bfloat16)
    y_py = blk(xd, e0.to(DEV), cosd, sind, ckd, cvd)
    y_c = block_forward_c(blk, xd, e0.to(DEV), cosd, sind, ckd, cvd)
    assert y_c.dtype == torch.bfloat16
    assert torch.equal(y_c, y_py), R.rel_rms(y_c.float(), y_py.float())
    assert R.rel_rms(y_c.float().cpu(), y_ref) < BLOCK_TOL
    y32 = block_forward_c(blk, x.to(DEV), e0.to(DEV), cosd, sind, ckd, cvd, out_dtype=torch.float32)
    assert y32.dtype == torch.float32
    assert R.rel_rms(y32.cpu(), y_ref) < R.rel_rms(y_c.float().cpu(), y_ref)  # no output rounding


def _golden_dit(mg, **kw):
    cfg = mg["cfg"]
    spec = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"], num_layers=cfg["num_layers"],
                   freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"], in_dim=cfg["in_dim"], out_dim=cfg["out_dim"],
                   text_len=cfg["text_len"])
    lat = mg["latent"]
    return FastWanDiT((spec, mg["state_dict"]), (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2), mg["guide"],
                      DEV, **kw)


def test_embeddings_and_head_on_the_kernels_vs_oracle():
    """The step driver's embeddings and head run on the library's kernels in bf16 (as the
    reference's `_time_embed` / `_FastPatch` / `_FastText` / `_FastHead` do): each against the fp32
    oracle (ref_fp32.py:77-98) on the golden model, and the head per token shard (the Q-local
    layouts' head, padded last shard included) against the whole-sequence head."""
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    fd = _golden_dit(mg)
    mp = fp32(mg["state_dict"])
    nf = fd.num_frames
    e, e0 = fd.time_embed(mg["t"])
    e_ref, e0_ref = R.time_embed(mp, mg["t"], nf, mg["cfg"]["freq_dim"])
    assert R.rel_rms(e.cpu(), e_ref[0]) < 1e-2 and R.rel_rms(e0.cpu(), e0_ref[0]) < 1e-2
    x = fd.patch(mg["latent"].to(DEV))
    x_ref = R.patch_embed(mp, mg["latent"].float())
    assert x.dtype == torch.float32 and R.rel_rms(x[0].cpu(), x_ref[0]) < 1e-2 and torch.equal(x[0], x[1])
    ctx = torch.stack([mg["ctx"], mg["ctx_null"]]).float()
    fd.set_context(mg["ctx"].to(DEV), mg["ctx_null"].to(DEV))
    ck0, _ = fd.context[0]
    ck_ref, _ = R.cross_kv(R.block_params(mp, 0), R.text_embed(mp, ctx), mg["cfg"]["num_heads"])
    assert R.rel_rms(ck0.float().cpu(), ck_ref) < 2e-2
    g = torch.Generator().manual_seed(5)
    L_, C = fd.seq_len, fd.spec.dim
    xs = torch.randn(2, L_, C, generator=g)
    es = torch.randn(nf, C, generator=g) * 0.1
    y_ref = R.head(mp, xs, es.unsqueeze(0), fd.grid)
    want = y_ref[1] + fd.guide_scale * (y_ref[0] - y_ref[1])
    whole = fd.head(xs.to(DEV), es.to(DEV))
    assert whole.dtype == torch.bfloat16 and R.rel_rms(whole.float().cpu(), want) < 1e-2
    tok = fd.head_tokens(xs.to(DEV), es.to(DEV))
    for sp in (2, 5):  # 5 shards of 5 leave the last one with 4 tokens + 1 pad row
        S = -(-L_ // sp)
        xp = torch.cat([xs, xs.new_zeros(2, sp * S - L_, C)], dim=1).to(DEV)
        parts = [fd.head_tokens(xp[:, r * S:(r + 1) * S].contiguous(), es.to(DEV), r * S) for r in range(sp)]
        got = torch.cat(parts, dim=1)[:, :L_]
        assert R.rel_rms(got.cpu(), tok.cpu()) < 1e-6, sp


def test_captured_step_replays_the_eager_step():
    """FastWanDiT.capture: the whole step as one CUDA graph gives the eager step's output bit for
    bit (the same kernels in the same order), follows new latents and timesteps through its static
    buffers (device or page-locked host latents), and refuses to run once set_context() replaced
    the cross K/V baked into the graph."""
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    fast = _golden_dit(mg)
    fast.set_context(mg["ctx"].to(DEV), mg["ctx_null"].to(DEV))
    lat = mg["latent"].to(DEV)
    lat2 = lat * 0.5 + 0.1
    want1 = fast(lat, mg["t"])
    want2 = fast(lat2, 500.0)
    assert not torch.equal(want1, want2)
    step = fast.capture(lat)
    assert torch.equal(step(lat, mg["t"]), want1)
    assert torch.equal(step(lat2.cpu().pin_memory(), 500.0), want2)
    assert torch.equal(step(lat, mg["t"]), want1)
    assert fast.check_device_errors() == 0 and step.check_device_errors() == 0
    # the denoise loop driven by the captured step: the eager loop's latent bit for bit
    from wanb200.unipc import denoise
    img = torch.randn(lat.shape[0], 1, lat.shape[2], lat.shape[3], generator=torch.Generator().manual_seed(9))
    assert torch.equal(denoise(step, lat, 3, 5.0, img.to(DEV)), denoise(fast, lat, 3, 5.0, img.to(DEV)))
    fast.set_context(mg["ctx"].to(DEV), mg["ctx_null"].to(DEV))
    with pytest.raises(RuntimeError, match="capture again"):
        step(lat, mg["t"])


def test_captured_step_full_width():
    """The captured step of the TI2V-5B architecture (dim 3072, 24 heads, 4 of its 30 layers, seeded
    weights) at 1080 tokens: the full-size kernel configurations (tile widths, key splits) under
    capture, bit-identical to the eager step for two timesteps."""
    from wanb200 import TI2V_5B, random_model_state
    spec = TI2V_5B
    sd = random_model_state(spec, seed=21, device=DEV, num_layers=4)
    g = torch.Generator().manual_seed(22)
    lat = torch.randn(48, 6, 24, 30, generator=g).to(DEV)
    ctx, ctx_null = torch.randn(512, 4096, generator=g), torch.randn(512, 4096, generator=g)
    fast = FastWanDiT((spec, sd), (6, 12, 15), 5.0, DEV, num_layers=4)
    fast.set_context(ctx.to(DEV), ctx_null.to(DEV))
    want = [fast(lat, t) for t in (999.0, 321.0)]
    step = fast.capture(lat)
    for t, w in zip((999.0, 321.0), want):
        got = step(lat, t)
        assert got.dtype == torch.bfloat16 and torch.equal(got, w), t
    assert fast.check_device_errors() == 0
