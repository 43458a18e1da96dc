"""Host-side logic of the step driver that runs without a GPU: the token-local head used by
the Q-local sequence-parallel layouts, and the layout table.

The head of `FastWanDiT` (LN + per-frame 2-way modulation + Linear, `_FastHead`,
models/fast_dit.py:480-505) is evaluated per token shard with a row offset and the shards are
concatenated as the SP all-gather would; the result must equal the oracle's head
(ref_fp32.py:90-98) on the whole sequence, padded last shard included.
"""
import os

import torch

from oracle import dit_ref as R
from wanb200 import FastWanDiT, WanSpec
from wanb200.parallel import KINDS, Layout

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bare_dit(mg, cfg_group=None):
    cfg = mg["cfg"]
    spec = WanSpec(dim=cfg["dim"], ffn_dim=cfg["ffn_dim"], num_heads=cfg["num_heads"], num_layers=cfg["num_layers"],
                   freq_dim=cfg["freq_dim"], text_dim=cfg["text_dim"], in_dim=cfg["in_dim"], out_dim=cfg["out_dim"],
                   text_len=cfg["text_len"])
    lat = mg["latent"]
    fd = FastWanDiT.__new__(FastWanDiT)  # only the attributes the head reads
    fd.spec = spec
    fd.grid = (lat.shape[1], lat.shape[2] // 2, lat.shape[3] // 2)
    fd.num_frames = fd.grid[0]
    fd.seq_len = fd.grid[0] * fd.grid[1] * fd.grid[2]
    fd.guide_scale = float(mg["guide"])
    fd.cfg_group, fd.pair_group = cfg_group, None
    fd.cfg_w = None
    fd.emb = {k: v.float() for k, v in mg["state_dict"].items() if not k.startswith("blocks.")}
    return fd


def test_sharded_head_matches_oracle_head():
    mg = torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)
    fd = _bare_dit(mg)
    L, C = fd.seq_len, fd.spec.dim
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, L, C, generator=g)
    e = torch.randn(1, fd.num_frames, C, generator=g) * 0.1
    y_ref = R.head(fd.emb, x, e, fd.grid)
    want = y_ref[1] + fd.guide_scale * (y_ref[0] - y_ref[1])
    whole = fd.head(x, e)
    # bf16 out, as _FastHead returns (fast_dit.py:503-505); fp32 math rounded once
    assert whole.dtype == torch.bfloat16
    assert R.rel_rms(whole, want) < 4e-3
    for sp in (2, 5):  # 24 tokens: 5 shards of 5 leave the last one with 4 tokens + 1 pad row
        S = -(-L // sp)
        xp = torch.cat([x, x.new_zeros(2, sp * S - L, C)], dim=1)
        parts = [fd.head_tokens(xp[:, r * S:(r + 1) * S], e, r * S) for r in range(sp)]
        tok = torch.cat(parts, dim=1)[:, :L]
        assert R.rel_rms(tok, fd.head_tokens(x, e)) < 1e-6, sp
        got = fd.combine(tok)
        assert got.dtype == torch.bfloat16 and R.rel_rms(got, want) < 4e-3, sp


def test_layout_kinds_and_names():
    assert KINDS == ("auto", "tp", "cfg", "sp", "cfgsp", "cfgsptp")
    assert Layout("single").describe(1) == "tp1"
    assert Layout("tp", tp_size=8).describe(8) == "tp8"
    assert Layout("cfg", cfg_group=0, tp_size=4).describe(8) == "cfg2x(sp+tp)4"
    assert Layout("cfg", cfg_group=0, tp_size=4).megatron_sp
    assert Layout("sp", sp_size=8).describe(8) == "sp8"
    assert Layout("cfgsp", cfg_group=1, sp_size=4).describe(8) == "cfg2xsp4"
    assert Layout("cfgsptp", cfg_group=0, tp_size=2, sp_size=2).describe(8) == "cfg2xsp2xtp2"


def test_kv_gather_packs_the_other_ranks_rows_contiguously():
    """The Q-local K/V push (wanb200.comm.KVGather): on rank p the shards of the other ranks are
    packed in the order p+1, p+2, ... so they tile rows [0, L - valid_p) exactly (the attention
    over the remote keys is one contiguous key range), padded last shards included."""
    from wanb200.comm import KVGather
    for T, L in ((2, 30), (4, 30), (4, 24), (8, 27280), (8, 7854), (3, 10)):
        g = KVGather.__new__(KVGather)  # the row arithmetic only (no process group)
        g.T = T
        S = -(-L // T)
        g.valid_all = [max(0, min(S, L - r * S)) for r in range(T)]
        assert sum(g.valid_all) == L
        for p in range(T):
            spans = sorted((g.chunk_row(p, r), g.chunk_row(p, r) + g.valid_all[r]) for r in range(T) if r != p)
            cursor = 0
            for a, b in spans:
                assert a == cursor, (T, L, p, spans)
                cursor = b
            assert cursor == L - g.valid_all[p]


def test_attention_custom_op_traces_without_a_device():
    """`torch.ops.wanb200.attn` (the reference's attention seam fn(q, k, v) -> o) has a fake kernel,
    so torch.compile / tracing can propagate shapes through it without running the kernel."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    from wanb200 import ops  # noqa: F401  (registers the op)
    with FakeTensorMode():
        q = torch.empty(2, 100, 3, 128, dtype=torch.bfloat16, device="meta")
        k = torch.empty(2, 77, 3, 128, dtype=torch.bfloat16, device="meta")
        o = torch.ops.wanb200.attn(q, k, k, 0.1)
    assert tuple(o.shape) == (2, 100, 3, 128) and o.dtype == torch.bfloat16
