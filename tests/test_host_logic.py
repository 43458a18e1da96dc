"""Host-side logic of the step driver that runs without a GPU: the layout table, the Q-local K/V
packing arithmetic, and the attention op's fake kernel.  (The head itself runs on the kernels; its
sharded evaluation against the oracle's head is a GPU test in tests/test_gpu_block.py.)
"""
import torch

from wanb200.parallel import KINDS, Layout


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
