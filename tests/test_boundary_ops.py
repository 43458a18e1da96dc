"""CPU checks of the Python boundary around the kernels (no GPU needed):

* the torch.library ops the reference's compiled units map to (`torch.ops.wanb200.block` for
  `_FastBlock.forward` / `_FastBlockSP.forward`, models/fast_dit.py:270, 349, compiled at 586;
  `torch.ops.wanb200.attn` / `cross_attn` for the attention seam, 186-255) have fake kernels, so a
  30-block step built from them traces into one graph without running a kernel;
* a device error word reported by the kernels stops the step driver (`FastWanDiT.__call__`,
  `check_device_errors`) and the denoise loop with WanB200Error, driven here by a fake probe.
"""
import pytest
import torch
from torch.fx.experimental.proxy_tensor import make_fx

from wanb200 import FastWanDiT, WanB200Error, denoise
from wanb200 import ops  # noqa: F401  (registers wanb200::attn / cross_attn)
from wanb200.block import block_op, register_block  # noqa: F401  (registers wanb200::block)


def _step(x, e, cos, sin, ck, cv, q):
    for h in range(1, 31):
        x = torch.ops.wanb200.block(x, e, cos, sin, ck, cv, h)
    y = torch.ops.wanb200.cross_attn(q, ck, cv, 0.088)
    return x * 2 + torch.ops.wanb200.attn(y, y, y, 0.088).sum()


def _inputs():
    return (torch.randn(2, 40, 256, dtype=torch.bfloat16), torch.randn(1, 2, 6, 256),
            torch.randn(1, 40, 1, 64), torch.randn(1, 40, 1, 64),
            torch.randn(2, 24, 2, 128, dtype=torch.bfloat16), torch.randn(2, 24, 2, 128, dtype=torch.bfloat16),
            torch.randn(2, 40, 2, 128, dtype=torch.bfloat16))


def test_thirty_block_step_traces_through_the_fake_kernels():
    gm = make_fx(_step, tracing_mode="fake")(*_inputs())
    targets = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert targets.count(torch.ops.wanb200.block.default) == 30
    assert targets.count(torch.ops.wanb200.cross_attn.default) == 1
    assert targets.count(torch.ops.wanb200.attn.default) == 1
    outs = [n for n in gm.graph.nodes if n.op == "output"]
    assert len(outs) == 1


def test_torch_export_of_a_block_stack_has_no_graph_break():
    class Stack(torch.nn.Module):
        def forward(self, x, e, cos, sin, ck, cv, q):
            return _step(x, e, cos, sin, ck, cv, q)

    ep = torch.export.export(Stack(), _inputs())
    names = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
    assert sum("wanb200.block" in t for t in names) == 30
    out = [n for n in ep.graph.nodes if n.op == "output"][0].args[0][0]
    assert tuple(out.meta["val"].shape) == (2, 40, 256)


def test_block_handles_are_weak():
    class Dummy:
        def forward(self, *a):
            return a[0]
    d = Dummy()
    h = register_block(d)
    from wanb200.block import _BLOCKS
    assert _BLOCKS[h] is d
    del d
    import gc
    gc.collect()
    assert h not in _BLOCKS


class FakeProbe:
    def __init__(self, code):
        self.code, self.posts = code, 0

    def poll(self):
        return self.code

    def post(self, stream=None):
        self.posts += 1

    def wait(self, stream=None):
        return self.code


def _bare(code):
    fd = FastWanDiT.__new__(FastWanDiT)
    fd.context = [None]
    fd._err_probe = FakeProbe(code)
    return fd


def test_step_driver_raises_on_a_reported_device_error():
    fd = _bare(401)
    with pytest.raises(WanB200Error, match="device error word 401"):
        fd(torch.zeros(48, 2, 4, 4), 999.0)  # raises before any kernel launch
    with pytest.raises(WanB200Error, match="device error word 401"):
        fd.check_device_errors()
    assert fd.check_device_errors(raise_error=False) == 401
    assert _bare(0).check_device_errors() == 0


def test_denoise_loop_ends_with_the_device_error_check():
    calls = []

    class Dit:
        def __call__(self, latent, t):
            calls.append(t)
            return torch.zeros_like(latent)

        def check_device_errors(self):
            raise WanB200Error("device error word 202")

    with pytest.raises(WanB200Error, match="202"):
        denoise(Dit(), torch.randn(4, 3, 2, 2), 2, 5.0)
    assert len(calls) == 2


def test_captured_step_refuses_the_multi_gpu_layouts():
    """FastWanDiT.capture is single-GPU only: the CFG-parallel, TP and SP layouts run NCCL
    collectives and peer barriers with host-side epochs that a graph replay would not advance."""
    from wanb200 import CapturedStep

    def bare(**kw):
        fd = FastWanDiT.__new__(FastWanDiT)
        fd.cfg_group, fd.pair_group, fd.tp_size, fd.sp, fd.kv_gather, fd.context = None, None, 1, False, None, None
        for k, v in kw.items():
            setattr(fd, k, v)
        return fd

    lat = torch.zeros(48, 2, 4, 4)
    for kw in ({"cfg_group": 0}, {"tp_size": 2}, {"sp": True}, {"kv_gather": object()}, {"pair_group": object()}):
        with pytest.raises(ValueError, match="single-GPU"):
            bare(context=[None], **kw).capture(lat)
    with pytest.raises(RuntimeError, match="set_context"):
        CapturedStep(bare(), lat)
    # a latent of another shape is refused (copy_ would broadcast it into the static buffer)
    step = CapturedStep.__new__(CapturedStep)
    step.model = _bare(0)
    step._ctx = step.model.context
    step.latent = torch.zeros(48, 2, 4, 4)
    with pytest.raises(ValueError, match="captured"):
        step(torch.zeros(48, 1, 4, 4), 999.0)
    # the denoise loop's closing check reaches the captured model's error word
    step.model = _bare(401)
    with pytest.raises(WanB200Error, match="device error word 401"):
        step.check_device_errors()
    assert step.check_device_errors(raise_error=False) == 401
