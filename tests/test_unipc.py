"""The device-side sampler (wanb200.unipc.FlowUniPC) against the reference's own
`FlowUniPCMultistepScheduler` (wan/utils/fm_solvers_unipc.py), run by
tests/golden/make_golden.py exactly as inference_neuron_ti2v.py:497-532 runs it.

On the CPU the restatement must reproduce the reference bit for bit: the timesteps, the sigma
schedule and every step's sample, for fp32 and bf16 latents, shift 5 (the pipeline's), 3 and 1
(the linear schedule of the 27280-token workload), 50 (the pipeline's default), 25, 10, 3 and 2
(first-order only) steps.
"""
import os

import pytest
import torch

from wanb200.unipc import FlowUniPC, denoise

GOLD = os.path.join(os.path.dirname(__file__), "golden", "unipc_small.pt")


@pytest.fixture(scope="module")
def cases():
    return torch.load(GOLD, weights_only=False)["cases"]


def test_schedule_matches_reference(cases):
    for c in cases:
        s = FlowUniPC()
        s.set_timesteps(c["steps"], c["shift"])
        assert torch.equal(s.timesteps, c["timesteps"]), c["shift"]
        assert torch.equal(s.sigmas, c["sigmas"]), c["shift"]


def test_steps_match_reference_bit_for_bit(cases):
    for c in cases:
        s = FlowUniPC()
        s.set_timesteps(c["steps"], c["shift"])
        x = c["x_init"].clone()
        for i, (mo, want) in enumerate(zip(c["model_outputs"], c["outputs"])):
            x = s.step(mo, x)
            assert x.dtype == want.dtype
            assert torch.equal(x, want), (c["dtype"], c["shift"], c["steps"], i,
                                          float((x.float() - want.float()).abs().max()))


def test_step_past_the_schedule_raises(cases):
    c = cases[-1]
    s = FlowUniPC()
    s.set_timesteps(c["steps"], c["shift"])
    x = c["x_init"].clone()
    for mo in c["model_outputs"]:
        x = s.step(mo, x)
    with pytest.raises(RuntimeError):
        s.step(c["model_outputs"][0], x)


def test_denoise_loop_pins_the_image_frame():
    """The loop calls the model once per timestep with the current latent and keeps frame 0 at
    the image latent (the reference's mask2 blend)."""
    g = torch.Generator().manual_seed(3)
    lat = torch.randn(48, 3, 4, 6, generator=g)
    img = torch.randn(48, 1, 4, 6, generator=g)
    seen = []

    def model(latent, t):
        seen.append((float(t), latent[:, :1].clone()))
        return 0.5 * latent + 0.01 * t

    out = denoise(model, lat, steps=4, shift=5.0, image_latent=img)
    assert len(seen) == 4 and seen[0][0] > seen[-1][0]
    for _, f0 in seen:
        assert torch.equal(f0, img)
    assert torch.equal(out[:, :1], img)
    # same sequence through the sampler alone, frame 0 blended as the reference does
    s = FlowUniPC()
    s.set_timesteps(4, 5.0)
    x = lat.clone()
    x[:, :1] = img
    for t in s.timesteps:
        x = s.step(0.5 * x + 0.01 * float(t), x)
        x = torch.cat([img, x[:, 1:]], dim=1)
    assert torch.equal(out, x)
