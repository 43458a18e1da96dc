"""The CPU oracle (oracle/dit_ref.py) against fixtures produced by the reference itself.

The fixtures come from tests/golden/make_golden.py, which runs yahavb/wan2-ti2v-5b's own
`scripts/validate/ref_fp32.py` (main() and block_fwd) and `models/fast_dit.py` helpers.
"""
import os

import pytest
import torch

from oracle import dit_ref as R

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return torch.load(os.path.join(GOLD, name), weights_only=False)


@pytest.fixture(scope="module")
def model_gold():
    return load("model_small.pt")


def fp32(sd):
    return {k: v.float() for k, v in sd.items()}


def test_rope_tables_match_reference():
    g = load("rope_small.pt")
    assert torch.equal(R.model_freqs(128), g["freqs"])
    for grid, (c, s, rows) in g["tables"].items():
        c2, s2 = R.rope_tables(R.model_freqs(128), grid, 128)
        if rows is not None:
            c2, s2 = c2[:, rows], s2[:, rows]
        assert torch.equal(c2, c) and torch.equal(s2, s), grid


def test_rope_rotation_matches_reference():
    g = load("rope_small.pt")
    c, s = R.rope_tables(g["freqs"], (2, 3, 4), 128)
    torch.testing.assert_close(R.rope(g["x"], c, s), g["rope_x"], rtol=0, atol=1e-6)


def test_block_matches_reference_block_fwd(model_gold):
    g = load("block_small.pt")
    bp = R.block_params(fp32(model_gold["state_dict"]), 0)
    y = R.block_fwd(bp, g["x"], g["e0"], g["cos"], g["sin"], g["ck"], g["cv"], g["grid"][0], g["num_heads"])
    assert R.rel_rms(y, g["y"]) < 1e-6


def test_cross_kv_matches_reference(model_gold):
    g = load("block_small.pt")
    bp = R.block_params(fp32(model_gold["state_dict"]), 0)
    ck, cv = R.cross_kv(bp, g["context"], g["num_heads"])
    assert R.rel_rms(ck, g["ck"]) < 1e-6 and R.rel_rms(cv, g["cv"]) < 1e-6


def test_time_and_text_embedding_match_reference(model_gold):
    g = load("block_small.pt")
    mp = fp32(model_gold["state_dict"])
    e, e0 = R.time_embed(mp, model_gold["t"], g["grid"][0], model_gold["cfg"]["freq_dim"])
    assert R.rel_rms(e0, g["e0"]) < 1e-6 and R.rel_rms(e, g["e"]) < 1e-6
    ctx = R.text_embed(mp, torch.stack([model_gold["ctx"], model_gold["ctx_null"]], 0))
    assert R.rel_rms(ctx, g["context"]) < 1e-6


def test_step_matches_reference_main(model_gold):
    """Whole step-0 CFG noise prediction vs the reference's ref_fp32.main() output."""
    mg = model_gold
    pred = R.step(fp32(mg["state_dict"]), mg["cfg"], mg["latent"], mg["t"], mg["ctx"], mg["ctx_null"], mg["guide"])
    assert pred.shape == mg["noise_pred"].shape
    assert R.rel_rms(pred, mg["noise_pred"]) < 1e-6


def test_reference_bf16_calibration():
    """The reference's own bf16 block paths sit at bf16-level error vs its fp32 oracle.

    This records the error floor the device implementation is compared against (the
    tolerance for one block is rel-RMS <= 2e-2)."""
    g = load("block_small.pt")
    for key in ("y_wan_bf16", "y_fast_bf16"):
        err = R.rel_rms(g[key], g["y"])
        assert err < 2e-2, (key, err)
