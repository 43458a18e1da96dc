"""The checkpoint loader (wanb200.checkpoint) on the CPU.

The golden model's weights are the reference's own small `WanModel` (tests/golden/make_golden.py).
Written in the layout `WanModel.from_pretrained` reads (config.json with the constructor
arguments + diffusion_pytorch_model.safetensors, or shards with an index), they must load back
bit for bit, and the loaded weights must drive the oracle to the reference's own step-0 output.
"""
import json
import os

import pytest
import torch

from oracle import dit_ref as R
from wanb200.checkpoint import INDEX_NAME, WEIGHTS_NAME, load_wan_checkpoint, save_wan_checkpoint, spec_from_config

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def golden():
    return torch.load(os.path.join(GOLD, "model_small.pt"), weights_only=False)


def _reference_layout(path, mg):
    """config.json as WanModel's constructor arguments and one safetensors file of its
    state_dict, written independently of save_wan_checkpoint."""
    from safetensors.torch import save_file
    cfg = mg["cfg"]
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump({"_class_name": "WanModel", "model_type": "ti2v", "patch_size": list(cfg["patch"]),
                   "text_len": cfg["text_len"], "in_dim": cfg["in_dim"], "dim": cfg["dim"], "ffn_dim": cfg["ffn_dim"],
                   "freq_dim": cfg["freq_dim"], "text_dim": cfg["text_dim"], "out_dim": cfg["out_dim"],
                   "num_heads": cfg["num_heads"], "num_layers": cfg["num_layers"], "window_size": [-1, -1],
                   "qk_norm": True, "cross_attn_norm": True, "eps": 1e-6}, f)
    save_file({k: v.contiguous() for k, v in mg["state_dict"].items()}, os.path.join(path, WEIGHTS_NAME))


def test_load_reference_layout_bit_for_bit_and_reproduce_the_reference_step(golden, tmp_path):
    _reference_layout(str(tmp_path), golden)
    spec, sd = load_wan_checkpoint(str(tmp_path))
    cfg = golden["cfg"]
    assert (spec.dim, spec.num_heads, spec.num_layers, spec.in_dim, spec.text_len) == \
        (cfg["dim"], cfg["num_heads"], cfg["num_layers"], cfg["in_dim"], cfg["text_len"])
    assert set(sd) == set(golden["state_dict"])
    for k, v in golden["state_dict"].items():
        assert sd[k].dtype == torch.bfloat16 and torch.equal(sd[k], v), k
    mp = {k: v.float() for k, v in sd.items()}
    ocfg = {k: cfg[k] for k in ("num_heads", "num_layers", "freq_dim", "out_dim")}
    ocfg["patch"] = cfg["patch"]
    pred = R.step(mp, ocfg, golden["latent"].float(), golden["t"], golden["ctx"].float(), golden["ctx_null"].float(),
                  golden["guide"])
    assert R.rel_rms(pred, golden["noise_pred"]) < 1e-5


def test_sharded_round_trip_and_layer_subset(golden, tmp_path):
    spec, _ = load_wan_checkpoint(_write_single(tmp_path / "one", golden))
    save_wan_checkpoint(str(tmp_path / "sharded"), spec, golden["state_dict"], max_shard_bytes=200_000)
    index = json.load(open(tmp_path / "sharded" / INDEX_NAME))
    assert len(set(index["weight_map"].values())) > 2
    spec2, sd2 = load_wan_checkpoint(str(tmp_path / "sharded"))
    assert spec2 == spec
    for k, v in golden["state_dict"].items():
        assert torch.equal(sd2[k], v), k
    _, sd1 = load_wan_checkpoint(str(tmp_path / "sharded"), num_layers=1)
    assert not any(k.startswith("blocks.1.") for k in sd1) and "blocks.0.ffn.0.weight" in sd1
    _, sd32 = load_wan_checkpoint(str(tmp_path / "sharded"), dtype=torch.float32)
    assert sd32["head.head.weight"].dtype == torch.float32


def _write_single(path, golden):
    _reference_layout(str(path), golden)
    return str(path)


def test_missing_or_misshapen_tensors_are_refused(golden, tmp_path):
    spec, _ = load_wan_checkpoint(_write_single(tmp_path / "ok", golden))
    sd = dict(golden["state_dict"])
    del sd["blocks.1.cross_attn.norm_k.weight"]
    save_wan_checkpoint(str(tmp_path / "missing"), spec, sd)
    with pytest.raises(ValueError, match="lacks"):
        load_wan_checkpoint(str(tmp_path / "missing"))
    sd = dict(golden["state_dict"])
    sd["blocks.0.ffn.0.weight"] = sd["blocks.0.ffn.0.weight"][:-1]
    save_wan_checkpoint(str(tmp_path / "shape"), spec, sd)
    with pytest.raises(ValueError, match="blocks.0.ffn.0.weight"):
        load_wan_checkpoint(str(tmp_path / "shape"))
    with pytest.raises(FileNotFoundError):
        load_wan_checkpoint(str(tmp_path))
    with pytest.raises(ValueError, match="config.json lacks"):
        spec_from_config({"dim": 256})


def test_configs_of_other_model_variants_are_refused(golden, tmp_path):
    """A checkpoint whose config asks for math the fast path does not implement must not load
    (WanModel.__init__ arguments, wan/modules/model.py:304-317): local-window attention, the
    i2v / other model types, a model without the QK or cross-attention norms."""
    path = str(tmp_path / "ck")
    _reference_layout(path, golden)
    cfg_path = os.path.join(path, "config.json")
    base = json.load(open(cfg_path))
    spec_from_config(base)  # the TI2V-5B config loads
    spec_from_config(dict(base, model_type="t2v"))
    for change, match in (({"window_size": [256, 256]}, "window_size"), ({"model_type": "i2v"}, "model_type"),
                          ({"model_type": "s2v"}, "model_type"), ({"qk_norm": False}, "qk_norm"),
                          ({"cross_attn_norm": False}, "cross_attn_norm")):
        with pytest.raises(ValueError, match=match):
            spec_from_config(dict(base, **change))
        with open(cfg_path, "w") as f:
            json.dump(dict(base, **change), f)
        with pytest.raises(ValueError, match=match):
            load_wan_checkpoint(path)


def test_fast_dit_from_checkpoint_builds_the_fused_weights(golden, tmp_path):
    """FastWanDiT.from_checkpoint: the blocks' fused Q/K/V weight is the checkpoint's q, k, v
    stacked (construction only; the step itself runs in the GPU tests)."""
    from wanb200 import FastWanDiT
    path = _write_single(tmp_path / "ck", golden)
    fd = FastWanDiT.from_checkpoint(path, (2, 3, 4), golden["guide"], "cpu", num_layers=1)
    assert len(fd.blocks) == 1
    sd = golden["state_dict"]
    want = torch.cat([sd["blocks.0.self_attn.q.weight"], sd["blocks.0.self_attn.k.weight"],
                      sd["blocks.0.self_attn.v.weight"]])
    assert torch.equal(fd.block_weights[0].w_qkv.cpu(), want)
