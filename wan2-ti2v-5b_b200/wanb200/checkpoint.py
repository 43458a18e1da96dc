"""The DiT weights of a Wan2.2 checkpoint directory, for `FastWanDiT((spec, state_dict), ...)`.

The reference loads its DiT with `WanModel.from_pretrained(MODEL_PATH)` (inference_neuron_ti2v.py:237;
`WanModel` is a diffusers `ModelMixin`, wan/modules/model.py:293-318): `config.json` holds the
constructor arguments (dim, ffn_dim, num_heads, num_layers, ...), the weights are
`diffusion_pytorch_model.safetensors`, or shards listed by
`diffusion_pytorch_model.safetensors.index.json` (`weight_map`: key -> shard file).  Parameter
names are the module paths of `WanModel` (`blocks.{i}.self_attn.q.weight`, ...).

`load_wan_checkpoint` reads exactly the tensors the fast path uses (the DiT: patch / text / time
embeddings, the blocks, the head), checks each against the shape the config implies, casts them
(bf16 by default, the reference casts the model to bf16 at inference_neuron_ti2v.py:287) and
returns `(WanSpec, state_dict)`; `BlockWeights` then fuses and slices them per rank.
`save_wan_checkpoint` writes the same layout (single file or shards), e.g. for tests or to store
a converted state dict.
"""
from __future__ import annotations

import json
import os

import torch

from .weights import WanSpec, model_shapes

WEIGHTS_NAME = "diffusion_pytorch_model.safetensors"
INDEX_NAME = WEIGHTS_NAME + ".index.json"


def spec_from_config(cfg: dict) -> WanSpec:
    """WanSpec from the WanModel constructor arguments stored in config.json."""
    need = ("dim", "ffn_dim", "num_heads", "num_layers", "freq_dim", "text_dim", "in_dim", "out_dim")
    missing = [k for k in need if k not in cfg]
    if missing:
        raise ValueError(f"config.json lacks {missing}")
    # the fast path implements the TI2V / T2V forward with full (global) attention; a config that
    # asks for something else must not load and silently run another model's math
    # (WanModel.__init__, wan/modules/model.py:304-317)
    window = tuple(int(x) for x in cfg.get("window_size", (-1, -1)))
    if window != (-1, -1):
        raise ValueError(f"window_size {window}: local-window attention is not implemented (only (-1, -1))")
    model_type = cfg.get("model_type", "t2v")
    if model_type not in ("t2v", "ti2v"):
        raise ValueError(f"model_type {model_type!r} is not implemented (only 't2v' / 'ti2v', the TI2V-5B DiT; "
                         "i2v adds image-embedding cross-attention)")
    for flag in ("qk_norm", "cross_attn_norm"):
        if not cfg.get(flag, True):
            raise ValueError(f"{flag}=False is not implemented (the TI2V-5B DiT has both norms)")
    return WanSpec(dim=int(cfg["dim"]), ffn_dim=int(cfg["ffn_dim"]), num_heads=int(cfg["num_heads"]),
                   num_layers=int(cfg["num_layers"]), freq_dim=int(cfg["freq_dim"]), text_dim=int(cfg["text_dim"]),
                   in_dim=int(cfg["in_dim"]), out_dim=int(cfg["out_dim"]),
                   patch_size=tuple(int(x) for x in cfg.get("patch_size", (1, 2, 2))),
                   text_len=int(cfg.get("text_len", 512)), eps=float(cfg.get("eps", 1e-6)))


def checkpoint_files(path: str) -> list:
    """The safetensors files of the checkpoint directory (the index's shards, or the single file)."""
    index = os.path.join(path, INDEX_NAME)
    if os.path.exists(index):
        with open(index) as f:
            shards = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, s) for s in shards]
    single = os.path.join(path, WEIGHTS_NAME)
    if os.path.exists(single):
        return [single]
    raise FileNotFoundError(f"{path} holds neither {INDEX_NAME} nor {WEIGHTS_NAME}")


def load_wan_checkpoint(path: str, dtype=torch.bfloat16, num_layers=None):
    """(WanSpec, state_dict) of the DiT in the checkpoint directory `path`.

    num_layers: read only blocks 0 .. num_layers-1 (a shortened model for tests / benches).
    Raises if a tensor the fast path needs is missing or has the wrong shape."""
    from safetensors import safe_open
    with open(os.path.join(path, "config.json")) as f:
        spec = spec_from_config(json.load(f))
    want = model_shapes(spec, num_layers)
    sd = {}
    for file in checkpoint_files(path):
        with safe_open(file, framework="pt", device="cpu") as r:
            for k in r.keys():
                if k in want:
                    t = r.get_tensor(k)
                    if tuple(t.shape) != tuple(want[k]):
                        raise ValueError(f"{k}: shape {tuple(t.shape)} in {os.path.basename(file)}, "
                                         f"the config implies {tuple(want[k])}")
                    sd[k] = t.to(dtype)
    missing = sorted(set(want) - set(sd))
    if missing:
        raise ValueError(f"{path} lacks {len(missing)} DiT tensors, e.g. {missing[:4]}")
    return spec, sd


def save_wan_checkpoint(path: str, spec: WanSpec, sd: dict, max_shard_bytes: int = 0, extra_config=None):
    """Write config.json and the weights in the layout load_wan_checkpoint (and from_pretrained)
    reads; max_shard_bytes > 0 splits them into shards with an index."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    cfg = {"_class_name": "WanModel", "model_type": "ti2v", "dim": spec.dim, "ffn_dim": spec.ffn_dim,
           "num_heads": spec.num_heads, "num_layers": spec.num_layers, "freq_dim": spec.freq_dim,
           "text_dim": spec.text_dim, "in_dim": spec.in_dim, "out_dim": spec.out_dim,
           "patch_size": list(spec.patch_size), "text_len": spec.text_len, "eps": spec.eps}
    cfg.update(extra_config or {})
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    tensors = {k: v.detach().contiguous().cpu() for k, v in sd.items()}
    if max_shard_bytes <= 0:
        save_file(tensors, os.path.join(path, WEIGHTS_NAME))
        return
    shards, cur, size = [], {}, 0
    for k in sorted(tensors):
        nb = tensors[k].numel() * tensors[k].element_size()
        if cur and size + nb > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = tensors[k]
        size += nb
    if cur:
        shards.append(cur)
    weight_map = {}
    for i, shard in enumerate(shards):
        name = f"diffusion_pytorch_model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(shard, os.path.join(path, name))
        weight_map.update({k: name for k in shard})
    total = sum(t.numel() * t.element_size() for t in tensors.values())
    with open(os.path.join(path, INDEX_NAME), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)
