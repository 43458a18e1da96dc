"""Process-group layouts for the DiT step over the GPUs of one node.

Mirrors the reference's group construction (inference_neuron_ti2v.py:241-274 for CFG-parallel,
models/parallel_state.py:64-96 for contiguous TP groups):
  * "tp":  one TP group of all ranks, batched CFG (batch 2) — BASELINE config 2's TP=N;
  * "cfg": two CFG groups of N/2 contiguous ranks (group 0 = cond, group 1 = uncond, batch 1
    each), TP inside each group, and pair groups {i, i + N/2} for the head's CFG combine.
Every rank creates every group in the same order (torch.distributed requires it).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch.distributed as dist


@dataclass
class Layout:
    name: str
    cfg_group: int | None = None
    pair_group: object = None
    tp_group: object = None
    tp_size: int = 1

    def describe(self, world: int) -> str:
        if self.cfg_group is None:
            return f"tp{world}"
        return "cfg2" if self.tp_size == 1 else f"cfg2x(sp+tp){self.tp_size}"


def make_layout(kind: str = "auto") -> Layout:
    """Build the groups for `kind` in {"auto", "tp", "cfg"} ("auto": cfg when the world size is even)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return Layout("single")
    world, rank = dist.get_world_size(), dist.get_rank()
    if kind == "auto":
        kind = "cfg" if world % 2 == 0 else "tp"
    if kind == "tp":
        return Layout("tp", tp_group=dist.group.WORLD, tp_size=world)
    if kind != "cfg" or world % 2:
        raise ValueError(f"layout {kind!r} needs an even world size (got {world})")
    half = world // 2
    tp_groups = [dist.new_group(list(range(g * half, (g + 1) * half))) for g in range(2)]
    pair_groups = [dist.new_group([i, i + half]) for i in range(half)]
    g = rank // half
    return Layout("cfg", cfg_group=g, pair_group=pair_groups[rank % half],
                  tp_group=tp_groups[g] if half > 1 else None, tp_size=half)
