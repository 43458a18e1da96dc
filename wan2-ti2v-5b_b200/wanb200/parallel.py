"""Process-group layouts for the DiT step over the GPUs of one node.

Mirrors the reference's group construction (inference_neuron_ti2v.py:241-274 for CFG-parallel,
models/parallel_state.py:64-96 for contiguous TP groups and strided attn-sp groups):
  * "tp":      one TP group of all ranks, batched CFG (batch 2) -- the benchmark's TP=N layout;
  * "cfg":     two CFG groups of N/2 contiguous ranks (group 0 = cond, group 1 = uncond, batch 1
               each), TP inside each group with the token-sharded residual (`_FastBlockSP`), and
               pair groups {i, i + N/2} for the head's CFG combine;
  * "sp":      Q-local sequence parallelism over all ranks (`WanSelfAttentionSP`), batched CFG,
               no TP: every rank runs the whole block on L/N tokens and gathers only K/V;
  * "cfgsp":   two CFG groups, Q-local SP over the N/2 ranks of each group;
  * "cfgsptp": two CFG groups of SP2 x TP(N/4) (config 3 at N=8: SP2 x TP2): TP groups of
               contiguous ranks, SP groups strided across them, as parallel_state.py builds
               its tp / attn-sp groups.
Every rank creates every group in the same order (torch.distributed requires it).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch.distributed as dist

KINDS = ("auto", "tp", "cfg", "sp", "cfgsp", "cfgsptp")


@dataclass
class Layout:
    name: str
    cfg_group: int | None = None
    pair_group: object = None
    tp_group: object = None
    tp_size: int = 1
    sp_group: object = None  # Q-local sequence-parallel group (K/V all-gather)
    sp_size: int = 1

    def describe(self, world: int) -> str:
        if self.name == "single":
            return "tp1"
        if self.name == "tp":
            return f"tp{world}"
        if self.name == "cfg":
            return "cfg2" if self.tp_size == 1 else f"cfg2x(sp+tp){self.tp_size}"
        if self.name == "sp":
            return f"sp{self.sp_size}"
        if self.name == "cfgsp":
            return "cfg2" if self.sp_size == 1 else f"cfg2xsp{self.sp_size}"
        return f"cfg2xsp{self.sp_size}xtp{self.tp_size}"

    @property
    def megatron_sp(self) -> bool:
        """The token-sharded residual with AG/RS around the TP GEMMs (`_FastBlockSP`)."""
        return self.name == "cfg" and self.tp_size > 1


def _cfg_split(world: int):
    if world % 2:
        raise ValueError(f"a CFG-parallel layout needs an even world size (got {world})")
    half = world // 2
    pair_groups = [dist.new_group([i, i + half]) for i in range(half)]
    return half, pair_groups


def make_layout(kind: str = "auto") -> Layout:
    """Build the groups for `kind` (one of KINDS; "auto": "cfgsp" when the world size is even --
    the fastest measured layout at 2, 4 and 8 B200s -- else "sp")."""
    if kind not in KINDS:
        raise ValueError(f"layout must be one of {KINDS}")
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return Layout("single")
    world, rank = dist.get_world_size(), dist.get_rank()
    if kind == "auto":
        kind = "cfgsp" if world % 2 == 0 else "sp"
    if kind == "tp":
        return Layout("tp", tp_group=dist.group.WORLD, tp_size=world)
    if kind == "sp":
        return Layout("sp", sp_group=dist.group.WORLD, sp_size=world)
    if kind == "cfg":
        half, pair_groups = _cfg_split(world)
        tp_groups = [dist.new_group(list(range(g * half, (g + 1) * half))) for g in range(2)]
        g = rank // half
        return Layout("cfg", cfg_group=g, pair_group=pair_groups[rank % half],
                      tp_group=tp_groups[g] if half > 1 else None, tp_size=half)
    if kind == "cfgsp":
        half, pair_groups = _cfg_split(world)
        sp_groups = [dist.new_group(list(range(g * half, (g + 1) * half))) for g in range(2)]
        g = rank // half
        return Layout("cfgsp", cfg_group=g, pair_group=pair_groups[rank % half],
                      sp_group=sp_groups[g] if half > 1 else None, sp_size=half)
    # cfgsptp: inside each CFG group of H = N/2 ranks, SP2 x TP(H/2)
    half, pair_groups = _cfg_split(world)
    if half % 2:
        raise ValueError(f"layout 'cfgsptp' needs the world size to be a multiple of 4 (got {world})")
    t = half // 2
    tp_groups, sp_groups = {}, {}
    for g in range(2):
        base = g * half
        for j in range(2):
            members = list(range(base + j * t, base + (j + 1) * t))
            grp = dist.new_group(members)
            for m in members:
                tp_groups[m] = grp
        for i in range(t):
            members = [base + i, base + t + i]
            grp = dist.new_group(members)
            for m in members:
                sp_groups[m] = grp
    return Layout("cfgsptp", cfg_group=rank // half, pair_group=pair_groups[rank % half],
                  tp_group=tp_groups[rank] if t > 1 else None, tp_size=t, sp_group=sp_groups[rank], sp_size=2)
