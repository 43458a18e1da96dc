"""Peer-memory buffers of one TP group for the fused collectives of the sequence-parallel block.

Instead of NCCL all-gather / reduce-scatter around the TP GEMMs (the reference's `_ag` / `_rs`,
models/fast_dit.py:112-123), the kernels move the data themselves over NVLink:
  * all-gather: the LayerNorm writes each normalised row of this rank's shard into the gathered
    buffer `hf` of every rank of the group (rows rank*S..);
  * reduce-scatter: the row-parallel GEMM's epilogue stores row r of its partial sum into the
    inbox of the rank that owns r, in the slice of this source rank; the owner sums the slices
    in its bias + gate + residual kernel;
  * `barrier()` (wanb200_peer_barrier) separates those producers from the consumers.
The buffers are symmetric (same offset on every rank) allocations from torch's symmetric memory
(CUDA backend); only their raw peer pointers reach the kernels.  Every rank must make the same
calls in the same order (the barrier epochs are counted on the host).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops

BF16 = torch.bfloat16


class PeerComm:
    def __init__(self, group, shard_rows: int, dim: int, device):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group
        self.T = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.S, self.C = shard_rows, dim
        self.device = torch.device(device)
        name = group.group_name
        try:
            symm_mem.enable_symm_mem_for_group(name)
        except Exception:
            pass
        Np = self.T * shard_rows

        def sym(shape, dtype):
            t = symm_mem.empty(shape, dtype=dtype, device=self.device)
            h = symm_mem.rendezvous(t, name)
            base = int(h.buffer_ptrs[self.rank])
            off = t.data_ptr() - base
            return t, [int(p) + off for p in h.buffer_ptrs], h

        self.hf, self.hf_ptrs, self._h1 = sym((Np, dim), BF16)        # gathered LN output
        self.inbox, self.inbox_ptrs, self._h2 = sym((Np, dim), BF16)  # T slices of S partial rows
        self.flags, self.flag_ptrs, self._h3 = sym((self.T,), torch.int32)
        self.flags.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        self.epoch = 0

    def barrier(self):
        """All ranks of the group have finished every kernel issued before this call."""
        self.epoch += 1
        ops.peer_barrier(self.flag_ptrs, self.rank, self.epoch, self.device)

    @property
    def push(self):
        """`push=` argument of the LayerNorm ops: this rank's rows land at rank*S in every hf."""
        return (self.hf_ptrs, self.rank * self.S)

    @property
    def scatter(self):
        """`scatter=` argument of ops.linear for the row-parallel GEMMs."""
        return (self.inbox_ptrs, self.rank, self.S)
