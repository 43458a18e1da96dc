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


class KVGather:
    """The gathered K/V of a sequence-parallel group (Q-local self-attention).

    `WanSelfAttentionSP` (models/dit_attention_sp.py:25-152) keeps each rank's L/SP query
    tokens local and all-gathers the normed, rotated K and V over the attn-sp group before the
    attention (88-99).  Here every rank holds the tokens rank*S .. rank*S + S - 1 of each batch
    element (S = ceil(L / SP); the last shard is zero-padded, `valid` rows are real).
      comm="peer" (overlapped): `start(kv)` pushes this rank's rows into the buffers of the other
        ranks over NVLink (wanb200_shard_gather) followed by a peer barrier, on a side stream, so
        the attention over this rank's own keys (read in place) runs meanwhile; `finish()` makes
        the current stream wait and returns [batch, remote_len, width]: the other ranks' rows,
        packed in the order rank+1, rank+2, ... (attention does not depend on the key order).
        Two buffers alternate by call, so a rank that runs ahead writes the buffer its slower
        peers finished reading one call ago (they passed the previous barrier after that read).
      comm="nccl": `gather(kv)` = torch.distributed.all_gather_into_tensor per batch element into
        [batch, SP*S, width]; rows 0 .. L-1 are the whole sequence.
    Every rank must make the same calls in the same order.
    """

    def __init__(self, group, batch: int, seq_len: int, width: int, device, comm: str = "peer"):
        self.group = group
        self.T = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.B, self.L, self.width = batch, seq_len, width
        self.S = -(-seq_len // self.T)
        self.valid_all = [max(0, min(self.S, seq_len - r * self.S)) for r in range(self.T)]
        self.valid = self.valid_all[self.rank]
        self.remote_len = seq_len - self.valid
        self.device = torch.device(device)
        self.comm = comm
        self.overlapped = comm == "peer"
        rows = self.T * self.S
        self.calls = 0
        if comm == "peer":
            import torch.distributed._symmetric_memory as symm_mem
            name = group.group_name
            try:
                symm_mem.enable_symm_mem_for_group(name)
            except Exception:
                pass
            self.bufs, self.ptrs, self._handles = [], [], []
            for _ in range(2):
                t = symm_mem.empty((batch, rows, width), dtype=BF16, device=self.device)
                h = symm_mem.rendezvous(t, name)
                off = t.data_ptr() - int(h.buffer_ptrs[self.rank])
                self.bufs.append(t)
                self.ptrs.append([int(p) + off for p in h.buffer_ptrs])
                self._handles.append(h)
            # destinations: the other ranks, starting with the next one so the ranks' first
            # stores go to different GPUs; each places this rank's rows after the chunks of the
            # ranks between them
            self.dst_ranks = [(self.rank + j) % self.T for j in range(1, self.T)]
            self.dst_rows = [self.chunk_row(p, self.rank) for p in self.dst_ranks]
            self.flags = symm_mem.empty((self.T,), dtype=torch.int32, device=self.device)
            hf = symm_mem.rendezvous(self.flags, name)
            foff = self.flags.data_ptr() - int(hf.buffer_ptrs[self.rank])
            self.flag_ptrs = [int(p) + foff for p in hf.buffer_ptrs]
            self._handles.append(hf)
            self.flags.zero_()
            self.epoch = 0
            self.side = torch.cuda.Stream(self.device)
            self._cur = None
        elif comm == "nccl":
            self.bufs = [torch.empty(batch, rows, width, dtype=BF16, device=self.device)]
            self.stage = torch.empty(batch, self.S, width, dtype=BF16, device=self.device)
        else:
            raise ValueError("comm must be 'peer' or 'nccl'")
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def chunk_row(self, p: int, r: int) -> int:
        """Row of rank r's shard in rank p's buffer: after the shards of p+1, p+2, ..., r-1."""
        row, j = 0, (p + 1) % self.T
        while j != r:
            row += self.valid_all[j]
            j = (j + 1) % self.T
        return row

    def start(self, kv: torch.Tensor):
        """kv: [batch * S, width] bf16 with unit column stride (this rank's shard, e.g. the k | v
        columns of the QKV buffer), complete on the current stream."""
        i = self.calls % 2
        self.calls += 1
        cur = torch.cuda.current_stream(self.device)
        self.side.wait_stream(cur)
        with torch.cuda.stream(self.side):
            ptrs = self.ptrs[i]
            ops.shard_gather(kv, self.B, self.S, self.valid, [ptrs[p] for p in self.dst_ranks], self.width,
                             self.T * self.S * self.width, self.dst_rows, self.device)
            self.epoch += 1
            ops.peer_barrier(self.flag_ptrs, self.rank, self.epoch, self.device)
        self._cur = (i, cur)

    def finish(self) -> torch.Tensor:
        i, cur = self._cur
        self._cur = None
        cur.wait_stream(self.side)
        return self.bufs[i][:, :self.remote_len]

    def gather(self, kv: torch.Tensor) -> torch.Tensor:
        """NCCL mode: the whole sequence's rows [batch, SP*S, width] (rows >= L are padding)."""
        self.calls += 1
        self.stage.view(self.B * self.S, self.width).copy_(kv[:self.B * self.S])
        out = self.bufs[0]
        for b in range(self.B):
            dist.all_gather_into_tensor(out[b], self.stage[b], group=self.group)
        return out
