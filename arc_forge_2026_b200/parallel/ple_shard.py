"""The PLE n-gram table split by rows over the ranks of a process group (the reference's row-sharded embedding,
``training/work/qwen38fn_lora/distributed_utils.py:65-97``: all-gather of ids, local lookup, reduce-scatter).

Two paths:

* peer memory (CUDA, world > 1): every rank's shard (and its block scales) sits in a symmetric heap; the native
  lookup (``csrc/ple.cu``) reads each row from its owner's HBM over NVLink with plain 16-byte loads. One kernel, no
  collective: the ids never leave the rank and only the rows it needs cross the link.
* collectives (CPU / gloo, or ``peer=False``): the reference's scheme — all-gather of every rank's n-gram ids, each
  rank fills the rows it owns (zeros elsewhere), a sum over ranks returns every rank its own rows (reduce-scatter
  on NCCL; all-reduce and a slice on gloo, which has no reduce-scatter).

Every rank holds ``rows_per_shard`` rows (a multiple of 128, so FP8 scale blocks never straddle shards); rank r
owns rows ``[r * rows_per_shard, (r + 1) * rows_per_shard)``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.ple import NgramHash
from ..quant.fp8 import dequant_weight_block, quantize_weight_block


def shard_rows(total_rows: int, world: int) -> int:
    per = -(-total_rows // world)
    return (per + 127) // 128 * 128


class ShardedPleTable:
    def __init__(self, hash_: NgramHash, weight_shard: torch.Tensor, rank: int, world: int, device, fp8: bool = True,
                 group=None, peer: bool | None = None):
        """``weight_shard``: this rank's rows [<= rows_per_shard, D] of the full table (the last shard may be short)."""
        self.hash, self.rank, self.world, self.group = hash_, rank, world, group
        self.device = torch.device(device)
        self.rows_per_shard = shard_rows(hash_.rows, world)
        self.D = weight_shard.shape[1]
        self.E = self.D * len(hash_.moduli)
        self.fp8 = fp8
        w = weight_shard.detach().float()
        if w.shape[0] < self.rows_per_shard:  # pad the short last shard
            w = torch.cat([w, w.new_zeros(self.rows_per_shard - w.shape[0], self.D)])
        if fp8:
            q, s = quantize_weight_block(w)
            self.rows, self.scale = q.to(self.device), s.to(self.device)
        else:
            self.rows, self.scale = w.to(self.device, torch.bfloat16), None
        self.peer = (self.device.type == "cuda" and world > 1) if peer is None else peer
        self.heap = self.table = None
        if self.peer:
            self._open_peer()

    # ------------------------------------------------------------------ peer-memory path
    def _open_peer(self):
        from ..ops import C
        from ..ops.ple import PleTable
        rows_b = self.rows.numel() * self.rows.element_size()
        rows_b = (rows_b + 255) // 256 * 256
        scale_b = self.scale.numel() * 4 if self.fp8 else 0
        ext = C()
        self.heap = ext.SymmHeap(rows_b + scale_b + 256, self.rank, self.world, self.device.index or 0)
        buf = self.heap.tensor()
        buf[: self.rows.numel() * self.rows.element_size()].copy_(self.rows.view(torch.uint8).reshape(-1))
        if self.fp8:
            buf[rows_b: rows_b + scale_b].copy_(self.scale.view(torch.uint8).reshape(-1))
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, self.heap.handle(), group=self.group)
            self.heap.open(handles)
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        shards = [(base, base + rows_b if self.fp8 else 0) for base in self.heap.peers()]
        self.table = PleTable(self.hash, self.rows, self.scale, shards=shards, rows_per_shard=self.rows_per_shard,
                              table_rows=self.hash.rows)

    # ------------------------------------------------------------------ lookups
    def _local_rows(self, ids: torch.Tensor) -> torch.Tensor:
        """Rows of ``ids`` [N, heads] this rank owns (dequantised, fp32), zeros for the others."""
        lo = self.rank * self.rows_per_shard
        local = ids - lo
        own = (local >= 0) & (local < self.rows_per_shard)
        dense = dequant_weight_block(self.rows, self.scale) if self.fp8 else self.rows.float()
        got = dense[local.clamp(0, self.rows_per_shard - 1)]
        return torch.where(own[..., None], got, torch.zeros_like(got))

    def lookup_tokens(self, tokens: torch.Tensor, seg_start: torch.Tensor | None = None) -> torch.Tensor:
        """[T, E] embeddings of this rank's tokens (bf16 on the peer path, fp32 on the collective path). Every rank
        of the group calls it (the collective path exchanges ids)."""
        if self.table is not None:
            return self.table.lookup_tokens(tokens.to(self.device), None if seg_start is None else
                                            seg_start.to(self.device))
        ids = self.hash.ids(tokens.reshape(-1).cpu(), None if seg_start is None else seg_start.cpu()).to(self.device)
        T, heads = ids.shape
        if self.world == 1:
            return self._local_rows(ids).flatten(-2)
        counts = [torch.zeros(1, dtype=torch.int64, device=self.device) for _ in range(self.world)]
        dist.all_gather(counts, torch.tensor([T], device=self.device), group=self.group)
        counts = [int(c) for c in counts]
        tmax = max(counts)
        pad = torch.full((tmax, heads), -1, dtype=ids.dtype, device=self.device)
        pad[:T] = ids
        every = [torch.empty_like(pad) for _ in range(self.world)]
        dist.all_gather(every, pad, group=self.group)
        contrib = self._local_rows(torch.cat(every)).flatten(-2)      # [world * tmax, E]
        if dist.get_backend(self.group) == "nccl":
            out = torch.empty(tmax, self.E, dtype=contrib.dtype, device=self.device)
            dist.reduce_scatter_tensor(out, contrib.contiguous(), group=self.group)
        else:
            dist.all_reduce(contrib, group=self.group)
            out = contrib[self.rank * tmax:(self.rank + 1) * tmax]
        return out[:T]

    def close(self):
        if self.heap is not None:
            torch.cuda.synchronize(self.device)
            self.heap.close()
            self.heap = None
            self.table = None
