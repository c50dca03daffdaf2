"""PLE n-gram table on the device and its native lookup (``csrc/ple.cu``: hash, gather and dequantisation in one
kernel; the reference's table lookups ``training/work/qwen38fn_lora/ple_packed.py:48-62``, ``fp8_base.py``).

The table is block FP8 (e4m3 rows, one fp32 scale per 128 x 128 block, the layout of the reference's FP8
checkpoints) or bf16. At the real size (16 heads x ~20M buckets x 160 dims) the e4m3 table is ~51 GB: it is kept in
HBM (180 GB per GPU) rather than in host RAM. It may be split by rows over ranks (``parallel/ple_shard.py``): the
kernel then reads each row from its owner's memory over NVLink. A hot table (``models/ple.py`` ``build_hot``) keeps
only the most used buckets of every head; a miss reads zeros.
"""
from __future__ import annotations

import numpy as np
import torch

from ..models.ple import NgramHash, hot_rows
from ..quant.fp8 import dequant_weight_block, quantize_weight_block
from . import C


def _round128(n: int) -> int:
    return (n + 127) // 128 * 128


class PleTable:
    def __init__(self, hash_: NgramHash, rows: torch.Tensor, scale: torch.Tensor | None, hot=None,
                 shards: list[tuple[int, int]] | None = None, rows_per_shard: int | None = None,
                 table_rows: int | None = None):
        """``rows`` [R, D] e4m3 (with ``scale`` [ceil(R/128), ceil(D/128)] fp32) or bf16: this process's rows.
        ``shards``: (row pointer, scale pointer) of every shard in row order when the table is split over ranks
        (``rows`` is then this rank's shard); ``hot``: per head the sorted kept buckets (a compact table)."""
        self.hash = hash_
        self.rows, self.scale = rows, scale
        self.fp8 = rows.dtype == torch.float8_e4m3fn
        if not self.fp8 and rows.dtype != torch.bfloat16:
            raise TypeError("PLE table rows are e4m3 (with block scales) or bf16")
        self.D = rows.shape[1]
        self.E = self.D * len(hash_.moduli)
        dev = rows.device
        self.mult, self.mod, self.off = hash_.tensors(dev)
        self.hot = hot
        if hot is not None:
            lens = [len(hot[h]) for h in range(len(hash_.moduli))]
            base = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
            self.hot_idx = torch.as_tensor(np.concatenate([hot[h] for h in range(len(lens))]).astype(np.int64),
                                           device=dev)
            self.hot_base = torch.as_tensor(base, device=dev)
            self.hot_len = torch.as_tensor(np.array(lens, dtype=np.int32), device=dev)
            total = int(sum(lens))
        else:
            self.hot_idx = self.hot_base = self.hot_len = None
            total = hash_.rows
        self.table_rows = total if table_rows is None else table_rows
        if shards is None:
            shards = [(rows.data_ptr(), scale.data_ptr() if self.fp8 else 0)]
            rows_per_shard = _round128(max(self.table_rows, 1))
        self.shards, self.rows_per_shard = shards, rows_per_shard

    @classmethod
    def from_weight(cls, hash_: NgramHash, weight: torch.Tensor, device, fp8: bool = True, hot=None) -> "PleTable":
        """From a full table ``weight`` [hash.rows, D] (any float dtype); ``hot`` keeps only those buckets."""
        w = weight.detach()
        if hot is not None:
            idx = np.concatenate([np.asarray(hot[h], dtype=np.int64) + hash_.offsets[h]
                                  for h in range(len(hash_.moduli))])
            w = w[torch.as_tensor(idx, device=w.device)]
        if fp8:
            q, s = quantize_weight_block(w.float())
            return cls(hash_, q.to(device), s.to(device), hot)
        return cls(hash_, w.to(device, torch.bfloat16).contiguous(), None, hot)

    def dense_rows(self) -> torch.Tensor:
        """This process's rows dequantised (fp32): the oracle of the native lookup."""
        return dequant_weight_block(self.rows, self.scale) if self.fp8 else self.rows.float()

    def lookup(self, ext: torch.Tensor, pos: torch.Tensor, seg: torch.Tensor, ids_out=None) -> torch.Tensor:
        """Embeddings [R, E] bf16 of rows ``pos`` of ``ext`` (tokens with history inline, int32) whose segments start
        at ``seg``."""
        out = torch.empty(pos.numel(), self.E, dtype=torch.bfloat16, device=ext.device)
        C().ple_lookup(ext.int().contiguous(), pos.long().contiguous(), seg.long().contiguous(), self.hash.n,
                       self.hash.hpn, self.hash.eos, self.mult, self.mod, self.off, [p for p, _ in self.shards],
                       [s for _, s in self.shards] if self.fp8 else [], self.fp8, self.D, self.rows_per_shard,
                       self.table_rows, out, ids_out, self.hot_idx, self.hot_base, self.hot_len)
        return out

    def lookup_tokens(self, tokens: torch.Tensor, seg_start: torch.Tensor | None = None) -> torch.Tensor:
        """One sequence or packed row ``tokens`` [T] (segment starts ``seg_start`` [T]) -> [T, E]."""
        T = tokens.numel()
        pos = torch.arange(T, device=tokens.device)
        seg = torch.zeros_like(pos) if seg_start is None else seg_start.long()
        return self.lookup(tokens.reshape(-1), pos, seg)

    def lookup_reference(self, tokens: torch.Tensor, seg_start: torch.Tensor | None = None) -> torch.Tensor:
        """The same in torch on one (unsharded) table: hash, hot remap, gather of the dequantised rows."""
        ids = self.hash.ids(tokens.reshape(-1).cpu(), None if seg_start is None else seg_start.cpu())
        if self.hot is not None:
            ids = hot_rows(self.hash, self.hot, ids)
        dense = self.dense_rows().cpu()
        dense = torch.cat([dense, torch.zeros(1, self.D)])           # row -1 -> zeros
        return dense[torch.where(ids < 0, torch.full_like(ids, dense.shape[0] - 1), ids)].flatten(-2)
