"""Packed training bins: many sequences in one row of up to ``max_len`` tokens, so long-context training runs without
padding to the longest sequence (the reference's ``training/src/arcforge/train/packed_text.py:1-30`` best-fit-
decreasing bins and ``training/work/qwen38fn_lora/packed_qwen4.py:63-89`` packed forward).

Each sequence starts at a multiple of ``align`` tokens (64: one GDN chunk) and is followed by padding up to the next
multiple, so that:

* attention is causal inside each aligned segment (``cu_seqlens``; a segment's padding sees only its own tokens and
  is never trained);
* the chunked gated delta rule restarts its state at every segment (``chunk_reset``: one flag per 64-token chunk);
* the causal conv reads no history across a segment start (``pos``: each token's position inside its sequence);
* RoPE positions restart per sequence (``pos``).

Labels are the next token inside the sequence, -1 (not trained) at its last token, on its padding and where the
caller's loss mask is 0 (e.g. prompt tokens of an SFT pair).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class PackedBin:
    ids: torch.Tensor          # [L] int64
    labels: torch.Tensor       # [L] int64, -1 = not trained
    pos: torch.Tensor          # [L] int32 position inside the sequence (padding continues the count)
    cu_seqlens: torch.Tensor   # [S + 1] int32 segment starts (aligned) and the end
    chunk_reset: torch.Tensor  # [ceil(L / 64)] int32, 1 where a sequence starts
    seq_index: list[int]       # which input sequences the bin holds, in order

    @property
    def tokens(self) -> int:
        return int((self.labels >= 0).sum())

    def to(self, device):
        return PackedBin(self.ids.to(device), self.labels.to(device), self.pos.to(device),
                         self.cu_seqlens.to(device), self.chunk_reset.to(device), self.seq_index)

    def forward_args(self) -> dict:
        """Keyword arguments of ``QADStudent.hidden(ids[None], pack=...)``."""
        return {"pos": self.pos[None], "cu_seqlens": self.cu_seqlens, "chunk_reset": self.chunk_reset,
                "max_seqlen": int((self.cu_seqlens[1:] - self.cu_seqlens[:-1]).max())}


def _aligned(n: int, align: int) -> int:
    return (n + align - 1) // align * align


def best_fit_decreasing(lengths: list[int], capacity: int) -> list[list[int]]:
    """Bins of indices: longest first, each into the fullest bin that still fits (a new bin when none does)."""
    bins: list[list[int]] = []
    free: list[int] = []
    for i in sorted(range(len(lengths)), key=lambda j: (-lengths[j], j)):
        n = lengths[i]
        if n > capacity:
            raise ValueError(f"sequence {i} needs {n} tokens, more than the bin's {capacity}")
        best = -1
        for b, f in enumerate(free):
            if n <= f and (best < 0 or f < free[best]):
                best = b
        if best < 0:
            bins.append([i])
            free.append(capacity - n)
        else:
            bins[best].append(i)
            free[best] -= n
    return bins


def pack(seqs: list[list[int]], max_len: int, align: int = 64, loss_masks: list[list[int]] | None = None,
         pad_id: int = 0) -> list[PackedBin]:
    if align % 64 or max_len % align:
        raise ValueError("align must be a multiple of 64 (a GDN chunk) and max_len a multiple of align")
    lens = [_aligned(len(s), align) for s in seqs]
    out = []
    for idx in best_fit_decreasing(lens, max_len):
        ids, labels, pos, starts = [], [], [], []
        for i in idx:
            s = list(seqs[i])
            m = loss_masks[i] if loss_masks is not None else [1] * len(s)
            n, na = len(s), lens[i]
            starts.append(len(ids))
            ids += s + [pad_id] * (na - n)
            labels += [s[j + 1] if m[j + 1] else -1 for j in range(n - 1)] + [-1] * (na - n + 1)
            pos += list(range(na))
        L = len(ids)
        reset = torch.zeros((L + 63) // 64, dtype=torch.int32)
        for st in starts:
            reset[st // 64] = 1
        out.append(PackedBin(torch.tensor(ids, dtype=torch.long), torch.tensor(labels, dtype=torch.long),
                             torch.tensor(pos, dtype=torch.int32),
                             torch.tensor(starts + [L], dtype=torch.int32), reset, list(idx)))
    return out
