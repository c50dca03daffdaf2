"""PLE n-gram table on the device and its native lookup (``csrc/ple.cu``: hash, gather and dequantisation in one
kernel; the reference's table lookups ``training/work/qwen38fn_lora/ple_packed.py:48-62``, ``fp8_base.py``).

The table is block FP8 (e4m3 rows, one fp32 scale per 128 x 128 block, the layout of the reference's FP8
checkpoints) or bf16. At the real size (16 heads x ~20M buckets x 160 dims) the e4m3 table is ~51 GB: it is kept in
HBM (180 GB per GPU) rather than in host RAM. It may be split by rows over ranks (``parallel/ple_shard.py``): the
kernel then reads each row from its owner's memory over NVLink. A hot table (``models/ple.py`` ``build_hot``) keeps
only the most used buckets of every head; a miss reads zeros.
"""
from __future__ import annotations

import math

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


# ---------------------------------------------------------------------------------------------- serving
def _group_rms(x: torch.Tensor, w: torch.Tensor, G: int, eps: float) -> torch.Tensor:
    z = x.float().unflatten(-1, (G, -1))
    z = z * torch.rsqrt(z.square().mean(-1, keepdim=True) + eps)
    return z.flatten(-2) * (1.0 + w)


class PleServeWeights:
    """One PLE layer in the serving layout: the device table, bf16 projections for the tcgen05 GEMM, fp32 norms and
    conv taps."""

    def __init__(self, table: PleTable, key_proj, value_proj, norm_key, norm_query, norm_conv, conv, G: int, H: int,
                 eps: float, dil: int):
        bf = torch.bfloat16
        self.table = table
        self.key_proj, self.value_proj = key_proj.to(bf).contiguous(), value_proj.to(bf).contiguous()
        self.norm_key, self.norm_query, self.norm_conv = (t.float().contiguous() for t in (norm_key, norm_query,
                                                                                           norm_conv))
        self.conv = conv.float().contiguous()
        self.G, self.H, self.eps, self.dil = G, H, eps, dil
        self.k = conv.shape[1]
        self.pad = (self.k - 1) * dil

    @classmethod
    def from_module(cls, mod, device, fp8: bool = True) -> "PleServeWeights":
        """From a ``models.ple.PLELayer``."""
        dev = torch.device(device)
        t = PleTable.from_weight(mod.hash, mod.table, dev, fp8=fp8)
        return cls(t, mod.key_proj.detach().to(dev), mod.value_proj.detach().to(dev), mod.norm_key.detach().to(dev),
                   mod.norm_query.detach().to(dev), mod.norm_conv.detach().to(dev), mod.conv.detach().to(dev),
                   mod.G, mod.H, mod.eps, mod.dil)


class PleServeState:
    """Per slot: the last n-1 committed tokens (right-aligned, ``hist_len`` valid), the last (k-1)·dil committed conv
    inputs, and the pending tokens / conv inputs of the last verify window (double-buffered by parity) that the next
    cycle commits up to its accepted count — the deferred commit the GDN verify uses, applied to the PLE side state
    (the reference's serving patch 0016 commits this state after verification)."""

    def __init__(self, w: PleServeWeights, slots: int, max_q: int, device):
        dev = torch.device(device)
        n1 = w.table.hash.n - 1
        C = w.G * w.H
        self.n1, self.max_q = n1, max_q
        self.hist = torch.zeros(slots, n1, dtype=torch.int64, device=dev)
        self.hist_len = torch.zeros(slots, dtype=torch.int64, device=dev)
        self.conv = torch.zeros(slots, w.pad, C, dtype=torch.float32, device=dev)
        self.ptok = torch.zeros(2, slots, max_q, dtype=torch.int64, device=dev)
        self.pconv = torch.zeros(2, slots, max_q, C, dtype=torch.float32, device=dev)

    def reset(self, slot: int):
        for t in (self.hist, self.hist_len, self.conv):
            t[slot].zero_()


def ple_serve(stream: torch.Tensor, tokens: torch.Tensor, w: PleServeWeights, st: PleServeState, seq_slot,
              n_commit, q_per_seq: int, parity: int, commit_current: bool):
    """Add the PLE update to ``stream`` [N, G, H] (bf16, in place) for a step of S = N / q_per_seq sequences of
    ``q_per_seq`` rows. Device-side only (fixed shapes): CUDA-graph capturable."""
    from . import C as _C
    S, W = seq_slot.numel(), q_per_seq
    N = S * W
    n1, pad = st.n1, w.pad
    slots = seq_slot.long()
    dev = stream.device
    if not commit_current:  # commit the previous window's accepted rows
        prev = parity ^ 1
        nc = n_commit.long()[slots]                                                     # [S]
        ext_t = torch.cat([st.hist[slots], st.ptok[prev, slots]], 1)                   # [S, n1 + max_q]
        st.hist[slots] = torch.gather(ext_t, 1, nc[:, None] + torch.arange(n1, device=dev))
        st.hist_len[slots] = torch.clamp(st.hist_len[slots] + nc, max=n1)
        if pad:
            ext_c = torch.cat([st.conv[slots], st.pconv[prev, slots]], 1)             # [S, pad + max_q, C]
            idx = (nc[:, None] + torch.arange(pad, device=dev))[..., None].expand(S, pad, ext_c.shape[2])
            st.conv[slots] = torch.gather(ext_c, 1, idx)
    hl = st.hist_len[slots]
    toks = tokens.view(S, W).long()
    ext = torch.cat([st.hist[slots], toks], 1)                                           # [S, n1 + W]
    base = torch.arange(S, device=dev)[:, None] * (n1 + W)
    pos = (base + n1 + torch.arange(W, device=dev)[None]).reshape(-1)
    seg = (base + n1 - hl[:, None]).expand(S, W).reshape(-1)
    e = w.table.lookup(ext.reshape(-1).int(), pos, seg)                                  # [N, E] bf16
    c = _C()
    G, H = w.G, w.H
    k = _group_rms(c.gemm(e, w.key_proj), w.norm_key, G, w.eps).view(N, G, H)
    q = _group_rms(stream.reshape(N, G * H), w.norm_query, G, w.eps).view(N, G, H)
    g = (k * q).sum(-1, keepdim=True) / math.sqrt(H)
    g = g.abs().clamp_min(1e-6).sqrt() * g.sign()
    v = torch.sigmoid(g) * c.gemm(e, w.value_proj).float()[:, None, :]                 # [N, G, H]
    cin = _group_rms(v.reshape(N, G * H), w.norm_conv, G, w.eps).view(S, W, G * H)
    ext_c = torch.cat([st.conv[slots], cin], 1) if pad else cin                        # [S, pad + W, C]
    out = torch.zeros_like(cin)
    for j in range(w.k):
        back = (w.k - 1 - j) * w.dil
        out += ext_c[:, pad - back: pad - back + W] * w.conv[:, j]
    stream += (v + out.view(N, G, H)).to(stream.dtype)
    if commit_current:  # prefill: every row is final
        both = torch.cat([st.hist[slots], toks], 1)
        st.hist[slots] = both[:, -n1:]
        st.hist_len[slots] = torch.clamp(hl + W, max=n1)
        if pad:
            st.conv[slots] = ext_c[:, -pad:]
    else:
        st.ptok[parity, slots, :W] = toks
        st.pconv[parity, slots, :W] = cin
