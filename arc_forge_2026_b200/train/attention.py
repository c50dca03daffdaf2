"""Native variable-length causal attention for training (``csrc/attention_train.cu``): forward, dQ and dK / dV on
tcgen05 with TMEM accumulators, deterministic (no atomics), in place of a library flash-attention.

The packed-row contract is flash-attention's varlen one (the reference trains its packed bins through
``flash_attn_varlen_func``, ``training/work/qwen38fn_lora/packed_qwen4.py:89-289``): ``q [T, Hq, D]``,
``k / v [T, Hkv, D]``, ``cu_seqlens`` the segment offsets; each query attends to the keys of its own segment at or
before its position, softmax scale ``1 / sqrt(D)``. D is 128 or 256; Hq a multiple of Hkv (GQA).
"""
from __future__ import annotations

import math

import torch

from ..ops import C

TILE = 64


def tile_lists(cu: list[int], device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(segment, first position) of the tiles of each kernel: the forward's 128-query tiles and dQ's 64-query tiles
    (longest causal prefix first), the dK / dV kernels' 128-key tiles (most query rows after the key tile first)."""
    def tiles(step):
        return [(s, p, cu[s + 1] - cu[s]) for s in range(len(cu) - 1) for p in range(0, cu[s + 1] - cu[s], step)]
    mk = lambda ts: torch.tensor([[s, p] for s, p, _ in ts], dtype=torch.int32).reshape(-1, 2).to(device)  # noqa: E731
    t128 = tiles(2 * TILE)
    return (mk(sorted(t128, key=lambda t: -t[1])), mk(sorted(tiles(TILE), key=lambda t: -t[1])),
            mk(sorted(t128, key=lambda t: -(t[2] - t[1]))))


class VarlenCausalAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, blkmap=None, qsa_block=64):
        cu_host = [int(x) for x in cu_seqlens.tolist()]
        cu = torch.tensor(cu_host, dtype=torch.int32, device=q.device)
        fwd_tiles, q_tiles, kv_tiles = tile_lists(cu_host, q.device)
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        T, Hq, D = q.shape
        out = torch.empty_like(q)
        lse = torch.empty(Hq, T, dtype=torch.float32, device=q.device)
        scale = 1.0 / math.sqrt(D)
        C().attn_train_fwd(q, k, v, cu, fwd_tiles, scale, out, lse, blkmap, qsa_block)
        ctx.save_for_backward(q, k, v, out, lse, cu, q_tiles, kv_tiles, blkmap)
        ctx.scale, ctx.qsa_block = scale, qsa_block
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, cu, q_tiles, kv_tiles, blkmap = ctx.saved_tensors
        dout = dout.contiguous().to(torch.bfloat16)
        delta = torch.empty_like(lse)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        # per-query-head fp32 dK / dV contributions (every row written; the reduce sums each KV group's heads in a
        # fixed order)
        dk_part = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        dv_part = torch.empty_like(dk_part)
        C().attn_train_bwd(q, k, v, cu, q_tiles, kv_tiles, ctx.scale, out, lse, dout, delta, dq, dk, dv, dk_part,
                           dv_part, blkmap, ctx.qsa_block)
        return dq, dk, dv, None, None, None


def varlen_attention(q, k, v, cu_seqlens, blkmap=None, qsa_block: int = 64) -> torch.Tensor:
    """Causal attention inside each segment of a packed row (bf16, CUDA): q [T, Hq, D], k / v [T, Hkv, D].
    ``blkmap`` (int32 [T, words], :func:`qsa_select_packed`): QSA, each row sees only its selected blocks of
    ``qsa_block`` tokens (and, as always, no future key)."""
    return VarlenCausalAttention.apply(q, k, v, cu_seqlens, blkmap, qsa_block)


def qsa_select_packed(idx_q, raw, k_norm, cos_t, sin_t, rot: int, eps: float, cu_seqlens, block: int, topk: int,
                      rows_per_set: int = 8) -> torch.Tensor:
    """QSA block selection of every position of a packed row, on the serving kernels (``csrc/qsa.cu``): idx_q
    [T, Hi, 128] (normed, rotated index queries), raw [T, 128] (raw index keys) -> int32 bitmap [T, words], bit b of
    row t = position t attends to block b of its segment (all complete blocks while there are <= topk of them,
    else the top-k by score; plus its own incomplete block). The reference selects the same set per query
    (``training/work/qwen38fn_lora/sparse_qsa.py:83-153``; grouped like ``qsa_union.py:316``).

    Each segment is laid out on its own 64-token pages (the raw keys copied page-aligned), its pooled keys are
    finalised, and its positions are cut into sets of ``rows_per_set`` consecutive rows that go through the
    tensor-core scores, the radix top-K and the per-set union like verify rows of one session; a last kernel
    spreads each set's union over its rows' bitmaps."""
    from ..ops.qsa import PAGE, QsaWorkspace
    dev = idx_q.device
    cu = [int(x) for x in cu_seqlens.tolist()]
    lens = [b - a for a, b in zip(cu[:-1], cu[1:])]
    nseg, W, Hi = len(lens), rows_per_set, idx_q.shape[1]
    pages = [(L + W + PAGE - 1) // PAGE for L in lens]  # + a set's padding rows past the segment end
    maxp = max(pages)
    pg0 = [0]
    for p in pages[:-1]:
        pg0.append(pg0[-1] + p)
    P = pg0[-1] + pages[-1]
    raw_pad = torch.zeros(P * PAGE, raw.shape[1], dtype=raw.dtype, device=dev)
    bt = torch.zeros(nseg, maxp, dtype=torch.int32)
    for s in range(nseg):
        raw_pad[pg0[s] * PAGE:pg0[s] * PAGE + lens[s]] = raw[cu[s]:cu[s + 1]]
        bt[s, :pages[s]] = torch.arange(pg0[s], pg0[s] + pages[s], dtype=torch.int32)
        bt[s, pages[s]:] = pg0[s]
    bt = bt.to(dev)
    nb = maxp * (PAGE // block)
    keys = torch.zeros(nseg * nb, raw.shape[1], dtype=raw.dtype, device=dev)
    fin = torch.zeros(nseg, dtype=torch.int32, device=dev)
    ctx = torch.tensor(lens, dtype=torch.int32, device=dev)
    C().qsa_finalize([raw_pad], [keys], [k_norm], bt, fin, ctx, cos_t, sin_t, rot, eps, block)
    # row sets: W consecutive positions of one segment (the last one padded past the segment end)
    seg_of, row0, nrows, ends = [], [], [], []
    for s in range(nseg):
        for p0 in range(0, lens[s], W):
            seg_of.append(s)
            row0.append(cu[s] + p0)
            nrows.append(min(W, lens[s] - p0))
            ends.append(p0 + W)
    S = len(seg_of)
    ws = QsaWorkspace(S, W, topk, maxp, Hi, dev, block=block)
    src = torch.tensor([r0 + r if r < n else -1 for r0, n in zip(row0, nrows) for r in range(W)], device=dev)
    ok = src >= 0
    ws.idx_q[:S * W][ok] = idx_q[src[ok]]
    i32 = dict(dtype=torch.int32, device=dev)
    C().qsa_select(ws.idx_q, keys, raw_pad, k_norm, bt, fin, torch.tensor(ends, **i32), W, topk, Hi, block, ws.sel,
                   cos_t, sin_t, rot, eps, ws.u_page, ws.u_lpage, ws.u_mask, ws.u_count,
                   torch.tensor(seg_of, **i32), ws.scores)
    words = (max(lens) // block + 1 + 31) // 32
    blkmap = torch.zeros(idx_q.shape[0], words, **i32)
    C().qsa_rowmap(ws.u_lpage, ws.u_mask, ws.u_count, torch.tensor(row0, **i32), torch.tensor(nrows, **i32), W,
                   blkmap)
    return blkmap


def varlen_attention_reference(q, k, v, cu_seqlens, allowed=None) -> torch.Tensor:
    """fp32 oracle of :func:`varlen_attention`; ``allowed`` [T, T] bool (packed rows x packed keys) restricts the
    keys further (QSA)."""
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    rep = q.shape[1] // k.shape[1]
    bounds = [int(x) for x in cu_seqlens.tolist()]
    for s0, s1 in zip(bounds[:-1], bounds[1:]):
        qq = q[s0:s1].float().transpose(0, 1)
        kk = k[s0:s1].float().repeat_interleave(rep, 1).transpose(0, 1)
        vv = v[s0:s1].float().repeat_interleave(rep, 1).transpose(0, 1)
        s = qq @ kk.transpose(1, 2) / math.sqrt(q.shape[-1])
        n = s1 - s0
        mask = torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1)
        if allowed is not None:
            mask = mask | ~allowed[s0:s1, s0:s1].to(q.device)
        s = s.masked_fill(mask, float("-inf"))
        out[s0:s1] = (torch.softmax(s, -1) @ vv).transpose(0, 1)
    return out
