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
    """(segment, first position) of every query tile of the forward (128 positions), and of every 64-position tile
    of the backward: ordered for the forward / dQ kernels (longest causal prefix first) and for the dK / dV kernels
    (most query tiles after the key tile first)."""
    def tiles(step):
        return [(s, p, cu[s + 1] - cu[s]) for s in range(len(cu) - 1) for p in range(0, cu[s + 1] - cu[s], step)]
    mk = lambda ts: torch.tensor([[s, p] for s, p, _ in ts], dtype=torch.int32).reshape(-1, 2).to(device)  # noqa: E731
    t64 = tiles(TILE)
    return (mk(sorted(tiles(2 * TILE), key=lambda t: -t[1])), mk(sorted(t64, key=lambda t: -t[1])),
            mk(sorted(t64, key=lambda t: -(t[2] - t[1]))))


class VarlenCausalAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens):
        cu_host = [int(x) for x in cu_seqlens.tolist()]
        cu = torch.tensor(cu_host, dtype=torch.int32, device=q.device)
        fwd_tiles, q_tiles, kv_tiles = tile_lists(cu_host, q.device)
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        T, Hq, D = q.shape
        out = torch.empty_like(q)
        lse = torch.empty(Hq, T, dtype=torch.float32, device=q.device)
        scale = 1.0 / math.sqrt(D)
        C().attn_train_fwd(q, k, v, cu, fwd_tiles, scale, out, lse)
        ctx.save_for_backward(q, k, v, out, lse, cu, q_tiles, kv_tiles)
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, cu, q_tiles, kv_tiles = ctx.saved_tensors
        dout = dout.contiguous().to(torch.bfloat16)
        delta = torch.empty_like(lse)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        # per-query-head fp32 dK / dV contributions (every row written; the reduce sums each KV group's heads in a
        # fixed order)
        dk_part = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        dv_part = torch.empty_like(dk_part)
        C().attn_train_bwd(q, k, v, cu, q_tiles, kv_tiles, ctx.scale, out, lse, dout, delta, dq, dk, dv, dk_part,
                           dv_part)
        return dq, dk, dv, None


def varlen_attention(q, k, v, cu_seqlens) -> torch.Tensor:
    """Causal attention inside each segment of a packed row (bf16, CUDA): q [T, Hq, D], k / v [T, Hkv, D]."""
    return VarlenCausalAttention.apply(q, k, v, cu_seqlens)


def varlen_attention_reference(q, k, v, cu_seqlens) -> torch.Tensor:
    """fp32 oracle of :func:`varlen_attention`."""
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
        s = s.masked_fill(mask, float("-inf"))
        out[s0:s1] = (torch.softmax(s, -1) @ vv).transpose(0, 1)
    return out
