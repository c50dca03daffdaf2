"""Paged decode / verify attention on the native kernel, its split heuristic, and the fp32 oracle."""
from __future__ import annotations

import math

import torch

from ._ext import C

PAGE = 64


def plan_splits(num_seqs: int, Hkv: int, max_pages: int, num_sms: int = 148) -> tuple[int, int]:
    """Split KV so that the grid covers ~6 waves of SMs (short tail when context lengths differ) while each split
    keeps >= 12 pages to amortise its prologue."""
    ctas = max(1, num_seqs * Hkv)
    splits = 1
    while ctas * splits < 6 * num_sms and math.ceil(max_pages / (splits * 2)) >= 12:
        splits *= 2
    pps = math.ceil(max(1, max_pages) / splits)
    return math.ceil(max(1, max_pages) / pps), pps


def paged_attention(q, kcache, vcache, block_table, seq_lens, q_per_seq, out, gate=None, gate_ld=0,
                    gate_head_stride=0, splits=None, max_pages=None, window=0, bt_row=None, kv_scales=None, impl=0):
    """``impl`` 0 runs the tcgen05 kernel wherever it applies (bf16 cache, dense, no window, no virtual rows) and the
    mma.sync kernel otherwise; 1 always runs the mma.sync kernel. ``max_pages`` bounds the pages any sequence spans (it sizes the split plan; defaults to the table width).
    ``window`` > 0 restricts each query to its last ``window`` keys. ``bt_row`` maps (virtual) sequences to
    block-table rows (prefill chunks of 8 queries share their sequence's row). ``kv_scales`` = (kscale, vscale):
    the cache is NVFP4 (see :func:`nvfp4_dequant`)."""
    D = q.shape[-1]
    mp = max_pages if max_pages is not None else block_table.shape[1]
    if window > 0:
        mp = min(mp, window // PAGE + 2)
    if splits is None:
        splits, pps = plan_splits(seq_lens.shape[0], kcache.shape[1], mp)
    else:
        pps = math.ceil(mp / splits)
    ks, vs = kv_scales if kv_scales else (None, None)
    C().paged_attention(q, kcache, vcache, block_table, seq_lens, q_per_seq, 1.0 / math.sqrt(D), out, gate,
                        gate_ld, gate_head_stride, splits, pps, window, bt_row, kscale=ks, vscale=vs, impl=impl)
    return out


# NVFP4 KV format: e2m1 values (sign, 2 exponent bits, 1 mantissa bit: 0, 0.5, 1, 1.5, 2, 3, 4, 6), two per byte
# with the first element in the low nibble, and one e4m3 scale per 16 consecutive elements of a row.
E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def new_nvfp4_kv(num_pages: int, Hkv: int, D: int, device):
    """An empty NVFP4 cache of one layer: (k, v, kscale, vscale) — codes [pages, Hkv, 64, D/2] and e4m3 scales
    [pages, Hkv, 64, D/16], all uint8 (0.5625 bytes per element against bf16's 2)."""
    codes = dict(dtype=torch.uint8, device=device)
    return (torch.zeros(num_pages, Hkv, PAGE, D // 2, **codes), torch.zeros(num_pages, Hkv, PAGE, D // 2, **codes),
            torch.zeros(num_pages, Hkv, PAGE, D // 16, **codes), torch.zeros(num_pages, Hkv, PAGE, D // 16, **codes))


def nvfp4_dequant(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """[..., D/2] uint8 codes and [..., D/16] e4m3 scales -> [..., D] fp32."""
    lut = E2M1.to(codes.device)
    lo, hi = lut[(codes & 15).long()], lut[(codes >> 4).long()]
    x = torch.stack([lo, hi], -1).flatten(-2)                                   # [..., D]
    s = scales.view(torch.float8_e4m3fn).float().repeat_interleave(16, -1)
    return x * s


def paged_attention_reference(q, kcache, vcache, block_table, seq_lens, q_per_seq, gate=None, window=0):
    """fp32 oracle. q [S*qp, Hq, D]; gate [S*qp, Hq, D] or None."""
    S = seq_lens.shape[0]
    Hq, D = q.shape[1], q.shape[2]
    Hkv = kcache.shape[1]
    rep = Hq // Hkv
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for s in range(S):
        L = int(seq_lens[s])
        pages = block_table[s, : (L + PAGE - 1) // PAGE].long()
        k = kcache[pages].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :L].float()
        v = vcache[pages].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :L].float()
        qq = q[s * q_per_seq:(s + 1) * q_per_seq].float()  # [qp, Hq, D]
        kk = k.repeat_interleave(rep, 0)
        vv = v.repeat_interleave(rep, 0)
        sc = torch.einsum("thd,hld->htl", qq, kk) / math.sqrt(D)
        pos = torch.arange(L - q_per_seq, L, device=q.device)
        keys = torch.arange(L, device=q.device)[None, :]
        mask = keys > pos[:, None]
        if window > 0:
            mask = mask | (keys <= pos[:, None] - window)
        sc = sc.masked_fill(mask[None], float("-inf"))
        o = torch.einsum("htl,hld->thd", torch.softmax(sc, -1), vv)
        out[s * q_per_seq:(s + 1) * q_per_seq] = o
    if gate is not None:
        out = out * torch.sigmoid(gate.float())
    return out
