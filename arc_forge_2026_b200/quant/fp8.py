"""Block-scaled FP8 (e4m3) formats.

* Weights: one fp32 scale per 128x128 block, stored as ``weight_scale_inv`` ``[ceil(N/128), ceil(K/128)]``
  (the DeepSeek-style layout the reference packages use, ``training/work/qwen38fn_eval/quantize_nonmoe_fp8.py:57-70``):
  ``scale = amax / 448`` (1 for an all-zero block), ``q = clamp(w / scale, +-448)`` cast to e4m3.
* Activations: one fp32 scale per (row, 128-column group) (``training/work/qwen38fn_lora/fp8_moe.py:78-100``).

Both are plain torch and serve as the oracle of the fused quantisers in the kernels.
"""
from __future__ import annotations

import torch

BLOCK = 128
FP8_MAX = 448.0
E4M3 = torch.float8_e4m3fn


def _pad_to(x: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    r, c = x.shape
    if r == rows and c == cols:
        return x
    out = x.new_zeros(rows, cols)
    out[:r, :c] = x
    return out


def quantize_weight_block(w: torch.Tensor, block: int = BLOCK):
    """w [N, K] -> (e4m3 [N, K], scale_inv fp32 [ceil(N/b), ceil(K/b)])."""
    N, K = w.shape
    nb, kb = -(-N // block), -(-K // block)
    wp = _pad_to(w.float(), nb * block, kb * block)
    blocked = wp.view(nb, block, kb, block)
    amax = blocked.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (blocked / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).view(nb * block, kb * block)
    return q[:N, :K].to(E4M3).contiguous(), scale.float()


def dequant_weight_block(q: torch.Tensor, scale_inv: torch.Tensor, block: int = BLOCK, dtype=torch.float32):
    N, K = q.shape
    s = scale_inv.float().repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return (q.float() * s).to(dtype)


def quantize_act_groups(x: torch.Tensor, group: int = BLOCK):
    """x [M, K] -> (e4m3 [M, K], scales fp32 [M, K/group]); scale = amax/448 per (row, group)."""
    M, K = x.shape
    if K % group:
        raise ValueError(f"activation groups of {group} need K % {group} == 0, got {K}")
    g = x.float().view(M, K // group, group)
    amax = g.abs().amax(-1)
    scale = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    q = (g / scale[..., None]).clamp(-FP8_MAX, FP8_MAX).view(M, K).to(E4M3)
    return q, scale


def dequant_act_groups(q: torch.Tensor, scales: torch.Tensor, group: int = BLOCK, dtype=torch.float32):
    return (q.float() * scales.float().repeat_interleave(group, -1)).to(dtype)


def quantize_rows(x: torch.Tensor):
    """Per-row e4m3 (the W3A8 expert input format): scale = max(amax, 1e-30)/448, values multiplied by the fp32
    reciprocal of the scale (as the kernels and the reference's quantiser do) and rounded to e4m3."""
    amax = x.float().abs().amax(-1).clamp_min(1e-30)
    scale = amax / FP8_MAX
    inv = 1.0 / scale
    return (x.float() * inv[:, None]).clamp(-FP8_MAX, FP8_MAX).to(E4M3), scale


def block_fp8_linear_ref(x: torch.Tensor, wq: torch.Tensor, w_scale_inv: torch.Tensor, group: int = BLOCK):
    """Reference W8A8 GEMM: activations quantised 1x128, weights 128x128, fp32 accumulate, per-block scale FMA."""
    xq, xs = quantize_act_groups(x, group)
    return dequant_act_groups(xq, xs, group) @ dequant_weight_block(wq, w_scale_inv, group).t()
