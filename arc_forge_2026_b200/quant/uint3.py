"""Humming-compatible ``uint3`` group-128 expert packs.

Stream format (must stay bit-identical to the reference's serving packs):
every 32 consecutive 3-bit codes along the last dim occupy 3 little-endian int32 words; code ``i`` sits
at bits ``3i .. 3i+2`` of that 96-bit group, least significant first, so codes 10 and 21 straddle a
word boundary (``training/work/qwen38fn_lora/int3_moe.py:76-97``; ``training/work/qwen38fn_eval/
export_int3_sidecar.py:32-39``). Dequantisation is ``(code - 4) * scale`` with one signed bf16 scale per
(row, 128-column group) and no zero point.

Expert pack layout (``export_int3_sidecar.py:1-15``)::

    w13_qweight int32 [E, 2I, H*3/32]   rows = gate then up
    w13_scales  bf16  [E, 2I, H/128]
    w2_qweight  int32 [E, H, I*3/32]
    w2_scales   bf16  [E, H, I/128]
"""
from __future__ import annotations

import torch

GROUP = 128
CODE_ZERO = 4


def _check_codes(codes: torch.Tensor):
    if codes.shape[-1] % 32:
        raise ValueError(f"uint3 packing needs the last dim to be a multiple of 32, got {codes.shape[-1]}")


def pack_uint3(codes: torch.Tensor) -> torch.Tensor:
    """uint8/int codes in 0..7, shape [..., k] -> int32 [..., 3k/32]."""
    _check_codes(codes)
    if codes.numel() and int(codes.max()) > 7 or (codes.numel() and int(codes.min()) < 0):
        raise ValueError("uint3 codes must lie in 0..7")
    lead, k = codes.shape[:-1], codes.shape[-1]
    c = codes.reshape(-1, k // 32, 32).to(torch.int64)
    words = torch.zeros(c.shape[0], k // 32, 3, dtype=torch.int64, device=codes.device)
    for i in range(32):
        bit = 3 * i
        w, s = divmod(bit, 32)
        words[..., w] |= (c[..., i] << s) & 0xFFFFFFFF
        if s > 29:  # the code spills into the next word
            words[..., w + 1] |= c[..., i] >> (32 - s)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32).reshape(*lead, 3 * k // 32)


def unpack_uint3(qweight: torch.Tensor, k: int) -> torch.Tensor:
    """int32 [..., 3k/32] -> uint8 codes [..., k]."""
    if qweight.dtype != torch.int32 or k % 32 or qweight.shape[-1] * 32 != 3 * k:
        raise ValueError(f"cannot unpack {k} three-bit codes per row from a {qweight.dtype} tensor of shape "
                         f"{tuple(qweight.shape)}: rows hold k codes in 3*k/32 int32 words, so k must be a "
                         f"multiple of 32")
    lead = qweight.shape[:-1]
    w = qweight.reshape(-1, k // 32, 3).to(torch.int64) & 0xFFFFFFFF
    out = torch.empty(w.shape[0], k // 32, 32, dtype=torch.uint8, device=qweight.device)
    for i in range(32):
        bit = 3 * i
        wi, s = divmod(bit, 32)
        v = w[..., wi] >> s
        if s > 29:
            v = v | (w[..., wi + 1] << (32 - s))
        out[..., i] = (v & 7).to(torch.uint8)
    return out.reshape(*lead, k)


def dequant_uint3(qweight: torch.Tensor, scales: torch.Tensor, k: int, dtype=torch.bfloat16) -> torch.Tensor:
    """(code - 4) * scale, rounded once to ``dtype`` like a bf16 ``__hmul2`` of the exact (code - 4)."""
    codes = unpack_uint3(qweight, k)
    s = scales.float().repeat_interleave(GROUP, dim=-1)
    return ((codes.float() - CODE_ZERO) * s).to(dtype)


def pack_experts(w13_codes, w13_scales, w2_codes, w2_scales) -> dict[str, torch.Tensor]:
    """Codes [E, rows, k] uint8 + scales [E, rows, k/128] -> the four pack tensors (Humming layout)."""
    return {
        "w13_qweight": pack_uint3(w13_codes),
        "w13_scales": w13_scales.to(torch.bfloat16).contiguous(),
        "w2_qweight": pack_uint3(w2_codes),
        "w2_scales": w2_scales.to(torch.bfloat16).contiguous(),
    }


def dequant_experts(pack: dict[str, torch.Tensor], hidden: int, inter: int, dtype=torch.bfloat16):
    w13 = dequant_uint3(pack["w13_qweight"], pack["w13_scales"], hidden, dtype)
    w2 = dequant_uint3(pack["w2_qweight"], pack["w2_scales"], inter, dtype)
    return w13, w2
