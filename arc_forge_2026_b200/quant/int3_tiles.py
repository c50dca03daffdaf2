"""Kernel tile layout of uint3 g128 experts (what the sm_100a expert GEMM streams).

The Humming ``uint3`` pack (``quant/uint3.py``) is the interchange format; at load time each expert matrix is
re-laid out, still at exactly 3 bits per weight, as::

    codes  int32 [E, R/128, K/128, 128 rows, 12 words]     one contiguous 6 KB tile per (row block, K group)
    scales bf16  [E, R/128, K/128, 128 rows]

so one bulk copy moves a tile. Within a row, each 32-code sub-group occupies 3 words: two low-bit planes and
one high-bit plane, arranged so that a byte-permute turns 4 codes into 4 e4m3 ``(code - 4)`` bytes::

    L0 nibble n = (c_n & 3) | (c_{8+n} & 3) << 2
    L1 nibble n = (c_{16+n} & 3) | (c_{24+n} & 3) << 2
    H  nibble n = (c_{16+n} >> 2) | (c_{24+n} >> 2) << 1 | (c_n >> 2) << 2 | (c_{8+n} >> 2) << 3

``to_tiles``/``from_tiles`` are exact inverses; the tests check them against the Humming stream.
"""
from __future__ import annotations

import torch

from .uint3 import unpack_uint3

GROUP = 128


def _nib(vals: torch.Tensor) -> torch.Tensor:
    """vals [..., 8] small ints (already positioned inside a nibble) -> int64 word with nibble n = vals[n]."""
    shifts = torch.arange(8, device=vals.device, dtype=torch.int64) * 4
    return (vals.to(torch.int64) << shifts).sum(-1)


def codes_to_tiles(codes: torch.Tensor) -> torch.Tensor:
    """codes uint8 [E, R, K] -> int32 [E, R/128, K/128, 128, 12]."""
    E, R, K = codes.shape
    if R % 128 or K % 128:
        raise ValueError(f"tile layout needs rows and K divisible by 128, got {R}x{K}")
    c = codes.to(torch.int64).reshape(E, R // 128, 128, K // 128, 4, 32)
    c0, c1, c2, c3 = c[..., 0:8], c[..., 8:16], c[..., 16:24], c[..., 24:32]
    L0 = _nib((c0 & 3) | ((c1 & 3) << 2))
    L1 = _nib((c2 & 3) | ((c3 & 3) << 2))
    Hw = _nib((c2 >> 2) | ((c3 >> 2) << 1) | ((c0 >> 2) << 2) | ((c1 >> 2) << 3))
    words = torch.stack([L0, L1, Hw], dim=-1)  # [E, RB, 128, KG, 4, 3]
    words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    return words.reshape(E, R // 128, 128, K // 128, 12).permute(0, 1, 3, 2, 4).contiguous()


def tiles_to_codes(tiles: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`codes_to_tiles`."""
    E, RB, KG, _, _ = tiles.shape
    w = tiles.permute(0, 1, 3, 2, 4).reshape(E, RB, 128, KG, 4, 3).to(torch.int64) & 0xFFFFFFFF
    n = torch.arange(8, device=tiles.device, dtype=torch.int64) * 4
    L0 = (w[..., 0:1] >> n) & 0xF
    L1 = (w[..., 1:2] >> n) & 0xF
    Hw = (w[..., 2:3] >> n) & 0xF
    c0 = (L0 & 3) | (((Hw >> 2) & 1) << 2)
    c1 = ((L0 >> 2) & 3) | (((Hw >> 3) & 1) << 2)
    c2 = (L1 & 3) | ((Hw & 1) << 2)
    c3 = ((L1 >> 2) & 3) | (((Hw >> 1) & 1) << 2)
    codes = torch.cat([c0, c1, c2, c3], dim=-1)  # [E, RB, 128, KG, 4, 32]
    return codes.reshape(E, RB * 128, KG * 128).to(torch.uint8)


def scales_to_tiles(scales: torch.Tensor) -> torch.Tensor:
    """bf16 [E, R, K/128] -> bf16 [E, R/128, K/128, 128]."""
    E, R, KG = scales.shape
    return scales.to(torch.bfloat16).reshape(E, R // 128, 128, KG).permute(0, 1, 3, 2).contiguous()


def tiles_to_scales(t: torch.Tensor) -> torch.Tensor:
    E, RB, KG, _ = t.shape
    return t.permute(0, 1, 3, 2).reshape(E, RB * 128, KG)


def pack_to_tiles(qweight: torch.Tensor, scales: torch.Tensor, k: int):
    """Humming pack (int32 [E, R, 3k/32], bf16 [E, R, k/128]) -> (tile codes, tile scales)."""
    codes = unpack_uint3(qweight, k)
    return codes_to_tiles(codes), scales_to_tiles(scales)
