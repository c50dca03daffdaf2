"""Grouped expert GEMMs of the QAD student on the tcgen05 GEMM kernel (``csrc/gemm_bf16.cu`` grouped modes), in
place of a library grouped GEMM (the reference's quack SM100 grouped GEMM for its W3A16 experts,
``training/work/qwen38fn_lora/int3_moe.py:373-467``).

    forward   Y[r] = X[r] W_e^T            ROWS mode: rows sorted by expert, one launch for every expert
    dX        dX[r] = dY[r] W_e             ROWS mode over the transposed bank W^T [E, K, N]
    dW        dW_e = dY_e^T X_e             REDUCE mode: X and dY copied into 64-row-aligned expert segments and
                                            transposed, so each expert's K range is whole 64-row blocks

All three accumulate in fp32 on the tensor cores and store bf16 (the dtype the INT3 scale STE consumes). Host work
is shape-only: the segment and tile prefixes stay on the device (no synchronisation).
"""
from __future__ import annotations

import torch

_BF = torch.bfloat16


def _prefix(v: torch.Tensor) -> torch.Tensor:
    return torch.cat([v.new_zeros(1), v.cumsum(0)]).int()


def grouped_rows(x: torch.Tensor, w: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    """x [R, K] bf16 (rows sorted by expert, ``counts`` [E] rows each), w [E, N, K] bf16 -> [R, N] bf16."""
    from ..ops import C
    E, N, K = w.shape
    R = x.shape[0]
    out = torch.empty(R, N, dtype=_BF, device=x.device)
    if R == 0:
        return out
    seg = _prefix(counts)
    tiles = _prefix((counts + 127) // 128)
    C().gemm_grouped(x.contiguous(), w.reshape(E * N, K).contiguous(), seg, tiles, 1, N, (R + 127) // 128 + E, out)
    return out


def grouped_reduce(dy: torch.Tensor, x: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    """dy [R, N], x [R, K] (rows sorted by expert) -> dW [E, N, K] bf16 = per expert dy_e^T x_e."""
    from ..ops import C
    R, N = dy.shape
    K = x.shape[1]
    E = counts.shape[0]
    dev = x.device
    padded = (counts + 63) // 64 * 64
    pseg = _prefix(padded)
    seg = _prefix(counts)
    rows = (R + 64 * E + 63) // 64 * 64  # upper bound of the padded rows (no host sync); 16-byte row pitch
    owner = torch.repeat_interleave(torch.arange(E, device=dev), counts, output_size=R)
    dst = (torch.arange(R, device=dev) - seg[owner] + pseg[owner]).long()
    c = C()
    # X^T and dY^T with every expert's rows at its 64-aligned column segment (one native transpose each)
    xt = torch.zeros(K, rows, dtype=_BF, device=dev)
    dyt = torch.zeros(N, rows, dtype=_BF, device=dev)
    c.transpose_bf16(x.to(_BF).contiguous(), dst, xt)
    c.transpose_bf16(dy.to(_BF).contiguous(), dst, dyt)
    out = torch.empty(E, N, K, dtype=_BF, device=dev)
    c.gemm_grouped(dyt, xt, pseg, None, 2, N, 0, out)
    return out


def transposed_bank(w: torch.Tensor) -> torch.Tensor:
    """[E, N, K] bf16 -> [E, K, N] (native tiled transpose)."""
    from ..ops import C
    E, N, K = w.shape
    out = torch.empty(E, K, N, dtype=_BF, device=w.device)
    C().transpose_bf16(w.contiguous(), None, out)
    return out


class GroupedLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, counts):
        xb, wb = x.to(_BF).contiguous(), w.to(_BF).contiguous()
        ctx.save_for_backward(xb, wb, counts)
        return grouped_rows(xb, wb, counts)

    @staticmethod
    def backward(ctx, dy):
        xb, wb, counts = ctx.saved_tensors
        dy = dy.to(_BF).contiguous()
        dx = grouped_rows(dy, transposed_bank(wb), counts) if ctx.needs_input_grad[0] else None
        dw = grouped_reduce(dy, xb, counts) if ctx.needs_input_grad[1] else None
        return dx, dw, None
