"""Straight-through quantisers of QAD: INT3 experts with trainable group scales, and block-FP8 dense QAT.

* :class:`Int3ScaleSTE` -- codes frozen, fp32 master scales trainable. Forward ``W = bf16((c - 4) * bf16(s))``
  (the serving product); backward ``dS[e, n, g] = sum_{k in g} (c - 4) * dW[e, n, k]`` (the reference's scale-QAT
  gradient, ``training/work/qwen38fn_qad/int3_scale_qat.py:1-29``; its ``scale_grad_triton.py`` computes the same
  group-reduce). Gradients of zero-valued scales are masked by the trainer (sign and zero invariants).
* :class:`FP8BlockSTE` -- fp32 master -> bf16 cast -> 128x128 block e4m3 round trip in the forward, identity in the
  backward (``training/work/qwen38fn_qad/dense_full_qat.py:1-20``).

On CUDA both run the native kernels; on CPU they run the plain-torch oracle (same math).
"""
from __future__ import annotations

import torch

from ..quant import fp8 as fp8q
from ..quant.int3_tiles import tiles_to_codes


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


class Int3ScaleSTE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, scales: torch.Tensor, codes: torch.Tensor):
        E, RB, KG = codes.shape[0], codes.shape[1], codes.shape[2]
        R, K = RB * 128, KG * 128
        ctx.save_for_backward(codes)
        if _cuda(scales):
            from ..ops import C
            out = torch.empty(E, R, K, dtype=torch.bfloat16, device=scales.device)
            C().int3_dequant(codes, scales.contiguous(), out)
            return out
        c = tiles_to_codes(codes).float() - 4.0
        s = scales.to(torch.bfloat16).float().repeat_interleave(128, -1)
        return (c * s).to(torch.bfloat16)

    @staticmethod
    def backward(ctx, dW: torch.Tensor):
        (codes,) = ctx.saved_tensors
        E, RB, KG = codes.shape[0], codes.shape[1], codes.shape[2]
        R = RB * 128
        if dW.is_cuda:
            from ..ops import C
            dS = torch.empty(E, R, KG, dtype=torch.float32, device=dW.device)
            C().int3_scale_grad(codes, dW.to(torch.bfloat16).contiguous(), dS)
            return dS, None
        c = tiles_to_codes(codes).float() - 4.0
        dS = (c * dW.to(torch.bfloat16).float()).view(E, R, KG, 128).sum(-1)
        return dS, None


class FP8BlockSTE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, w: torch.Tensor):
        if _cuda(w):
            from ..ops import C
            out = torch.empty(w.shape, dtype=torch.bfloat16, device=w.device)
            C().fp8_block_fakequant(w.contiguous(), out, None)
            return out
        q, s = fp8q.quantize_weight_block(w.to(torch.bfloat16).float())
        return fp8q.dequant_weight_block(q, s).to(torch.bfloat16)

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        return g.float()


def int3_weight(scales, codes):
    from . import kernels
    if scales.is_cuda:
        kernels.hit("int3_weight", True)
    return Int3ScaleSTE.apply(scales, codes)


def fp8_weight(master):
    from . import kernels
    if master.is_cuda:
        kernels.hit("fp8_weight", True)
    return FP8BlockSTE.apply(master)
