"""AdamW with bf16 moment states on fp32 masters ("bf16 AdamW").

On CUDA every parameter update is one fused kernel (moments, bias correction, decoupled weight decay, update, and
an optional bf16 copy of the new weights). Parameter groups carry their own learning rate (the reference QAD uses
1e-5 for scales, 3e-6 for routers, 2e-6 for dense weights: ``training/work/qwen38fn_qad/train_qad.py:540-541``).
Gradient clipping by global norm is done by :func:`clip_grad_norm_` over all groups (and all ranks when a process
group is given).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


class AdamWBF16(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-5, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure=None):
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.dtype != torch.float32:
                    raise TypeError("AdamWBF16 keeps fp32 master parameters")
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["m"] = torch.zeros_like(p, dtype=torch.bfloat16)
                    st["v"] = torch.zeros_like(p, dtype=torch.bfloat16)
                st["step"] += 1
                g = p.grad if p.grad.dtype == torch.float32 else p.grad.float()
                if p.is_cuda:
                    from ..ops import C
                    C().adamw(p.data, g.contiguous(), st["m"], st["v"], None, group["lr"], b1, b2, group["eps"],
                              group["weight_decay"], st["step"])
                else:
                    m = b1 * st["m"].float() + (1 - b1) * g
                    v = b2 * st["v"].float() + (1 - b2) * g * g
                    st["m"].copy_(m)
                    st["v"].copy_(v)
                    bc1 = 1 - b1 ** st["step"]
                    bc2 = 1 - b2 ** st["step"]
                    p.sub_(group["lr"] * (group["weight_decay"] * p + (m / bc1) / ((v / bc2).sqrt() + group["eps"])))


@torch.no_grad()
def clip_grad_norm_(params, max_norm: float, group=None) -> float:
    """Global-norm clipping; with a process group the squared norms are summed over ranks (sharded grads)."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return 0.0
    sq = torch.stack([g.float().pow(2).sum() for g in grads]).sum()
    if group is not None and dist.is_initialized():
        dist.all_reduce(sq, group=group)
    norm = float(sq.sqrt())
    if not math.isfinite(norm):
        raise FloatingPointError(f"non-finite gradient norm {norm}")
    if max_norm > 0 and norm > max_norm:
        scale = max_norm / (norm + 1e-6)
        for g in grads:
            g.mul_(scale)
    return norm
