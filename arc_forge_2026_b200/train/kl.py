"""Top-k + tail KL of a student against teacher top-k log-probs (the QAD distillation loss).

For each position the teacher gives ``k`` ids (full-vocabulary log-probs ``t_lp``) and the tail mass
``t_tail = log(1 - sum exp(t_lp))``; the student's full softmax ``q`` is coarsened to the same ``k + 1``
classes (tail = logsumexp of the non-top-k logits). Loss and gradients (``training/work/qwen38fn_qad/
topk_tail_kl.py:1-28`` states the same contract; ``k`` is 32 there and configurable here, 64 for BASELINE
config 4)::

    forward:  L = sum_i p_i (log p_i - log q_i) + p_R (log p_R - log q_R)
              dL/dz_j = q_j - p_j (j in K);   q_j (1 - p_R / q_R) (j not in K)
    reverse:  L = sum_c Q_c g_c,  g_c = log Q_c - log P_c
              dL/dz_j = q_j (g_{c(j)} - L)

This module is the fp32/fp64 oracle; the fused LM-head + loss kernel is tested against it.
"""
from __future__ import annotations

import torch

DIRECTIONS = ("forward", "reverse")


def topk_tail_kl(z: torch.Tensor, ids: torch.Tensor, t_lp: torch.Tensor, t_tail: torch.Tensor,
                 direction: str = "forward"):
    """z [N, V] student logits (fp32 math) -> (loss [N], dL/dz [N, V])."""
    if direction not in DIRECTIONS:
        raise ValueError(f"direction {direction!r}")
    z = z.float()
    lse = z.logsumexp(-1)
    lq_k = z.gather(1, ids) - lse[:, None]
    lq_r = z.scatter(1, ids, float("-inf")).logsumexp(-1) - lse
    q = (z - lse[:, None]).exp()
    if direction == "forward":
        p_k, p_r = t_lp.float().exp(), t_tail.float().exp()
        head = (p_k * (t_lp - lq_k)).sum(-1)
        tail = torch.where(p_r > 0, p_r * (t_tail - lq_r), torch.zeros_like(p_r))
        loss = head + tail
        q_r = lq_r.exp()
        factor = torch.where(q_r > 0, 1 - p_r / q_r, torch.ones_like(q_r))
        dz = q * factor[:, None]
        dz.scatter_(1, ids, lq_k.exp() - p_k)
        return loss, dz
    g_k = lq_k - t_lp
    g_r = lq_r - t_tail
    q_k, q_r = lq_k.exp(), lq_r.exp()
    head = torch.where(q_k > 0, q_k * g_k, torch.zeros_like(q_k)).sum(-1)
    tail = torch.where(q_r > 0, q_r * g_r, torch.zeros_like(q_r))
    loss = head + tail
    g_r = torch.where(q_r > 0, g_r, torch.zeros_like(g_r))
    dz = q * (g_r - loss)[:, None]
    dz.scatter_(1, ids, torch.where(q_k > 0, q_k * (g_k - loss[:, None]), torch.zeros_like(q_k)))
    return loss, dz


def teacher_topk(z: torch.Tensor, k: int):
    """Teacher logits [N, V] -> (ids int64 [N, k], log-probs fp32 [N, k], tail fp32 [N])."""
    z = z.float()
    lse = z.logsumexp(-1)
    vals, ids = torch.topk(z, k, dim=-1)
    lp = vals - lse[:, None]
    tail = z.scatter(1, ids, float("-inf")).logsumexp(-1) - lse
    return ids, lp, tail


class TopKTailKL(torch.autograd.Function):
    """Autograd wrapper over :func:`topk_tail_kl` on logits (oracle path; the GPU path fuses the LM head)."""

    @staticmethod
    def forward(ctx, z, ids, t_lp, t_tail, direction):
        loss, dz = topk_tail_kl(z, ids, t_lp, t_tail, direction)
        ctx.save_for_backward(dz)
        return loss.sum()

    @staticmethod
    def backward(ctx, g):
        (dz,) = ctx.saved_tensors
        return dz * g, None, None, None, None
