"""Top-k + tail KL of a student against teacher top-k log-probs (the QAD distillation loss).

Contract (the same one ``training/work/qwen38fn_qad/topk_tail_kl.py:1-28`` states; ``k`` is 32 there and
configurable here, 64 for BASELINE config 4): the teacher gives, per position, ``k`` token ids with their
full-vocabulary log-probs ``t_lp`` and the log of the remaining mass ``t_tail``. Both distributions are coarsened
to the same ``k + 1`` classes -- the listed ids, one class each, and "rest" for every other token -- and the loss is
the KL divergence between the two coarse distributions, forward ``KL(P||Q)`` or reverse ``KL(Q||P)``.

Gradient, derived once for both directions. With ``s = softmax(z)`` the coarse student probabilities are
``Q_c = sum_{j in c} s_j``. Write ``c(j)`` for the class of token ``j`` and ``r_j = s_j / Q_{c(j)}`` for its share
of that class (1 for a listed token). Then ``d log Q_c / dz_j = [j in c] r_j - s_j``, so for any loss with
``u_c = dL/d log Q_c`` the chain rule gives

    dL/dz_j = u_{c(j)} r_j - s_j sum_c u_c

The two losses differ only in ``u``:

    forward  L = sum_c P_c (log P_c - log Q_c)     u_c = -P_c                         sum_c u_c = -1
    reverse  L = sum_c Q_c (log Q_c - log P_c)     u_c = Q_c (log Q_c - log P_c + 1)   sum_c u_c = L + 1

so a listed token gets ``s_j - P_j`` (forward) and every token of class ``c`` gets ``s_j (g_c - L)`` with
``g_c = log Q_c - log P_c`` (reverse). Classes with zero probability contribute nothing (``0 log 0 = 0``). ``r_j``
is formed in log space (``exp(log s_j - log Q_c)``), so it stays exact when a whole class underflows in fp32.

``topk_tail_kl`` evaluates this closed form in fp32; ``topk_tail_kl_autograd`` is an independent oracle that
differentiates the coarse KL with autograd in fp64. The fused LM-head + loss kernel is tested against both.
"""
from __future__ import annotations

import torch

DIRECTIONS = ("forward", "reverse")


def coarse_log_probs(z: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """Student logits [N, V] -> log-probs [N, k + 1] of the listed ids (columns 0..k-1) and of the rest (column k)."""
    logz = z.logsumexp(-1, keepdim=True)
    listed = z.gather(1, ids) - logz
    rest = z.scatter(1, ids, float("-inf")).logsumexp(-1, keepdim=True) - logz
    return torch.cat([listed, rest], 1)


def coarse_kl(log_q: torch.Tensor, log_p: torch.Tensor, direction: str) -> torch.Tensor:
    """KL between two coarse distributions given as log-probs [N, C]; zero-probability classes add nothing."""
    if direction == "forward":
        src, lsrc, lother = log_p.exp(), log_p, log_q
    else:
        src, lsrc, lother = log_q.exp(), log_q, log_p
    terms = torch.where(src > 0, src * (lsrc - lother), torch.zeros_like(src))
    return terms.sum(-1)


def _check(direction):
    if direction not in DIRECTIONS:
        raise ValueError(f"direction {direction!r}")


def topk_tail_kl(z: torch.Tensor, ids: torch.Tensor, t_lp: torch.Tensor, t_tail: torch.Tensor,
                 direction: str = "forward"):
    """z [N, V] student logits (fp32 math) -> (loss [N], dL/dz [N, V]) by the closed form above."""
    _check(direction)
    z = z.float()
    log_q = coarse_log_probs(z, ids)                                   # [N, k + 1]
    log_p = torch.cat([t_lp.float(), t_tail.float()[:, None]], 1)
    loss = coarse_kl(log_q, log_p, direction)
    if direction == "forward":
        u = -log_p.exp()                                                # u_c = -P_c
        u_sum = -torch.ones_like(loss)
    else:
        q = log_q.exp()
        u = torch.where(q > 0, q * (log_q - log_p + 1), torch.zeros_like(q))  # u_c = Q_c (g_c + 1)
        u_sum = loss + 1
    log_s = z - z.logsumexp(-1, keepdim=True)
    # every token starts in the rest class (r_j = exp(log s_j - log Q_rest)); listed tokens have r_j = 1
    r = (log_s - log_q[:, -1:]).exp().nan_to_num(0.0)
    dz = u[:, -1:] * r - log_s.exp() * u_sum[:, None]
    dz.scatter_(1, ids, u[:, :-1] - log_s.gather(1, ids).exp() * u_sum[:, None])
    return loss, dz


def topk_tail_kl_autograd(z: torch.Tensor, ids: torch.Tensor, t_lp: torch.Tensor, t_tail: torch.Tensor,
                          direction: str = "forward"):
    """fp64 oracle: the coarse KL of :func:`coarse_log_probs` differentiated by autograd -> (loss, dL/dz) in fp32."""
    _check(direction)
    with torch.enable_grad():
        z64 = z.detach().double().requires_grad_(True)
        log_p = torch.cat([t_lp.double(), t_tail.double()[:, None]], 1)
        loss = coarse_kl(coarse_log_probs(z64, ids), log_p, direction)
        (dz,) = torch.autograd.grad(loss.sum(), z64)
    return loss.detach().float(), dz.float()


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
