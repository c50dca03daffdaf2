"""Fused LM-head + top-k tail KL (the QAD loss) and the RL token losses.

``fused_topk_tail_kl(hidden, weight, weight_t, ids, t_lp, t_tail)`` computes, chunk by chunk of rows, the fp32
logits with the native tcgen05 GEMM, the per-row loss and dL/dz with the ``topk_tail_kl`` kernel (one pass for the
log-sum-exps, one for the gradient), and dL/dhidden = dz @ W with the native GEMM against the pre-transposed head
(``weight_t`` [H, V]). The [rows, V] logits never exist beyond one chunk, and the LM head is frozen (no weight
gradient), as in the reference (``training/work/qwen38fn_qad/topk_tail_kl.py:1-28``). Backward scales the saved
dL/dhidden by the upstream gradient. The CPU path runs the fp32 oracle of ``train.kl``.
"""
from __future__ import annotations

import torch

from .kl import topk_tail_kl

CHUNK_ROWS = 2048


class FusedTopKTailKL(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, weight_t, ids, t_lp, t_tail, reverse, chunk_rows):
        N, H = hidden.shape
        V = weight.shape[0]
        dh = torch.empty(N, H, dtype=torch.bfloat16, device=hidden.device)
        total = torch.zeros((), dtype=torch.float32, device=hidden.device)
        if hidden.is_cuda:
            from ..ops import C
            c = C()
            rows = min(chunk_rows, N)
            z = torch.empty(rows, V, dtype=torch.float32, device=hidden.device)
            dz = torch.empty(rows, V, dtype=torch.bfloat16, device=hidden.device)
            loss = torch.empty(rows, dtype=torch.float32, device=hidden.device)
            hb = hidden.to(torch.bfloat16).contiguous()
            for r0 in range(0, N, rows):
                n = min(rows, N - r0)
                c.gemm(hb[r0:r0 + n], weight, out=z[:n], out_fp32=True)
                c.topk_tail_kl(z[:n], ids[r0:r0 + n], t_lp[r0:r0 + n], t_tail[r0:r0 + n], reverse, 1.0, loss[:n],
                               dz[:n])
                c.gemm(dz[:n], weight_t, out=dh[r0:r0 + n])
                total += loss[:n].sum()
        else:
            for r0 in range(0, N, chunk_rows):
                h = hidden[r0:r0 + chunk_rows].float()
                zc = h @ weight.float().t()
                l, g = topk_tail_kl(zc, ids[r0:r0 + chunk_rows], t_lp[r0:r0 + chunk_rows],
                                    t_tail[r0:r0 + chunk_rows], "reverse" if reverse else "forward")
                total += l.sum()
                dh[r0:r0 + chunk_rows] = (g @ weight.float()).to(torch.bfloat16)
        ctx.save_for_backward(dh)
        ctx.dtype = hidden.dtype
        return total

    @staticmethod
    def backward(ctx, g):
        (dh,) = ctx.saved_tensors
        return (dh.float() * g).to(ctx.dtype), None, None, None, None, None, None, None


def fused_topk_tail_kl(hidden, weight, weight_t, ids, t_lp, t_tail, direction="forward", chunk_rows=CHUNK_ROWS):
    """Summed loss over rows (divide by the number of rows for the mean)."""
    if direction not in ("forward", "reverse"):
        raise ValueError(direction)
    if hidden.is_cuda:
        from . import kernels
        kernels.hit("topk_tail_kl", True)
    return FusedTopKTailKL.apply(hidden, weight, weight_t, ids, t_lp, t_tail, direction == "reverse", chunk_rows)


# ------------------------------------------------------------------------------------------------ RL losses
def selective_logprob(hidden, weight, labels, temperature=1.0, chunk_rows=CHUNK_ROWS):
    """log softmax(h W^T / T)[label] and the entropy per row, chunked (``training/work/qwen38fn_lora/rl_loss.py``)."""
    out_lp, out_ent = [], []
    for r0 in range(0, hidden.shape[0], chunk_rows):
        z = (hidden[r0:r0 + chunk_rows].float() @ weight.float().t()) / temperature
        lp = torch.log_softmax(z, -1)
        out_lp.append(lp.gather(1, labels[r0:r0 + chunk_rows, None]).squeeze(1))
        out_ent.append(-(lp.exp() * lp).sum(-1))
    return torch.cat(out_lp), torch.cat(out_ent)


def bpo_loss(logp, old_logp, advantages, mask, clip=(0.2, 0.28)):
    """Clipped importance-ratio policy loss per token (PPO-style bounds), mean over masked tokens."""
    ratio = torch.exp(logp - old_logp)
    lo, hi = 1.0 - clip[0], 1.0 + clip[1]
    unclipped = ratio * advantages
    clipped = ratio.clamp(lo, hi) * advantages
    per_tok = -torch.minimum(unclipped, clipped)
    return (per_tok * mask).sum() / mask.sum().clamp_min(1)


def mis_loss(logp, behavior_logp, advantages, mask, cap=2.0):
    """Truncated importance-sampling REINFORCE: -min(w, cap) * A * logp with w = exp(logp - behavior), w detached."""
    w = torch.exp(logp.detach() - behavior_logp).clamp(max=cap)
    per_tok = -(w * advantages * logp)
    return (per_tok * mask).sum() / mask.sum().clamp_min(1)
