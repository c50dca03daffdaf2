"""GPTQ INT3 group-128 quantisation of routed experts (symmetric uint3, zero 4, signed bf16 scales).

The quantiser contract is the reference's (``training/work/qwen38fn_eval/gptq_int3.py:1-14,31-73``):

* codes ``q`` in ``0..7``, dequant ``(q - 4) * scale``; the grid ``[-4, 3] * scale`` is asymmetric, so both
  signs of the scale are tried and the one with the lower error kept;
* the scale is rounded to bf16 before any code is chosen (what the serving pack stores);
* the scale is searched on a clipping grid (``grid`` steps down to ``maxshrink``) minimising
  ``sum |dq - w|^norm`` with ``norm = 2.4``;
* the group equals the 128-column GPTQ block, so a group's scale is fixed from the block-start weights
  after the error feedback of earlier blocks.

The error-feedback loop is the textbook GPTQ of Frantar et al. (2022): Cholesky factor of the damped inverse
Hessian, per-column quantise, propagate ``err / d`` along the row inside the block, then a GEMM to the
columns after the block. This module is plain torch (CPU or GPU), batched over experts.
"""
from __future__ import annotations

import torch

GROUP = 128
MAXQ = 7
HALF = 4


def _qdq(x, scale, zero):
    q = torch.clamp(torch.round(x / scale) + zero, 0, MAXQ)
    return q, (q - zero) * scale


@torch.no_grad()
def find_scales(w: torch.Tensor, grid: int = 100, maxshrink: float = 0.8, norm: float = 2.4, mse: bool = True,
                scale_dtype=torch.bfloat16) -> torch.Tensor:
    """Best signed scale per row of ``w`` ([..., GROUP]) for the symmetric uint3 grid; fp32 values that are
    exactly representable in ``scale_dtype``."""
    w = w.float()
    lo = w.amin(-1).clamp_max(0)
    hi = w.amax(-1).clamp_min(0)
    best_err, best = None, None
    for sign in (1.0, -1.0):
        steps = int(maxshrink * grid) if mse else 1
        for i in range(steps):
            p = 1.0 - i / grid
            a, b = p * lo, p * hi
            if sign > 0:  # long end (-4) on the negative side
                mag = torch.maximum(-a / HALF, b / (HALF - 1))
            else:  # negative scale puts the long end on the positive side
                mag = torch.maximum(b / HALF, -a / (HALF - 1))
            s = (sign * mag.clamp_min(1e-8)).to(scale_dtype).float()
            _, dq = _qdq(w, s[..., None], HALF)
            err = (dq - w).abs().pow(norm).sum(-1)
            if best is None:
                best_err, best = err, s
            else:
                better = err < best_err
                best_err = torch.where(better, err, best_err)
                best = torch.where(better, s, best)
    return best


@torch.no_grad()
def rtn_quantize(w: torch.Tensor, **kw):
    """Round-to-nearest with the searched scales (the fallback for experts that saw no tokens).
    w [..., O, I] -> codes uint8 [..., O, I], scales fp32 [..., O, I/128]."""
    *lead, o, i = w.shape
    g = w.float().reshape(*lead, o, i // GROUP, GROUP)
    s = find_scales(g, **kw)
    q, _ = _qdq(g, s[..., None], HALF)
    return q.reshape(*lead, o, i).to(torch.uint8), s


@torch.no_grad()
def gptq_quantize(w: torch.Tensor, H: torch.Tensor, damp: float = 0.01, **kw):
    """GPTQ one weight matrix (or a batch [E, O, I] with Hessians [E, I, I]).

    Returns (codes uint8 [..., O, I], scales fp32 [..., O, I/128]) with scales exactly bf16-representable.
    """
    if w.dim() == 3:
        outs = [gptq_quantize(w[e], H[e], damp, **kw) for e in range(w.shape[0])]
        return torch.stack([o[0] for o in outs]), torch.stack([o[1] for o in outs])
    W = w.float().clone()
    O, I = W.shape
    if I % GROUP:
        raise ValueError(f"GPTQ group 128 needs the input dim to be a multiple of 128, got {I}")
    Hm = H.double().clone()
    dead = torch.diag(Hm) == 0
    Hm[dead, dead] = 1.0
    W[:, dead] = 0.0
    Hm += damp * torch.mean(torch.diag(Hm)) * torch.eye(I, dtype=Hm.dtype, device=Hm.device)
    L = torch.linalg.cholesky(Hm)
    Hinv = torch.cholesky_inverse(L)
    U = torch.linalg.cholesky(Hinv, upper=True).float()
    codes = torch.zeros(O, I, dtype=torch.uint8, device=W.device)
    scales = torch.zeros(O, I // GROUP, dtype=torch.float32, device=W.device)
    for i1 in range(0, I, GROUP):
        i2 = i1 + GROUP
        W1 = W[:, i1:i2].clone()
        E1 = torch.zeros_like(W1)
        s = find_scales(W1, **kw)
        scales[:, i1 // GROUP] = s
        Ub = U[i1:i2, i1:i2]
        for j in range(GROUP):
            col = W1[:, j]
            q, dq = _qdq(col, s, HALF)
            codes[:, i1 + j] = q.to(torch.uint8)
            err = (col - dq) / Ub[j, j]
            W1[:, j:] -= err[:, None] * Ub[j, j:][None, :]
            E1[:, j] = err
        W[:, i2:] -= E1 @ U[i1:i2, i2:]
    return codes, scales


def hessian(x: torch.Tensor) -> torch.Tensor:
    """GPTQ Hessian 2/n * X^T X of calibration rows x [n, I] (fp64 accumulation)."""
    xd = x.double()
    return 2.0 * (xd.t() @ xd) / max(1, x.shape[0])


def dequant(codes: torch.Tensor, scales: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    s = scales.float().repeat_interleave(GROUP, dim=-1)
    return ((codes.float() - HALF) * s).to(dtype)
