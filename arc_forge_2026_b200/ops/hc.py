"""Hyper-connections in the serving forward: the branch stream ``h [N, G, H]`` replaces the single residual.

Each sub-layer (attention / GDN, then the MoE) reads one mixed input from the G branches and writes its output back
to every branch with a per-branch gate (the reference's HC read ``hc_mix.py:117`` / ``gated_residual_forward:204``,
its ``hc_gate`` kernel ``runtime/patches/sglang-0.5.20/0006-qwen4-mnnvl-hc.patch:408-541`` and the write-back
epilogue of the same patch ``:27-50``):

    zb   = rmsnorm_g(h) * (1 + w)                 grouped over the G branches      (kernel hc_norm)
    du   = zb @ [W_down; W_inject; 0]^T            one GEMM for the low-rank path and the gate logits
    pre  = silu(du[:, :R] / 4) @ W_up^T
    x    = mean_g(sigmoid(pre) * zb)               the sub-layer input              (kernel hc_mix)
    gate = 2 sigmoid(du[:, R:R+G] / 4)
    h   += y * gate                                the write-back, in place         (kernel hc_inject)

The gate logits ride in the down-projection GEMM (rows R..R+G of the stacked weight, padded with zero rows to a
multiple of 8 for the GEMM's alignment), so the separate gate kernel of the reference's serving patch disappears.
No all-reduce precedes the write-back in this design: attention is data-parallel over sessions, so the
sub-layer output is already complete on its rank.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import C

_BF = torch.bfloat16


@dataclass
class HCWeights:
    norm_w: torch.Tensor   # fp32 [G*H]
    wcat: torch.Tensor     # bf16 [ceil8(R + G), G*H]: W_down rows, then W_inject rows, then zero rows
    w_up: torch.Tensor     # bf16 [G*H, R]
    rank: int
    inject: bool
    eps: float

    @classmethod
    def from_tensors(cls, norm_w, w_down, w_up, w_inject, eps: float, device) -> "HCWeights":
        dev = torch.device(device)
        R, GH = w_down.shape
        G = 0 if w_inject is None else w_inject.shape[0]
        rows = (R + G + 7) // 8 * 8
        wcat = torch.zeros(rows, GH, dtype=_BF, device=dev)
        wcat[:R] = w_down.detach().to(dev, _BF)
        if w_inject is not None:
            wcat[R:R + G] = w_inject.detach().to(dev, _BF)
        return cls(norm_w.detach().float().to(dev).contiguous(), wcat, w_up.detach().to(dev, _BF).contiguous(), R,
                   w_inject is not None, float(eps))

    @classmethod
    def from_module(cls, mod, device) -> "HCWeights":
        """From a ``models.reference.HyperConnection``."""
        return cls.from_tensors(mod.hc_norm.weight, mod.w_down, mod.w_up, mod.w_inject, mod.eps, device)

    @classmethod
    def random(cls, G: int, H: int, R: int, std: float, eps: float, inject: bool, gen, device) -> "HCWeights":
        dev = torch.device(device)

        def rn(*s):
            return torch.randn(*s, generator=gen, device=dev) * std
        return cls.from_tensors(torch.zeros(G * H, device=dev), rn(R, G * H), rn(G * H, R),
                                rn(G, G * H) if inject else None, eps, dev)


def hc_read(h: torch.Tensor, w: HCWeights, G: int) -> tuple[torch.Tensor, torch.Tensor | None]:
    """h [N, G, H] bf16 -> (x [N, H] bf16, gate [N, G] bf16 or None for the final readout)."""
    N, _, H = h.shape
    c = C()
    zb = torch.empty(N, G, H, dtype=_BF, device=h.device)
    rstd = torch.empty(N, G, dtype=torch.float32, device=h.device)
    c.hc_norm(h, w.norm_w, w.eps, zb, rstd, None, None)
    du = c.gemm(zb.view(N, G * H), w.wcat)
    s = torch.empty(N, w.rank, dtype=_BF, device=h.device)
    gate = torch.empty(N, G, dtype=_BF, device=h.device) if w.inject else None
    c.hc_act(du, w.rank, G, s, gate)  # s = silu(du_down / 4), gate = 2 sigmoid(du_inject / 4)
    pre = c.gemm(s, w.w_up)
    x = torch.empty(N, H, dtype=_BF, device=h.device)
    c.hc_mix(pre, zb, x, None, None, None)
    return x, gate


def hc_inject_(h: torch.Tensor, y: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """h[n, g, :] += y[n, :] * gate[n, g] in place (each element is read and written by the same thread)."""
    C().hc_inject(h, y, gate, h, None, None, None)
    return h
