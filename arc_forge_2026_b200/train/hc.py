"""Hyper-connection read and write-back as autograd ops over the native kernels of ``csrc/hc.cu`` (the reference's
``training/work/qwen38fn_lora/hc_mix.py`` custom ops ``hc_mix_fwd`` / ``hc_mix_bwd`` and the inject kernels).

``hc_read(h, module)`` -> (x, gate): the mixed sub-layer input and the write-back gate of every branch (gate None for
the final readout); ``hc_inject(h, y, gate)`` -> h + y * gate per branch. The hyper-connection weights are frozen (the
backward forms dX only, as the reference's op does, which raises if one requires a gradient). The two projections
are cuBLAS GEMMs; the norm, the branch mix, the gates and the write-back are one kernel each way. Off the GPU both
fall back to ``models.reference`` (the oracle of the GPU tests).
"""
from __future__ import annotations

import torch

from ..models import reference as R

_BF = torch.bfloat16
_H = (256, 512, 1024, 2048, 2560)


def _ext():
    from ..ops import C
    return C()


class _HCRead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, norm_w, w_down, w_up, w_inject, eps):
        G, H = h.shape[-2], h.shape[-1]
        R_ = w_down.shape[0]
        lead = h.shape[:-2]
        h2 = h.reshape(-1, G, H)
        rows = h2.shape[0]
        zb = torch.empty(rows, G, H, dtype=_BF, device=h.device)
        rstd = torch.empty(rows, G, dtype=torch.float32, device=h.device)
        c = _ext()
        c.hc_norm(h2, norm_w, eps, zb, rstd, None, None)
        # [W_down; W_inject] padded to a multiple of 16 rows: one GEMM gives the low-rank input and the gate logits
        n_out = R_ + (0 if w_inject is None else G)
        wcat = torch.zeros((n_out + 15) // 16 * 16, G * H, dtype=_BF, device=h.device)
        wcat[:R_] = w_down
        if w_inject is not None:
            wcat[R_:n_out] = w_inject
        du = zb.view(rows, G * H) @ wcat.t()                         # [rows, R (+ G) + pad]
        s = torch.empty(rows, R_, dtype=_BF, device=h.device)
        gate = None if w_inject is None else torch.empty(rows, G, dtype=_BF, device=h.device)
        c.hc_act(du, R_, G, s, gate)                                  # silu(du / 4), 2 sigmoid(di / 4)
        pre = s @ w_up.t()                                            # [rows, G*H]
        x = torch.empty(rows, H, dtype=_BF, device=h.device)
        c.hc_mix(pre.contiguous(), zb, x, None, None, None)
        ctx.save_for_backward(h2, norm_w, wcat, w_up, rstd, zb, du, pre)
        ctx.shape, ctx.R, ctx.has_gate = (lead, G, H), R_, w_inject is not None
        return x.view(*lead, H), (gate.view(*lead, G) if gate is not None else None)

    @staticmethod
    def backward(ctx, dx, dgate):
        h2, norm_w, wcat, w_up, rstd, zb, du, pre = ctx.saved_tensors
        if any(ctx.needs_input_grad[1:5]):
            raise RuntimeError("hyper-connection weights must be frozen (the backward forms dX only)")
        (lead, G, H), R_ = ctx.shape, ctx.R
        rows = h2.shape[0]
        c = _ext()
        dx = (torch.zeros(rows, H, dtype=_BF, device=h2.device) if dx is None
              else dx.reshape(rows, H).to(_BF).contiguous())
        dpre = torch.empty(rows, G * H, dtype=_BF, device=h2.device)
        dzb = torch.empty(rows, G, H, dtype=torch.float32, device=h2.device)
        c.hc_mix(pre.contiguous(), zb, dx, dx, dpre, dzb)
        ds = dpre @ w_up                                              # [rows, R]
        v = du[:, :R_].float() * 0.25
        sv = torch.sigmoid(v)
        ddu = torch.zeros_like(du, dtype=torch.float32)
        ddu[:, :R_] = ds.float() * sv * (1.0 + v * (1.0 - sv)) * 0.25
        if ctx.has_gate and dgate is not None:
            sg = torch.sigmoid(du[:, R_:R_ + G].float() * 0.25)
            ddu[:, R_:R_ + G] = dgate.reshape(rows, G).float() * 2.0 * sg * (1.0 - sg) * 0.25
        dzb += (ddu.to(_BF) @ wcat).float().view(rows, G, H)
        dh = torch.empty_like(h2)
        c.hc_norm(h2, norm_w, 0.0, dh, rstd, dzb, dh)
        return dh.view(*lead, G, H), None, None, None, None, None


class _HCInject(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, y, gate):
        G, H = h.shape[-2], h.shape[-1]
        out = torch.empty_like(h)
        _ext().hc_inject(h, y.contiguous(), gate.contiguous(), out, None, None, None)
        ctx.save_for_backward(y, gate)
        ctx.GH = (G, H)
        return out

    @staticmethod
    def backward(ctx, dout):
        y, gate = ctx.saved_tensors
        dout = dout.to(_BF).contiguous()
        dy = torch.empty_like(y)
        dgate = torch.empty(gate.shape, dtype=torch.float32, device=gate.device)
        _ext().hc_inject(dout, y.contiguous(), gate.contiguous(), dout, dout, dy, dgate)
        return dout, dy, dgate.to(gate.dtype)


def _native(h) -> bool:
    return h.is_cuda and h.dtype == _BF and h.is_contiguous() and h.shape[-1] in _H and h.shape[-2] <= 8


def hc_read(h: torch.Tensor, mod) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``mod``: a ``models.reference.HyperConnection`` (or anything with its weight attributes)."""
    from . import kernels
    if kernels.use("hc") and _native(h):
        kernels.hit("hc", True)
        bf = _BF
        return _HCRead.apply(h, mod.hc_norm.weight.detach().float().contiguous(), mod.w_down.detach().to(bf),
                             mod.w_up.detach().to(bf), None if mod.w_inject is None else mod.w_inject.detach().to(bf),
                             mod.eps)
    if h.is_cuda:
        kernels.hit("hc", False)
    return mod(h)


def hc_inject(h: torch.Tensor, y: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    if _native(h) and y.dtype == _BF:
        return _HCInject.apply(h, y, gate.to(_BF))
    return R.hc_inject(h, y, gate)
