"""Fused training ops of the QAD student (``csrc/train_fused.cu``): one kernel each way instead of a chain of
PyTorch element-wise ops, bf16 in and out with fp32 math, fixed-order reductions.

Each function takes the student's tensors as they are (strided views included) and falls back to the plain-torch
math of ``models.reference`` off the GPU, or when a shape is outside what the kernels cover; the CPU paths are the
oracles the GPU tests compare against. The reference's counterparts are its fused Triton training kernels
(``training/work/qwen38fn_lora/trainer_kernels.py:234-290`` GatedRMSNormFLA, ``int3_moe.py:108-152,376-430``
SwiGLU and token aggregation, ``fp8_moe.py`` _swiglu_backward / _routing_backward).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..models import reference as R
from . import kernels

_BF = torch.bfloat16
_NORM_H = (128, 256, 512, 1024, 2048)


def _ext():
    from ..ops import C
    return C()


def _gpu_bf16(*ts) -> bool:
    return all(t.is_cuda and t.dtype == _BF and t.stride(-1) == 1 for t in ts)


class _ConvSiLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, pos):
        y = torch.empty(x.shape, dtype=_BF, device=x.device)
        _ext().conv_silu(x, w, y, None, None, pos)
        ctx.save_for_backward(x, w, pos)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, pos = ctx.saved_tensors
        dx = torch.empty(x.shape, dtype=_BF, device=x.device)
        _ext().conv_silu(x, w, dx, dy.to(_BF).contiguous(), dx, pos)
        return dx, None, None


def conv_silu(x: torch.Tensor, w: torch.Tensor, pos: torch.Tensor | None = None) -> torch.Tensor:
    """Causal depthwise conv (kernel 4, zero history) + SiLU over x [B, T, C] (a strided view is fine); frozen w.
    ``pos`` [B, T] (packed sequences): each token's position inside its sequence; taps before the start read 0."""
    if (kernels.use("conv_silu") and _gpu_bf16(x) and x.dim() == 3 and w.shape[-1] == 4 and x.shape[-1] % 8 == 0
            and x.stride(1) % 8 == 0 and x.stride(0) == x.shape[1] * x.stride(1) and not w.requires_grad):
        kernels.hit("conv_silu", True)
        return _ConvSiLU.apply(x, w.float().contiguous(), None if pos is None else pos.int().contiguous())
    if x.is_cuda:
        kernels.hit("conv_silu", False)
    if pos is None:
        return R.causal_conv1d(x, w)[0]
    return conv_silu_reference(x, w, pos)


def conv_silu_reference(x, w, pos):
    """Plain-torch causal conv + SiLU with per-token sequence positions (the packed-sequence oracle)."""
    B, T, Cc = x.shape
    K = w.shape[1]
    xf = x.float()
    pre = torch.zeros(B, T, Cc, dtype=torch.float32, device=x.device)
    for k in range(K):
        lag = K - 1 - k
        if lag >= T:
            continue
        shifted = torch.zeros_like(xf)
        shifted[:, lag:] = xf[:, : T - lag]
        live = (pos >= lag).to(xf.dtype)[..., None]
        pre = pre + w[:, k].float() * shifted * live
    return F.silu(pre).to(x.dtype)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, z):
        H = x.shape[-1]
        y = torch.empty(x.shape, dtype=_BF, device=x.device)
        rstd = torch.empty(x.numel() // H, dtype=torch.float32, device=x.device)
        _ext().rmsnorm_train(x, z, w, eps, y, rstd, None, None, None)
        ctx.save_for_backward(x, w, rstd, z)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd, z = ctx.saved_tensors
        dx = torch.empty(x.shape, dtype=_BF, device=x.device)
        dz = torch.empty(z.shape, dtype=_BF, device=x.device) if z is not None else None
        _ext().rmsnorm_train(x, z, w, ctx.eps, dx, rstd, dy.to(_BF).contiguous(), dx, dz)
        return dx, None, None, dz


def _norm_ok(x, w) -> bool:
    return _gpu_bf16(x) and x.shape[-1] in _NORM_H and x.dim() >= 2 and not w.requires_grad


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Zero-centred RMSNorm ``x / rms(x) * (1 + w)`` (frozen w) of ``models.reference.rms_norm``."""
    if kernels.use("rms_norm") and _norm_ok(x, w):
        kernels.hit("rms_norm", True)
        return _RMSNorm.apply(x, w.float().contiguous(), eps, None)
    if x.is_cuda:
        kernels.hit("rms_norm", False)
    return R.rms_norm(x, w, eps)


def gated_rms_norm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """GDN output norm ``x / rms(x) * w * silu(z)`` (frozen w) of ``models.reference.gated_rms_norm``."""
    if kernels.use("gated_rms_norm") and _norm_ok(x, w) and _gpu_bf16(z) and z.shape == x.shape:
        kernels.hit("gated_rms_norm", True)
        return _RMSNorm.apply(x, w.float().contiguous(), eps, z)
    if x.is_cuda:
        kernels.hit("gated_rms_norm", False)
    return R.gated_rms_norm(x, z, w, eps)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        I = gu.shape[-1] // 2
        h = torch.empty(*gu.shape[:-1], I, dtype=_BF, device=gu.device)
        _ext().swiglu_train(gu, h, None)
        ctx.save_for_backward(gu)
        return h

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        dgu = torch.empty_like(gu)
        _ext().swiglu_train(gu, dgu, dh.to(_BF).contiguous())
        return dgu


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` of ``gu = [gate | up]`` along the last dim."""
    I = gu.shape[-1] // 2
    if kernels.use("swiglu") and _gpu_bf16(gu) and gu.is_contiguous() and I % 8 == 0:
        kernels.hit("swiglu", True)
        return _SwiGLU.apply(gu)
    if gu.is_cuda:
        kernels.hit("swiglu", False)
    return F.silu(gu[..., :I].float()).to(gu.dtype) * gu[..., I:]


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, inv, w):
        out = torch.empty(w.shape[0], y.shape[1], dtype=_BF, device=y.device)
        _ext().moe_combine_train(y, inv, w, out, None, None, None)
        ctx.save_for_backward(y, inv, w)
        return out

    @staticmethod
    def backward(ctx, dout):
        y, inv, w = ctx.saved_tensors
        dy, dw = torch.empty_like(y), torch.empty_like(w)
        _ext().moe_combine_train(y, inv, w, dy, dout.to(_BF).contiguous(), dy, dw)
        return dy, None, dw


def moe_combine(y: torch.Tensor, inv: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """out[t] = sum_k w[t, k] y[inv[t*K + k]]: routed rows (expert order) back to their tokens, weighted."""
    T, K = w.shape
    H = y.shape[-1]
    if kernels.use("moe_combine") and _gpu_bf16(y) and y.is_contiguous() and H in (256, 512, 1024, 2048):
        kernels.hit("moe_combine", True)
        return _Combine.apply(y, inv.contiguous(), w.float().contiguous())
    if y.is_cuda:
        kernels.hit("moe_combine", False)
    yt = y.index_select(0, inv).view(T, K, H)
    return (yt * w.to(yt.dtype)[..., None]).sum(1)


class _Dispatch(torch.autograd.Function):
    """xs = x[order // K] (every token once per routed expert, in expert order); the gradient sums each token's K
    rows through the inverse permutation in one kernel."""

    @staticmethod
    def forward(ctx, x, order, inv, K):
        ctx.save_for_backward(inv)
        ctx.K, ctx.T = K, x.shape[0]
        return x.index_select(0, torch.div(order, K, rounding_mode="floor"))

    @staticmethod
    def backward(ctx, g):
        (inv,) = ctx.saved_tensors
        g = g.to(_BF).contiguous()
        dx = torch.empty(ctx.T, g.shape[-1], dtype=_BF, device=g.device)
        _ext().moe_dispatch_bwd(g, inv, ctx.K, dx)
        return dx, None, None, None


def moe_dispatch(x: torch.Tensor, order: torch.Tensor, inv: torch.Tensor, K: int) -> torch.Tensor:
    if kernels.use("moe_dispatch") and _gpu_bf16(x) and x.shape[-1] in (256, 512, 1024, 2048):
        kernels.hit("moe_dispatch", True)
        return _Dispatch.apply(x, order, inv.contiguous(), K)
    if x.is_cuda:
        kernels.hit("moe_dispatch", False)
    return None
