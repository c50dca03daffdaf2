"""Routed-expert MoE block on the native kernels, plus the oracle of its numerics.

Per MoE layer (one launch each, all on the current stream, no host sync):

1. router GEMM (tcgen05, fp32 out) over ``[W_router; w_shared_gate; 0-pad]`` -- the shared-expert gate logit rides
   along as column E;
2. softmax + top-k + renormalise (one warp per token);
   (the same kernel appends every (token, slot) entry to its expert's list: no sort);
3. e4m3 quantisation of each token row, one scale per row (the reference's W3A8 activation rule:
   s = max(amax, 1e-30) / 448, ``training/work/qwen38fn_lora/int3_moe.py:1-14,108-118``);
5. INT3 w13 GEMM over each expert's listed entries (rows gathered inside the kernel) with SwiGLU fused in its
   epilogue, h stored bf16 per entry;
6. per-row e4m3 quantisation of h;
7. INT3 w2 GEMM with the routing weight fused in its epilogue, y per entry;
8. shared expert (two dense GEMMs + SwiGLU);
9. combine: residual + sigmoid(gate) * shared + sum of the k routed rows of each token, in slot order.

Block-FP8 experts (the QAD teacher) keep the block-FP8 contract instead: 1 x 128 activation scales for both GEMMs
and the w13 epilogue's e4m3-per-128 SwiGLU output.

``moe_reference`` computes the same contracts in fp32 PyTorch (weights (code - 4) * scale with group partial sums
scaled in fp32; activations per row, h rounded to bf16 before its quantisation).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..quant import fp8 as fp8q
from ..quant.int3_tiles import codes_to_tiles, scales_to_tiles, tiles_to_codes, tiles_to_scales
from ._ext import C


@dataclass
class Int3ExpertBank:
    """One layer's routed experts in the kernel tile layout."""
    w13_codes: torch.Tensor   # int32 [E, 2I/128, H/128, 128, 12]
    w13_scales: torch.Tensor  # bf16  [E, 2I/128, H/128, 128]
    w2_codes: torch.Tensor    # int32 [E, H/128, I/128, 128, 12]
    w2_scales: torch.Tensor   # bf16  [E, H/128, I/128, 128]

    @property
    def num_experts(self) -> int:
        return self.w13_codes.shape[0]

    @property
    def hidden(self) -> int:
        return self.w13_codes.shape[2] * 128

    @property
    def inter(self) -> int:
        return self.w2_codes.shape[2] * 128

    @classmethod
    def from_codes(cls, w13_codes, w13_scales, w2_codes, w2_scales, device=None):
        t = cls(codes_to_tiles(w13_codes), scales_to_tiles(w13_scales), codes_to_tiles(w2_codes),
                scales_to_tiles(w2_scales))
        return t.to(device) if device is not None else t

    @classmethod
    def random(cls, E: int, H: int, I: int, device, seed: int = 0, scale_std: float = 0.02 / 2.3):
        """Random codes and bf16 scales (a random-init model's experts: weights ~ N(0, 0.02) after dequant)."""
        g = torch.Generator(device="cpu").manual_seed(seed)
        w13_codes = torch.randint(0, 8, (E, 2 * I, H), generator=g, dtype=torch.uint8)
        w2_codes = torch.randint(0, 8, (E, H, I), generator=g, dtype=torch.uint8)
        w13_s = (torch.randn(E, 2 * I, H // 128, generator=g) * scale_std).to(torch.bfloat16)
        w2_s = (torch.randn(E, H, I // 128, generator=g) * scale_std).to(torch.bfloat16)
        return cls.from_codes(w13_codes, w13_s, w2_codes, w2_s, device)

    def to(self, device):
        return Int3ExpertBank(*(t.to(device) for t in (self.w13_codes, self.w13_scales, self.w2_codes,
                                                          self.w2_scales)))

    def dequant(self, dtype=torch.float32):
        """(w13 [E, 2I, H], w2 [E, H, I]) = (code - 4) * scale."""
        def dq(codes, scales):
            c = tiles_to_codes(codes).float() - 4.0
            return (c * tiles_to_scales(scales).float().repeat_interleave(128, -1)).to(dtype)
        return dq(self.w13_codes, self.w13_scales), dq(self.w2_codes, self.w2_scales)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.w13_codes, self.w13_scales, self.w2_codes,
                                                          self.w2_scales))


@dataclass
class Fp8ExpertBank:
    """One layer's routed experts in block FP8 (the teacher's format): e4m3 weights and one fp32 scale per 128 x 128
    block (``weight_scale_inv``). The expert kernels take it in place of an ``Int3ExpertBank``."""
    w13_codes: torch.Tensor   # e4m3 [E, 2I, H]
    w13_scales: torch.Tensor  # fp32 [E, 2I/128, H/128]
    w2_codes: torch.Tensor    # e4m3 [E, H, I]
    w2_scales: torch.Tensor   # fp32 [E, H/128, I/128]

    @property
    def num_experts(self) -> int:
        return self.w13_codes.shape[0]

    @property
    def hidden(self) -> int:
        return self.w13_codes.shape[2]

    @property
    def inter(self) -> int:
        return self.w2_codes.shape[2]

    @classmethod
    def from_weights(cls, w13: torch.Tensor, w2: torch.Tensor, device=None):
        """Block-quantise fp32/bf16 expert weights [E, 2I, H] / [E, H, I]."""
        def q(w):
            qs = [fp8q.quantize_weight_block(w[e].float()) for e in range(w.shape[0])]
            return torch.stack([a for a, _ in qs]), torch.stack([b for _, b in qs])
        a, sa = q(w13)
        b, sb = q(w2)
        t = cls(a, sa.float(), b, sb.float())
        return t.to(device) if device is not None else t

    def to(self, device):
        return Fp8ExpertBank(*(t.to(device) for t in (self.w13_codes, self.w13_scales, self.w2_codes,
                                                         self.w2_scales)))

    def dequant(self, dtype=torch.float32):
        def dq(w, s):
            return torch.stack([fp8q.dequant_weight_block(w[e], s[e]) for e in range(w.shape[0])]).to(dtype)
        return dq(self.w13_codes, self.w13_scales), dq(self.w2_codes, self.w2_scales)


class MoEWorkspace:
    """Preallocated buffers for up to ``max_tokens`` tokens (stable addresses for CUDA graphs). Routed rows are
    numbered by entry (token * k + slot)."""

    def __init__(self, max_tokens: int, E: int, k: int, H: int, I: int, Is: int, device):
        n = max_tokens * k
        self.k, self.E, self.rows = k, E, n
        dev = torch.device(device)
        i32 = dict(dtype=torch.int32, device=dev)
        self.logits = torch.empty(max_tokens, E + 8, dtype=torch.float32, device=dev)
        self.ids = torch.empty(max_tokens, k, **i32)
        self.weights = torch.empty(max_tokens, k, dtype=torch.float32, device=dev)
        self.cnt = torch.zeros(E, **i32)                 # entries per expert (the router fills both)
        self.list = torch.zeros(E, max_tokens, **i32)    # each expert's entries
        self.xq = torch.empty(max_tokens, H, dtype=torch.float8_e4m3fn, device=dev)
        self.xs = torch.zeros(max_tokens, dtype=torch.float32, device=dev)   # INT3: one scale per token row
        self.h = torch.empty(n, I, dtype=torch.bfloat16, device=dev)         # INT3: w13 output (SwiGLU, bf16)
        self.hq = torch.empty(n, I, dtype=torch.float8_e4m3fn, device=dev)
        self.hs = torch.zeros(n, dtype=torch.float32, device=dev)
        # block-FP8 experts: 1 x 128 activation scales, group-major
        self.xs_g = torch.zeros(H // 128, max_tokens, dtype=torch.float32, device=dev)
        self.hs_g = torch.zeros(I // 128, n, dtype=torch.float32, device=dev)
        self.y = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        self.sh_gu = torch.empty(max_tokens, 2 * Is, dtype=torch.bfloat16, device=dev)
        self.sh_h = torch.empty(max_tokens, Is, dtype=torch.bfloat16, device=dev)
        self.sh_out = torch.empty(max_tokens, H, dtype=torch.bfloat16, device=dev)


def router_weight_with_shared_gate(router_w: torch.Tensor, shared_gate_w: torch.Tensor) -> torch.Tensor:
    """[E, H] router + [1, H] shared-expert gate -> [E + 8, H] (rows E+1.. are zero padding)."""
    E, H = router_w.shape
    out = torch.zeros(E + 8, H, dtype=torch.bfloat16, device=router_w.device)
    out[:E] = router_w
    out[E] = shared_gate_w.reshape(H)
    return out


def moe_forward(x: torch.Tensor, resid: torch.Tensor, router_ext: torch.Tensor, bank: Int3ExpertBank,
                shared_w13: torch.Tensor, shared_w2: torch.Tensor, k: int, ws: MoEWorkspace,
                out: torch.Tensor | None = None, renorm: bool = True) -> torch.Tensor:
    """x [T, H] (normed input), resid [T, H] -> out = resid + MoE(x). All bf16."""
    c = C()
    T, H = x.shape
    E = bank.num_experts
    n = T * k
    logits = ws.logits[:T]
    c.gemm(x, router_ext, out=logits, out_fp32=True)
    ids, w = ws.ids[:T], ws.weights[:T]
    c.router_topk(logits, E, k, renorm, ids, w, ws.cnt, ws.list)
    expert_gemms(c, bank, ws, x, T, w.view(-1))
    c.gemm(x, shared_w13, out=ws.sh_gu[:T])
    c.swiglu(ws.sh_gu[:T], ws.sh_h[:T])
    c.gemm(ws.sh_h[:T], shared_w2, out=ws.sh_out[:T])
    out = torch.empty_like(x) if out is None else out
    c.moe_combine(ws.y[:n], None, k, ws.sh_out[:T], logits, E, resid, out)
    return out


def expert_gemms(c, bank, ws, x, T, route_w):
    """The listed entries of ``T`` tokens -> w13 -> w2 on the native kernels; y rows per entry."""
    k = ws.k
    n = T * k
    if isinstance(bank, Fp8ExpertBank):
        c.quant_rows_e4m3(x, None, None, T, ws.xq[:T], ws.xs_g, True)
        c.moe_int3_gemm(bank.w13_codes, bank.w13_scales, ws.cnt, ws.list, k, ws.xq[:T], ws.xs_g, True, ws.hq[:n],
                        ws.hs_g, None, None)
        c.moe_int3_gemm(bank.w2_codes, bank.w2_scales, ws.cnt, ws.list, 1, ws.hq[:n], ws.hs_g, False, None, None,
                        ws.y[:n], route_w)
        return
    c.quant_rows_e4m3_row(x, None, None, T, ws.xq[:T], ws.xs)
    c.moe_int3_gemm(bank.w13_codes, bank.w13_scales, ws.cnt, ws.list, k, ws.xq[:T], ws.xs, True, None, None,
                    ws.h[:n], None)
    c.quant_rows_e4m3_row(ws.h[:n], None, None, n, ws.hq[:n], ws.hs)
    c.moe_int3_gemm(bank.w2_codes, bank.w2_scales, ws.cnt, ws.list, 1, ws.hq[:n], ws.hs, False, None, None,
                    ws.y[:n], route_w)


def moe_reference(x, resid, router_ext, bank: Int3ExpertBank, shared_w13, shared_w2, k, renorm=True):
    """fp32 oracle of :func:`moe_forward` (same W3A8 contract, same fp8 activation quantisation)."""
    xf = x.float()
    E = bank.num_experts
    logits = xf @ router_ext.float().t()
    probs = torch.softmax(logits[:, :E], -1)
    w, ids = torch.topk(probs, k, -1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    w13, w2 = bank.dequant(torch.float32)
    I = bank.inter
    fp8_bank = isinstance(bank, Fp8ExpertBank)

    def q(a):  # the activation quantisation of each contract, returned dequantised
        if fp8_bank:
            aq, s_ = fp8q.quantize_act_groups(a)
            return fp8q.dequant_act_groups(aq, s_)
        aq, s_ = fp8q.quantize_rows(a)
        return aq.float() * s_[:, None]

    out = torch.zeros_like(xf)
    for e in torch.unique(ids).tolist():
        tok, slot = (ids == e).nonzero(as_tuple=True)
        h = q(x[tok].float()) @ w13[e].t()
        hh = F.silu(h[:, :I]) * h[:, I:]
        if not fp8_bank:
            hh = hh.bfloat16().float()  # the server stores the SwiGLU output in bf16 before quantising it
        y = q(hh) @ w2[e].t()
        out.index_add_(0, tok, y * w[tok, slot][:, None])
    sh = (F.silu(xf @ shared_w13.float()[: shared_w13.shape[0] // 2].t()) *
          (xf @ shared_w13.float()[shared_w13.shape[0] // 2:].t())) @ shared_w2.float().t()
    sg = torch.sigmoid(logits[:, E:E + 1])
    return resid.float() + out + sg * sh
