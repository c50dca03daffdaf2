"""Routed-expert MoE block on the native kernels, plus the oracle of its numerics.

Per MoE layer (one launch each, all on the current stream, no host sync):

1. router GEMM (tcgen05, fp32 out) over ``[W_router; w_shared_gate; 0-pad]`` -- the shared-expert gate logit rides
   along as column E;
2. softmax + top-k + renormalise (one warp per token);
3. stable counting sort of the (token, slot) entries by expert;
4. gather + e4m3 quantisation of the routed rows, one scale per (row, 128 columns);
5. INT3 w13 GEMM with SwiGLU and e4m3 requantisation fused in its epilogue;
6. INT3 w2 GEMM with the routing weight fused in its epilogue;
7. shared expert (two dense GEMMs + SwiGLU);
8. combine: residual + sigmoid(gate) * shared + sum of the k routed rows, in a fixed order.

``moe_reference`` computes the same contract in fp32 PyTorch (activations quantised per 128-group to e4m3,
weights (code - 4) * scale, group partial sums scaled in fp32).
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


SEG_PAD = 8  # expert segments start on multiples of 8 rows (16-byte bulk copies of per-row scales)


class MoEWorkspace:
    """Preallocated buffers for up to ``max_tokens`` tokens (stable addresses for CUDA graphs)."""

    def __init__(self, max_tokens: int, E: int, k: int, H: int, I: int, Is: int, device):
        R = max_tokens * k + (SEG_PAD - 1) * E  # routed rows + per-expert segment padding
        self.k, self.E = k, E
        dev = torch.device(device)
        i32 = dict(dtype=torch.int32, device=dev)
        self.logits = torch.empty(max_tokens, E + 8, dtype=torch.float32, device=dev)
        self.ids = torch.empty(max_tokens, k, **i32)
        self.weights = torch.empty(max_tokens, k, dtype=torch.float32, device=dev)
        self.offsets = torch.empty(E + 1, **i32)
        self.row_token = torch.empty(R, **i32)
        self.row_entry = torch.empty(R, **i32)
        self.entry_row = torch.empty(max_tokens * k, **i32)
        self.rows = R
        self.xq = torch.empty(R, H, dtype=torch.float8_e4m3fn, device=dev)
        ld = (R + 32 + 3) // 4 * 4  # +32: chunk over-read slack; multiple of 4 for 16-byte bulk copies
        self.xs = torch.zeros(H // 128, ld, dtype=torch.float32, device=dev)
        self.hq = torch.empty(R, I, dtype=torch.float8_e4m3fn, device=dev)
        self.hs = torch.zeros(I // 128, ld, dtype=torch.float32, device=dev)
        self.y = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
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
    c.router_topk(logits, E, k, renorm, ids, w)
    R = n + (SEG_PAD - 1) * E
    c.expert_sort(ids, E, None, ws.offsets, ws.row_token[:R], ws.row_entry[:R], ws.entry_row[:n], SEG_PAD)
    # rows actually used = offsets[E] (device scalar): the launch covers the capacity, the kernel stops early
    c.quant_rows_e4m3(x, ws.row_token[:R], ws.offsets[E:], R, ws.xq[:R], ws.xs, True)
    c.moe_int3_gemm(bank.w13_codes, bank.w13_scales, ws.offsets, ws.xq[:R], ws.xs, True, ws.hq[:R], ws.hs, None,
                    None, None)
    c.moe_int3_gemm(bank.w2_codes, bank.w2_scales, ws.offsets, ws.hq[:R], ws.hs, False, None, None, ws.y[:R],
                    w.view(-1), ws.row_entry[:R])
    c.gemm(x, shared_w13, out=ws.sh_gu[:T])
    c.swiglu(ws.sh_gu[:T], ws.sh_h[:T])
    c.gemm(ws.sh_h[:T], shared_w2, out=ws.sh_out[:T])
    out = torch.empty_like(x) if out is None else out
    c.moe_combine(ws.y[:R], ws.entry_row[:n], k, ws.sh_out[:T], logits, E, resid, out)
    return out


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
    out = torch.zeros_like(xf)
    for e in torch.unique(ids).tolist():
        tok, slot = (ids == e).nonzero(as_tuple=True)
        xq, xs = fp8q.quantize_act_groups(x[tok].float())
        xd = fp8q.dequant_act_groups(xq, xs)
        h = xd @ w13[e].t()
        hh = F.silu(h[:, :I]) * h[:, I:]
        hq, hs = fp8q.quantize_act_groups(hh)
        y = fp8q.dequant_act_groups(hq, hs) @ w2[e].t()
        out.index_add_(0, tok, y * w[tok, slot][:, None])
    sh = (F.silu(xf @ shared_w13.float()[: shared_w13.shape[0] // 2].t()) *
          (xf @ shared_w13.float()[shared_w13.shape[0] // 2:].t())) @ shared_w2.float().t()
    sg = torch.sigmoid(logits[:, E:E + 1])
    return resid.float() + out + sg * sh
