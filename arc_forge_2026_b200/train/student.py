"""Trainable QAD student: the hybrid MoE with INT3 experts (frozen codes, trainable fp32 group scales), block-FP8 QAT
dense projections, an fp32 router, bf16 shared experts, and frozen norms / embeddings / LM head.

Trainable parameter groups (names of the reference's QAD v2, ``training/work/qwen38fn_qad/train_qad.py:100-126``):
``scale`` (expert w13/w2 scales), ``router``, ``shared`` (shared expert + its gate), ``dense_fp8`` (GDN
in_proj_qkvz / out_proj, attention q/k/v), ``dense_bf16`` (GDN in_proj_ba, attention o_proj). Every trainable
tensor is an fp32 master; the forward computes in bf16 (FP8 QAT weights round-trip through e4m3 128x128 blocks).

Layers are activation-checkpointed (one layer's inputs kept, the rest recomputed in backward) so a 16k-token
sequence fits with the dequantised expert banks of only one layer alive at a time.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn
from torch.utils.checkpoint import checkpoint

from ..config import FULL, ModelConfig
from ..models import reference as R
from ..models.ple import PLELayer
from ..quant.int3_tiles import codes_to_tiles
from . import fused
from .fakequant import fp8_weight, int3_weight
from .hc import hc_inject, hc_read
from .gdn_chunk import chunk_gated_delta_rule

GROUPS = ("scale", "router", "shared", "dense_fp8", "dense_bf16")


def _master(t: torch.Tensor) -> nn.Parameter:
    return nn.Parameter(t.detach().float().clone())


def grouped_linear(x: torch.Tensor, w: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    """x [R, K] rows sorted by expert, w [E, N, K], counts [E] -> [R, N]. CUDA: the grouped tcgen05 GEMM
    (``train/grouped.py``; forward, dX and dW native); CPU: one GEMM per expert."""
    from . import kernels
    if x.is_cuda and kernels.use("grouped_gemm") and x.dtype == torch.bfloat16 and x.shape[1] % 8 == 0 \
            and w.shape[1] % 8 == 0:
        from .grouped import GroupedLinear
        kernels.hit("grouped_gemm", True)
        return GroupedLinear.apply(x, w, counts)
    if x.is_cuda:
        kernels.hit("grouped_gemm", False)
    if x.is_cuda and hasattr(torch, "_grouped_mm"):
        offs = counts.cumsum(0).to(torch.int32)
        return torch._grouped_mm(x, w.transpose(-2, -1), offs=offs)
    outs, o = [], 0
    for e, c in enumerate(counts.tolist()):
        if c:
            outs.append(x[o:o + c] @ w[e].t())
        o += c
    return torch.cat(outs) if outs else x.new_zeros(0, w.shape[1])


class _Dispatch(torch.autograd.Function):
    """xs = x[order // K]: every token once per routed expert, in expert order. The gradient gathers the K copies of
    each token back with the inverse permutation and sums them (no scatter-add)."""

    @staticmethod
    def forward(ctx, x, order, inv, K):
        ctx.save_for_backward(inv)
        ctx.K = K
        return x.index_select(0, torch.div(order, K, rounding_mode="floor"))

    @staticmethod
    def backward(ctx, g):
        (inv,) = ctx.saved_tensors
        return g.index_select(0, inv).view(-1, ctx.K, g.shape[-1]).sum(1), None, None, None


def packed_attention(q, k, v, cu_seqlens, max_seqlen: int):
    """Causal attention inside each segment of a packed row: q [T, Hq, D], k / v [T, Hkv, D] -> [T, Hq, D].
    CUDA: the native tcgen05 varlen kernels (``train/attention.py``: forward, dQ, dK / dV, deterministic), or with
    that fast kernel disabled the library flash-attention varlen kernel with its deterministic backward; otherwise
    one SDPA call per segment."""
    from . import kernels
    if q.is_cuda and q.dtype == torch.bfloat16 and q.shape[-1] in (128, 256):
        native = kernels.use("attention")
        kernels.hit("attention", native)
        if native:
            from .attention import varlen_attention
            return varlen_attention(q, k, v, cu_seqlens)
    if q.is_cuda:
        try:
            from flash_attn import flash_attn_varlen_func
        except ImportError:  # pragma: no cover - the image ships flash_attn
            flash_attn_varlen_func = None
        if flash_attn_varlen_func is not None and q.dtype in (torch.bfloat16, torch.float16):
            cu = cu_seqlens.to(device=q.device, dtype=torch.int32)
            return flash_attn_varlen_func(q.contiguous(), k.contiguous(), v.contiguous(), cu, cu, max_seqlen,
                                          max_seqlen, causal=True, deterministic=True)
    outs = []
    bounds = cu_seqlens.tolist()
    for s0, s1 in zip(bounds[:-1], bounds[1:]):
        o = F.scaled_dot_product_attention(q[s0:s1].transpose(0, 1)[None], k[s0:s1].transpose(0, 1)[None],
                                           v[s0:s1].transpose(0, 1)[None], is_causal=True, enable_gqa=True)
        outs.append(o[0].transpose(0, 1))
    return torch.cat(outs)


class StudentMoE(nn.Module):
    def __init__(self, cfg: ModelConfig, router, w13_codes, w13_scales, w2_codes, w2_scales, shared_gate, shared_up,
                 shared_down, shared_expert_gate):
        super().__init__()
        self.cfg = cfg
        self.router = _master(router)
        self.register_buffer("w13_codes", w13_codes, persistent=True)
        self.register_buffer("w2_codes", w2_codes, persistent=True)
        self.w13_scales = _master(w13_scales)
        self.w2_scales = _master(w2_scales)
        self.shared_w13 = _master(torch.cat([shared_gate, shared_up]))
        self.shared_down = _master(shared_down)
        self.shared_expert_gate = _master(shared_expert_gate)
        self.replay = None  # (RoutingReplay, layer index) when the rollout's expert choices are forced

    def forward(self, x):
        c = self.cfg
        T, H = x.shape
        logits = x.float() @ self.router.t()
        if self.replay is not None:
            rep, index = self.replay
            w, ids = rep.route(index, logits, c.num_experts_per_tok, c.norm_topk_prob)
        else:
            w, ids = R.route(logits, c.num_experts_per_tok, c.norm_topk_prob)
        K = c.num_experts_per_tok
        flat = ids.flatten()
        order = torch.argsort(flat, stable=True)  # (token, k) entries sorted by expert
        inv = torch.empty_like(order)
        inv[order] = torch.arange(order.numel(), device=order.device)
        counts = torch.bincount(flat, minlength=c.num_experts)
        xs = fused.moe_dispatch(x, order, inv, K)
        if xs is None:
            xs = _Dispatch.apply(x, order, inv, K)
        W13 = int3_weight(self.w13_scales, self.w13_codes).to(x.dtype)
        h = fused.swiglu(grouped_linear(xs, W13, counts))
        W2 = int3_weight(self.w2_scales, self.w2_codes).to(x.dtype)
        y = grouped_linear(h, W2, counts)
        # back to (token, k) order, weighted by the router and summed over k
        out = fused.moe_combine(y, inv, w)
        gu = x @ self.shared_w13.to(x.dtype).t()
        sh = fused.swiglu(gu) @ self.shared_down.to(x.dtype).t()
        sg = torch.sigmoid(x.float() @ self.shared_expert_gate.t()).to(x.dtype)
        return out + sg * sh


def layer_tensors_from_reference(L: R.DecoderLayer, codes_scales) -> dict:
    m, moe = L.mixer, L.mlp
    t = dict(in_norm=L.input_layernorm.weight, post_norm=L.post_attention_layernorm.weight)
    if L.kind == FULL:
        t.update(q_proj=m.q_proj.weight, k_proj=m.k_proj.weight, v_proj=m.v_proj.weight, o_proj=m.o_proj.weight,
                 q_norm=m.q_norm.weight, k_norm=m.k_norm.weight)
        if getattr(m, "index_qk_proj", None) is not None:  # QSA indexer (frozen)
            t.update(index_qk_proj=m.index_qk_proj.weight, index_q_norm=m.index_q_norm.weight,
                     index_k_norm=m.index_k_norm.weight)
    else:
        t.update(in_proj_qkvz=m.in_proj_qkvz.weight, in_proj_ba=m.in_proj_ba.weight, out_proj=m.out_proj.weight,
                 conv1d=m.conv1d, A_log=m.A_log, dt_bias=m.dt_bias, g_norm=m.norm)
    c13, s13, c2, s2 = codes_scales
    t.update(router=moe.gate.weight, w13_codes=codes_to_tiles(c13), w13_scales=s13, w2_codes=codes_to_tiles(c2),
             w2_scales=s2, shared_gate=moe.shared_gate_proj.weight, shared_up=moe.shared_up_proj.weight,
             shared_down=moe.shared_down_proj.weight, shared_expert_gate=moe.shared_expert_gate.weight)
    out = {k: v.detach() for k, v in t.items()}
    if getattr(L, "ple", None) is not None:  # per-layer n-gram embedding (frozen)
        out["ple"] = {k: v.detach() for k, v in L.ple.state_dict().items()}
    if getattr(L, "hc", False):  # hyper-connection weights (frozen)
        out["hc_attn"] = {k: v.detach() for k, v in L.hc_attn.state_dict().items()}
        out["hc_mlp"] = {k: v.detach() for k, v in L.hc_mlp.state_dict().items()}
    return out


def random_hc_tensors(cfg: ModelConfig, device, gen, inject: bool = True) -> dict:
    G, H, R_ = cfg.hc_count, cfg.hidden_size, cfg.hc_lowrank
    std = cfg.init_std
    t = {"hc_norm.weight": torch.zeros(G * H, device=device),
         "w_down": torch.randn(R_, G * H, generator=gen, device=device) * std,
         "w_up": torch.randn(G * H, R_, generator=gen, device=device) * std}
    if inject:
        t["w_inject"] = torch.randn(G, G * H, generator=gen, device=device) * std
    return t


def _hc_module(cfg, state: dict, inject: bool, device):
    m = R.HyperConnection(cfg, inject=inject)
    m.load_state_dict({k: v.float() for k, v in state.items()})
    return m.to(device).requires_grad_(False)


def random_layer_tensors(cfg: ModelConfig, kind: str, device, gen: torch.Generator) -> dict:
    """Random weights of one layer made on the device (INT3 codes as random tile words: every bit pattern is valid)."""
    std = cfg.init_std
    H = cfg.hidden_size

    def rn(*shape, s=std):
        return torch.randn(*shape, generator=gen, device=device) * s
    t = dict(in_norm=torch.zeros(H, device=device), post_norm=torch.zeros(H, device=device))
    if kind == FULL:
        D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_kv_heads
        t.update(q_proj=rn(Hq * 2 * D, H), k_proj=rn(Hkv * D, H), v_proj=rn(Hkv * D, H), o_proj=rn(H, Hq * D),
                 q_norm=torch.zeros(D, device=device), k_norm=torch.zeros(D, device=device))
        if cfg.qsa_topk:
            Di = cfg.qsa_indexer_dim
            t.update(index_qk_proj=rn((cfg.qsa_indexer_heads + 1) * Di, H), index_q_norm=torch.zeros(Di, device=device),
                     index_k_norm=torch.zeros(Di, device=device))
    else:
        Hv, Dv = cfg.linear_num_value_heads, cfg.linear_value_head_dim
        dt = torch.exp(torch.empty(Hv, device=device).uniform_(math.log(1e-3), math.log(1e-1), generator=gen))
        t.update(in_proj_qkvz=rn(cfg.gdn_qkvz_dim, H), in_proj_ba=rn(2 * Hv, H), out_proj=rn(H, Hv * Dv),
                 conv1d=rn(cfg.gdn_conv_dim, cfg.linear_conv_kernel, s=0.3),
                 A_log=torch.log(torch.empty(Hv, device=device).uniform_(1, 16, generator=gen)),
                 dt_bias=dt + torch.log(-torch.expm1(-dt)), g_norm=torch.ones(Dv, device=device))
    E, I, Is = cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    t.update(router=rn(E, H),
             w13_codes=torch.randint(-2**31, 2**31 - 1, (E, 2 * I // 128, H // 128, 128, 12), dtype=torch.int32,
                                     device=device, generator=gen),
             w13_scales=rn(E, 2 * I, H // 128, s=std / 2.3),
             w2_codes=torch.randint(-2**31, 2**31 - 1, (E, H // 128, I // 128, 128, 12), dtype=torch.int32,
                                    device=device, generator=gen),
             w2_scales=rn(E, H, I // 128, s=std / 2.3),
             shared_gate=rn(Is, H), shared_up=rn(Is, H), shared_down=rn(H, Is), shared_expert_gate=rn(1, H))
    if cfg.hc_count > 1:
        t["hc_attn"] = random_hc_tensors(cfg, device, gen)
        t["hc_mlp"] = random_hc_tensors(cfg, device, gen)
    return t


def random_ple_tensors(cfg: ModelConfig, device, gen) -> dict:
    """Random weights of one PLE layer (the n-gram table at ``init_std``)."""
    m = PLELayer(cfg)
    return {k: (torch.randn(v.shape, generator=gen, device=device) * cfg.init_std if v.dim() == 2
                else torch.zeros(v.shape, device=device)) for k, v in m.state_dict().items()}


class StudentLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, kind: str, t: dict):
        super().__init__()
        self.cfg, self.kind = cfg, kind

        def buf(name):
            self.register_buffer(name, t[name].float().clone())
        buf("in_norm")
        buf("post_norm")
        if kind == FULL:
            for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
                setattr(self, n, _master(t[n]))
            buf("q_norm")
            buf("k_norm")
            if "index_qk_proj" in t:  # QSA indexer: frozen (selection only, no gradient through it)
                self.register_buffer("index_qk_proj", t["index_qk_proj"].to(torch.bfloat16).clone())
                buf("index_q_norm")
                buf("index_k_norm")
        else:
            for n in ("in_proj_qkvz", "in_proj_ba", "out_proj"):
                setattr(self, n, _master(t[n]))
            for n in ("conv1d", "A_log", "dt_bias", "g_norm"):
                buf(n)
        self.moe = StudentMoE(cfg, t["router"], t["w13_codes"], t["w13_scales"], t["w2_codes"], t["w2_scales"],
                              t["shared_gate"], t["shared_up"], t["shared_down"], t["shared_expert_gate"])
        self.lora = nn.ModuleDict()  # optional adapters by projection name (train/lora.py)
        self.hc_attn = self.hc_mlp = None
        if cfg.hc_count > 1:  # hyper-connections: the layer reads a mix of the branches and writes back gated
            dev = t["in_norm"].device
            self.hc_attn = _hc_module(cfg, t["hc_attn"], True, dev)
            self.hc_mlp = _hc_module(cfg, t["hc_mlp"], True, dev)
        self.ple = None
        if "ple" in t:  # per-layer n-gram embedding, frozen; its table lookup is the native kernel on the GPU
            self.ple = PLELayer(cfg)
            self.ple.load_state_dict({k: v.float() for k, v in t["ple"].items()})
            self.ple.to(t["in_norm"].device).requires_grad_(False)
        self._ple_table = None

    def _ple_update(self, x, tokens, pack):
        """The PLE stream update of x ([B, T, H] or [B, T, G, H]) for token ids [B, T]."""
        from . import kernels
        ple = self.ple
        B, T = tokens.shape
        xs = x if self.hc_attn is not None else x.unsqueeze(-2)
        seg = None
        if pack is not None:  # each token's segment start in the packed row
            seg = torch.arange(T, device=tokens.device) - pack["pos"].reshape(-1).long()
        native = tokens.is_cuda and kernels.use("ple")
        if native and self._ple_table is None:
            from ..ops.ple import PleTable
            self._ple_table = PleTable.from_weight(ple.hash, ple.table, tokens.device, fp8=True)
        outs = []
        for b in range(B):
            if native:
                e = self._ple_table.lookup_tokens(tokens[b], seg)
            else:
                e = ple.embed(ple.hash.ids(tokens[b], seg))
            if tokens.is_cuda:
                kernels.hit("ple", native)
            outs.append(ple.mix(xs[b], e.float(), seg)[0])
        upd = torch.stack(outs).to(x.dtype)
        return upd if self.hc_attn is not None else upd.squeeze(-2)

    def _lin(self, name: str, x, fp8: bool):
        """x @ W^T for projection ``name`` (block-FP8 QAT weight when ``fp8``), plus its LoRA adapter if attached."""
        w = getattr(self, name)
        y = F.linear(x, (fp8_weight(w) if fp8 else w).to(x.dtype))
        if name in self.lora:
            y = y + self.lora[name](x).to(y.dtype)
        return y

    def groups(self):
        g = {k: [] for k in GROUPS}
        g["scale"] += [self.moe.w13_scales, self.moe.w2_scales]
        g["router"].append(self.moe.router)
        g["shared"] += [self.moe.shared_w13, self.moe.shared_down, self.moe.shared_expert_gate]
        if self.kind == FULL:
            g["dense_fp8"] += [self.q_proj, self.k_proj, self.v_proj]
            g["dense_bf16"].append(self.o_proj)
        else:
            g["dense_fp8"] += [self.in_proj_qkvz, self.out_proj]
            g["dense_bf16"].append(self.in_proj_ba)
        return g

    def _attn(self, x, B, T, pack=None):
        c = self.cfg
        D = c.head_dim
        qg = self._lin("q_proj", x, True).view(B, T, c.num_attention_heads, 2 * D)
        q, gate = qg[..., :D], qg[..., D:].reshape(B, T, -1)
        k = self._lin("k_proj", x, True).view(B, T, c.num_kv_heads, D)
        v = self._lin("v_proj", x, True).view(B, T, c.num_kv_heads, D)
        q, k = fused.rms_norm(q, self.q_norm, c.rms_norm_eps), fused.rms_norm(k, self.k_norm, c.rms_norm_eps)
        positions = torch.arange(T, device=x.device) if pack is None else pack["pos"][0]
        rope_pos = pack["pos3"] if pack is not None and pack.get("pos3") is not None else positions
        if R.is_three_row(rope_pos) and (c.mrope_section is None or c.qsa_topk):
            raise ValueError("three-row (multimodal) positions need cfg.mrope_section and no QSA")
        cos, sin = R.rope_cos_sin(rope_pos, c.rotary_dim, c.rope_theta, c.mrope_section)
        q, k = R.apply_rope(q, cos, sin), R.apply_rope(k, cos, sin)
        blkmap = self._qsa_blocks(x, positions, pack) if pack is not None else None
        if pack is None and q.is_cuda and q.dtype == torch.bfloat16 and D in (128, 256):
            # unpacked rows are B segments of T tokens: the native varlen kernels
            cu = torch.arange(B + 1, dtype=torch.int32) * T
            o = packed_attention(q.reshape(B * T, *q.shape[2:]), k.reshape(B * T, *k.shape[2:]),
                                 v.reshape(B * T, *v.shape[2:]), cu, T).reshape(B, T, -1)
        elif pack is None:
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               is_causal=True, enable_gqa=True).transpose(1, 2).reshape(B, T, -1)
        elif blkmap is not None:
            from .attention import varlen_attention
            o = varlen_attention(q[0], k[0], v[0], pack["cu_seqlens"], blkmap, c.qsa_block).reshape(B, T, -1)
        else:
            o = packed_attention(q[0], k[0], v[0], pack["cu_seqlens"], pack["max_seqlen"]).reshape(B, T, -1)
        o = o * torch.sigmoid(gate.float()).to(o.dtype)
        return self._lin("o_proj", o, False)

    @torch.no_grad()
    def _qsa_blocks(self, x, positions, pack):
        """QSA selection of a packed row (``train/attention.py`` ``qsa_select_packed``), or None while every
        segment fits the budget (topk x block tokens: each query then keeps all its blocks, the dense path). The
        indexer is frozen: index queries and raw keys come from its projection without a gradient."""
        c = self.cfg
        if not c.qsa_topk or getattr(self, "index_qk_proj", None) is None or not x.is_cuda:
            return None
        if int(pack["max_seqlen"]) <= c.qsa_topk * c.qsa_block:
            return None
        from .attention import qsa_select_packed
        Hi, Di = c.qsa_indexer_heads, c.qsa_indexer_dim
        proj = F.linear(x[0].to(torch.bfloat16), self.index_qk_proj)
        iq = R.rms_norm(proj[:, :Hi * Di].view(-1, Hi, Di), self.index_q_norm, c.rms_norm_eps)
        cos, sin = R.rope_cos_sin(positions, c.rotary_dim, c.rope_theta)
        iq = R.apply_rope(iq[None], cos[None], sin[None])[0].to(torch.bfloat16).contiguous()
        raw = proj[:, Hi * Di:].contiguous()
        tab_cos, tab_sin = R.rope_cos_sin(torch.arange(int(pack["max_seqlen"]) + 64, device=x.device), c.rotary_dim,
                                          c.rope_theta)
        return qsa_select_packed(iq, raw, self.index_k_norm.to(torch.bfloat16), tab_cos.contiguous(),
                                 tab_sin.contiguous(), c.rotary_dim, c.rms_norm_eps, pack["cu_seqlens"], c.qsa_block,
                                 c.qsa_topk)

    def _gdn(self, x, B, T, pack=None):
        c = self.cfg
        qkvz = self._lin("in_proj_qkvz", x, True)
        ba = self._lin("in_proj_ba", x, False)
        mixed, z = qkvz[..., : c.gdn_conv_dim], qkvz[..., c.gdn_conv_dim:]
        b, a = ba[..., : c.linear_num_value_heads], ba[..., c.linear_num_value_heads:]
        mixed = fused.conv_silu(mixed, self.conv1d, None if pack is None else pack["pos"])
        nk = c.linear_num_key_heads * c.linear_key_head_dim
        q = mixed[..., :nk].reshape(B, T, c.linear_num_key_heads, -1)
        k = mixed[..., nk:2 * nk].reshape(B, T, c.linear_num_key_heads, -1)
        v = mixed[..., 2 * nk:].reshape(B, T, c.linear_num_value_heads, -1)
        q = R.l2norm(q) * c.linear_key_head_dim ** -0.5  # grouped values: chunk_gated_delta_rule maps heads
        k = R.l2norm(k)
        g, beta = R.gdn_gates(b, a, self.A_log, self.dt_bias)
        o, _ = chunk_gated_delta_rule(q, k, v, g, beta, chunk_reset=None if pack is None else pack["chunk_reset"])
        o = fused.gated_rms_norm(o.to(x.dtype), z.reshape(B, T, c.linear_num_value_heads, -1), self.g_norm,
                                 c.rms_norm_eps)
        return self._lin("out_proj", o.reshape(B, T, -1), True)

    def forward(self, x, pack=None, tokens=None):
        c = self.cfg
        B, T, H = x.shape[0], x.shape[1], x.shape[-1]
        if pack is not None and B != 1:
            raise ValueError("packed bins are single rows (B = 1)")
        if self.ple is not None:
            if tokens is None:
                raise ValueError("a PLE layer needs the token ids")
            x = x + self._ple_update(x, tokens, pack)
        if self.hc_attn is not None:  # x: the branch stream [B, T, G, H]
            a, g = hc_read(x, self.hc_attn)
            y = fused.rms_norm(a, self.in_norm, c.rms_norm_eps)
            x = hc_inject(x, self._attn(y, B, T, pack) if self.kind == FULL else self._gdn(y, B, T, pack), g)
            a, g = hc_read(x, self.hc_mlp)
            y = fused.rms_norm(a, self.post_norm, c.rms_norm_eps)
            return hc_inject(x, self.moe(y.reshape(B * T, H)).reshape(B, T, H), g)
        y = fused.rms_norm(x, self.in_norm, c.rms_norm_eps)
        x = x + (self._attn(y, B, T, pack) if self.kind == FULL else self._gdn(y, B, T, pack))
        y = fused.rms_norm(x, self.post_norm, c.rms_norm_eps)
        return x + self.moe(y.reshape(B * T, H)).reshape(B, T, H)


class QADStudent(nn.Module):
    def __init__(self, cfg: ModelConfig, ref: R.HybridMoE, codes_scales, compute_dtype=torch.bfloat16,
                 checkpoint_layers: bool = True):
        super().__init__()
        self.cfg = cfg
        self.dtype = compute_dtype
        self.ckpt = checkpoint_layers
        self.register_buffer("embed", ref.embed_tokens.weight.detach().to(compute_dtype).clone())
        self.register_buffer("final_norm", ref.norm.weight.detach().float().clone())
        self.register_buffer("lm_head", ref.lm_head.weight.detach().to(compute_dtype).clone())
        self.layers = nn.ModuleList([StudentLayer(cfg, L.kind, layer_tensors_from_reference(L, codes_scales[i]))
                                     for i, L in enumerate(ref.layers)])
        self.hc_final = None
        if cfg.hc_count > 1:
            self.hc_final = _hc_module(cfg, {k: v.detach() for k, v in ref.hc_final.state_dict().items()}, False,
                                       self.embed.device)
        self._lm_head_t = None

    @property
    def lm_head_t(self):
        if self._lm_head_t is None or self._lm_head_t.device != self.lm_head.device:
            self._lm_head_t = self.lm_head.t().contiguous()
        return self._lm_head_t

    def param_groups(self):
        g = {k: [] for k in GROUPS}
        for L in self.layers:
            for k, v in L.groups().items():
                g[k] += v
        return g

    def hidden(self, ids, pack: dict | None = None, image_features=None, deepstack=None,
               image_token_id: int | None = None):
        """Final hidden states of ``ids`` [B, T]; ``pack`` (``train/packing.py`` ``PackedBin.forward_args``) makes
        the row a packed bin of several sequences (B = 1). Multimodal rows (the same contract as
        ``models.reference.HybridMoE.hidden``): ``pack["pos3"]`` three-row positions [3, T], ``image_features``
        [n, H] over the ``image_token_id`` tokens, ``deepstack[i]`` added to them after layer i."""
        x = F.embedding(ids, self.embed)
        mask = None
        if image_features is not None:
            mask = ids == image_token_id
            if int(mask.sum()) != image_features.shape[0]:
                raise ValueError(f"{int(mask.sum())} image tokens for {image_features.shape[0]} image features")
            x = x.clone()
            x[mask] = image_features.to(x.dtype)
        hc = getattr(self, "hc_final", None)
        if hc is not None:  # every branch starts as the embedding
            x = x[..., None, :].expand(*x.shape[:-1], self.cfg.hc_count, x.shape[-1]).contiguous()
        for i, L in enumerate(self.layers):
            if self.ckpt and torch.is_grad_enabled():
                x = checkpoint(L, x, pack, ids, use_reentrant=False)
            else:
                x = L(x, pack, ids)
            if deepstack is not None and i < len(deepstack):
                add = deepstack[i].to(x.dtype)
                x = x.clone()
                x[mask] = x[mask] + (add[:, None, :] if hc is not None else add)
        if hc is not None:
            x = hc_read(x, hc)[0]
        return fused.rms_norm(x, self.final_norm, self.cfg.rms_norm_eps)


def random_student(cfg: ModelConfig, device, seed: int = 0, checkpoint_layers=True) -> "QADStudent":
    """Student of ``cfg`` with random weights made directly on ``device`` (synthetic benchmarking)."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    st = QADStudent.__new__(QADStudent)
    nn.Module.__init__(st)
    st.cfg, st.dtype, st.ckpt, st._lm_head_t = cfg, torch.bfloat16, checkpoint_layers, None
    H, V = cfg.hidden_size, cfg.vocab_size
    st.register_buffer("embed", (torch.randn(V, H, generator=gen, device=dev) * cfg.init_std).to(torch.bfloat16))
    st.register_buffer("final_norm", torch.zeros(H, device=dev))
    st.register_buffer("lm_head", (torch.randn(V, H, generator=gen, device=dev) * cfg.init_std).to(torch.bfloat16))
    layers = []
    for i, kind in enumerate(cfg.layer_types):
        t = random_layer_tensors(cfg, kind, dev, gen)
        if i in cfg.ple_layer_ids:
            t["ple"] = random_ple_tensors(cfg, dev, gen)
        layers.append(StudentLayer(cfg, kind, t))
    st.layers = nn.ModuleList(layers)
    st.hc_final = _hc_module(cfg, random_hc_tensors(cfg, dev, gen, inject=False), False, dev) if cfg.hc_count > 1 else None
    return st
