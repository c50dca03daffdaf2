"""Plain-PyTorch hybrid MoE: the numerical oracle for every kernel, format and engine test.

A Qwen3-Next-style stack: ``num_layers`` layers, every ``full_attention_interval``-th one gated
attention and the rest Gated DeltaNet (GDN), each followed by a routed MoE with one sigmoid-gated
shared expert. It runs on any device in any float dtype; the tests use fp32 on CPU.

Semantics (what the reference serves, ``training/run_records/A4/config/recorded-config-99c11efb.json``
and the HF ``qwen3_next`` family it monkey-patches):

* RMSNorm multiplies by ``(1 + w)`` (zero-centred weight), the GDN output norm by ``w`` and ``silu(z)``
  (``training/work/qwen38fn_dflash/model.py:93-111`` shows the (1+w) form).
* Gated attention: ``q_proj`` yields ``[q | gate]`` per head, per-head q/k RMSNorm, partial NeoX RoPE
  on the first ``rotary_dim`` channels, causal softmax attention with GQA, output times ``sigmoid(gate)``.
* GDN: causal depthwise conv (kernel 4) + SiLU over ``[q | k | v]``, L2-normalised q/k (q scaled by
  ``Dk^-0.5``), ``beta = sigmoid(b)``, ``g = -exp(A_log) * softplus(a + dt_bias)``, and the gated delta
  rule per value head (key head ``h // (Hv/Hk)``)::

      S <- S * exp(g_t);  S <- S + k_t (beta_t (v_t - S^T k_t))^T;  o_t = S^T q_t       (S is [Dk, Dv])

* MoE: fp32 softmax router, top-k, renormalised (``norm_topk_prob``), SwiGLU experts with ``w13`` rows
  = gate then up (the packed-expert layout of ``training/work/qwen38fn_eval/export_int3_sidecar.py:1-15``).

Layer weights use contiguous projections ``in_proj_qkvz = [q | k | v | z]`` and ``in_proj_ba = [b | a]``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from ..config import FULL, ModelConfig


# ----------------------------------------------------------------------------------------------- functional pieces
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Zero-centred RMSNorm: ``x / rms(x) * (1 + w)`` computed in fp32."""
    z = x.float()
    z = z * torch.rsqrt(z.square().mean(-1, keepdim=True) + eps)
    return (z * (1.0 + w.float())).to(x.dtype)


def gated_rms_norm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """GDN output norm: ``x / rms(x) * w * silu(z)`` over the last dim, fp32 math."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return (xf * w.float() * F.silu(z.float())).to(x.dtype)


def rope_cos_sin(positions: torch.Tensor, rot: int, theta: float,
                 sections: tuple | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin [..., rot / 2] of positions [...]. With ``sections`` (multimodal RoPE) ``positions`` may be three-row
    [3, ...] (temporal, height, width): frequency f takes the height row when f = 1 (mod 3) and f < 3 sections[1],
    the width row when f = 2 (mod 3) and f < 3 sections[2], else the temporal row (the interleaved layout)."""
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float64, device=positions.device) / rot))
    if sections is not None and positions.dim() >= 2 and positions.shape[0] == 3:
        f = torch.arange(rot // 2, device=positions.device)
        row = torch.zeros_like(f)
        row[(f % 3 == 1) & (f < 3 * sections[1])] = 1
        row[(f % 3 == 2) & (f < 3 * sections[2])] = 2
        pos = positions.double().movedim(0, -1)[..., row]  # [..., rot / 2]
        ang = pos * inv
    else:
        ang = positions.double()[..., None] * inv
    return ang.cos().float(), ang.sin().float()


def is_three_row(positions) -> bool:
    return positions is not None and positions.dim() >= 2 and positions.shape[0] == 3


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """NeoX rotate-half RoPE on the first ``2 * cos.shape[-1]`` channels; x is [..., T, H, D], cos [..., T, rot/2]."""
    half = cos.shape[-1]
    xr, xp = x[..., : 2 * half].float(), x[..., 2 * half:]
    x1, x2 = xr[..., :half], xr[..., half:]
    c, s = cos[..., None, :], sin[..., None, :]
    out = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)
    return torch.cat([out, xp], dim=-1)


def gdn_gates(b: torch.Tensor, a: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    beta = torch.sigmoid(b.float())
    g = -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())
    return g, beta


def gated_delta_rule(q, k, v, g, beta, state=None):
    """Recurrent gated delta rule. q,k [B,T,Hv,Dk] (already L2-normalised, q scaled), v [B,T,Hv,Dv],
    g/beta [B,T,Hv]; state [B,Hv,Dk,Dv] fp32 or None. Returns (o [B,T,Hv,Dv], final state)."""
    B, T, H, Dk = k.shape
    Dv = v.shape[-1]
    S = torch.zeros(B, H, Dk, Dv, dtype=torch.float32, device=q.device) if state is None else state.float().clone()
    out = torch.empty(B, T, H, Dv, dtype=torch.float32, device=q.device)
    qf, kf, vf = q.float(), k.float(), v.float()
    for t in range(T):
        S = S * torch.exp(g[:, t].float())[..., None, None]
        kt = kf[:, t]
        mem = torch.einsum("bhk,bhkv->bhv", kt, S)
        delta = (vf[:, t] - mem) * beta[:, t].float()[..., None]
        S = S + kt[..., :, None] * delta[..., None, :]
        out[:, t] = torch.einsum("bhk,bhkv->bhv", qf[:, t], S)
    return out.to(v.dtype), S


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, conv_state: torch.Tensor | None = None):
    """Depthwise causal conv + SiLU. x [B,T,C], w [C,K], conv_state [B,C,K-1] (previous inputs) or None.
    Returns (y [B,T,C], new conv_state [B,C,K-1])."""
    B, T, C = x.shape
    K = w.shape[1]
    prev = torch.zeros(B, C, K - 1, dtype=x.dtype, device=x.device) if conv_state is None else conv_state.to(x.dtype)
    full = torch.cat([prev, x.transpose(1, 2)], dim=-1)  # [B, C, K-1+T]
    y = F.conv1d(full.float(), w.float()[:, None, :], groups=C)  # [B, C, T]
    new_state = full[..., -(K - 1):].contiguous() if K > 1 else prev
    return F.silu(y).transpose(1, 2).to(x.dtype), new_state


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().sum(-1, keepdim=True) + eps)).to(x.dtype)


def route(logits: torch.Tensor, top_k: int, renorm: bool):
    """fp32 softmax router -> (weights [N,k] fp32, ids [N,k] int64), best first."""
    probs = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(probs, top_k, dim=-1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return w, ids


# ----------------------------------------------------------------------------------------------- modules
class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(dim))
        self.eps = eps

    def forward(self, x):
        return rms_norm(x, self.weight, self.eps)


class GatedAttention(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        H, D = cfg.hidden_size, cfg.head_dim
        self.q_proj = nn.Linear(H, cfg.num_attention_heads * D * 2, bias=False)
        self.k_proj = nn.Linear(H, cfg.num_kv_heads * D, bias=False)
        self.v_proj = nn.Linear(H, cfg.num_kv_heads * D, bias=False)
        self.o_proj = nn.Linear(cfg.num_attention_heads * D, H, bias=False)
        self.q_norm = RMSNorm(D, cfg.rms_norm_eps)
        self.k_norm = RMSNorm(D, cfg.rms_norm_eps)
        if cfg.qsa_topk:  # QSA indexer: Hi query heads + one raw key per token, zero-centred norms
            Di, Hi = cfg.qsa_indexer_dim, cfg.qsa_indexer_heads
            self.index_qk_proj = nn.Linear(H, (Hi + 1) * Di, bias=False)
            self.index_q_norm = RMSNorm(Di, cfg.rms_norm_eps)
            self.index_k_norm = RMSNorm(Di, cfg.rms_norm_eps)

    def qsa_allowed(self, x, positions, cache, S):
        """QSA block selection (``training/work/qwen38fn_lora/sparse_qsa.py:83-153``) -> allowed [B, T, S] or None
        (every query keeps all its complete blocks). A query at position p sees its complete blocks b < (p + 1) / B:
        all when there are <= K, else the top-K by sum_h relu(q_h . k_b) / sqrt(Di) (ties to the lower index), plus
        its own incomplete block. k_b = RoPE_{B b}(norm_k(mean of the block's raw keys, in the raw keys' dtype))."""
        c = self.cfg
        Bsz, T, _ = x.shape
        Di, Hi, Bk, K = c.qsa_indexer_dim, c.qsa_indexer_heads, c.qsa_block, c.qsa_topk
        if is_three_row(positions):
            raise ValueError("QSA selection with multimodal (three-row) positions is not supported")
        proj = self.index_qk_proj(x)
        iq, raw = proj[..., :Hi * Di].view(Bsz, T, Hi, Di), proj[..., Hi * Di:]
        cos, sin = rope_cos_sin(positions, c.rotary_dim, c.rope_theta)
        iq = apply_rope(self.index_q_norm(iq), cos, sin)
        if cache is not None:
            if "idx_raw" in cache:
                raw = torch.cat([cache["idx_raw"], raw], dim=1)
            cache["idx_raw"] = raw
        qpos = torch.arange(S - T, S, device=x.device)
        complete = (qpos + 1) // Bk
        nb = S // Bk
        if int(complete.max()) <= K:
            return None
        pooled = raw[:, :nb * Bk].reshape(Bsz, nb, Bk, Di).float().mean(2).to(raw.dtype)
        bc, bs = rope_cos_sin(torch.arange(nb, device=x.device) * Bk, c.rotary_dim, c.rope_theta)
        keys = apply_rope(self.index_k_norm(pooled)[:, :, None], bc, bs)[:, :, 0]
        sc = torch.einsum("bthd,bnd->bthn", iq.float(), keys.float()).relu().sum(2) / math.sqrt(Di)
        allowed = torch.ones(Bsz, T, S, dtype=torch.bool, device=x.device)
        blk = torch.arange(S, device=x.device) // Bk
        for t in range(T):
            n = int(complete[t])
            if n <= K:
                continue
            for b in range(Bsz):
                order = torch.sort(sc[b, t, :n], descending=True, stable=True).indices[:K]
                keep = torch.zeros(nb + 1, dtype=torch.bool, device=x.device)
                keep[order] = True
                keep[n:] = True  # the own incomplete block (later keys are causally masked)
                allowed[b, t] = keep[blk]
        return allowed

    def qkv(self, x, positions):
        """x [B,T,H] -> q [B,T,Hq,D] (normed, roped), gate [B,T,Hq*D], k,v [B,T,Hkv,D] (k normed, roped)."""
        c = self.cfg
        B, T, _ = x.shape
        qg = self.q_proj(x).view(B, T, c.num_attention_heads, 2 * c.head_dim)
        q, gate = qg[..., : c.head_dim], qg[..., c.head_dim:]
        k = self.k_proj(x).view(B, T, c.num_kv_heads, c.head_dim)
        v = self.v_proj(x).view(B, T, c.num_kv_heads, c.head_dim)
        q, k = self.q_norm(q), self.k_norm(k)
        cos, sin = rope_cos_sin(positions, c.rotary_dim, c.rope_theta, c.mrope_section)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        return q, gate.reshape(B, T, -1), k, v

    def forward(self, x, positions, cache: dict | None = None):
        c = self.cfg
        B, T, _ = x.shape
        q, gate, k, v = self.qkv(x, positions)
        if cache is not None:
            if "k" in cache:
                k = torch.cat([cache["k"], k], dim=1)
                v = torch.cat([cache["v"], v], dim=1)
            cache["k"], cache["v"] = k, v
        S = k.shape[1]
        allowed = self.qsa_allowed(x, positions, cache, S) if c.qsa_topk else None
        rep = c.num_attention_heads // c.num_kv_heads
        kk = k.repeat_interleave(rep, dim=2)
        vv = v.repeat_interleave(rep, dim=2)
        scores = torch.einsum("bthd,bshd->bhts", q.float(), kk.float()) / math.sqrt(c.head_dim)
        qpos = torch.arange(S - T, S, device=x.device)
        mask = torch.arange(S, device=x.device)[None, :] > qpos[:, None]
        scores = scores.masked_fill(mask, float("-inf"))
        if allowed is not None:
            scores = scores.masked_fill(~allowed[:, None], float("-inf"))
        attn = torch.einsum("bhts,bshd->bthd", torch.softmax(scores, dim=-1), vv.float()).to(x.dtype)
        out = attn.reshape(B, T, -1) * torch.sigmoid(gate.float()).to(x.dtype)
        return self.o_proj(out)


class GatedDeltaNet(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        H = cfg.hidden_size
        Hv, Dv = cfg.linear_num_value_heads, cfg.linear_value_head_dim
        self.in_proj_qkvz = nn.Linear(H, cfg.gdn_qkvz_dim, bias=False)
        self.in_proj_ba = nn.Linear(H, 2 * Hv, bias=False)
        self.conv1d = nn.Parameter(torch.empty(cfg.gdn_conv_dim, cfg.linear_conv_kernel))
        self.A_log = nn.Parameter(torch.empty(Hv))
        self.dt_bias = nn.Parameter(torch.empty(Hv))
        self.norm = nn.Parameter(torch.ones(Dv))
        self.out_proj = nn.Linear(Hv * Dv, H, bias=False)

    def split(self, mixed):
        c = self.cfg
        nk = c.linear_num_key_heads * c.linear_key_head_dim
        q = mixed[..., :nk]
        k = mixed[..., nk: 2 * nk]
        v = mixed[..., 2 * nk:]
        B, T = mixed.shape[:2]
        return (q.reshape(B, T, c.linear_num_key_heads, c.linear_key_head_dim),
                k.reshape(B, T, c.linear_num_key_heads, c.linear_key_head_dim),
                v.reshape(B, T, c.linear_num_value_heads, c.linear_value_head_dim))

    def forward(self, x, positions=None, cache: dict | None = None):
        c = self.cfg
        B, T, _ = x.shape
        qkvz = self.in_proj_qkvz(x)
        mixed, z = qkvz[..., : c.gdn_conv_dim], qkvz[..., c.gdn_conv_dim:]
        ba = self.in_proj_ba(x)
        b, a = ba[..., : c.linear_num_value_heads], ba[..., c.linear_num_value_heads:]
        conv_state = cache.get("conv") if cache is not None else None
        mixed, new_conv = causal_conv1d(mixed, self.conv1d, conv_state)
        q, k, v = self.split(mixed)
        rep = c.linear_num_value_heads // c.linear_num_key_heads
        q = l2norm(q) * (c.linear_key_head_dim ** -0.5)
        k = l2norm(k)
        q, k = q.repeat_interleave(rep, dim=2), k.repeat_interleave(rep, dim=2)
        g, beta = gdn_gates(b, a, self.A_log, self.dt_bias)
        state = cache.get("ssm") if cache is not None else None
        o, S = gated_delta_rule(q, k, v, g, beta, state)
        if cache is not None:
            cache["conv"], cache["ssm"] = new_conv, S
        o = gated_rms_norm(o, z.reshape(B, T, c.linear_num_value_heads, c.linear_value_head_dim), self.norm,
                           c.rms_norm_eps)
        return self.out_proj(o.reshape(B, T, -1))


@dataclass
class SaliencyAccumulator:
    """REAP/gEAN cumulants per (layer, expert): counts, sum_g, sum_f, sum_f2, sum_gf
    (field order of ``training/work/qwen38fn_eval/reap_mm_select.py:33-35``)."""
    num_layers: int
    num_experts: int
    acc: torch.Tensor = field(init=False)

    FIELDS = ("counts", "sum_g", "sum_f", "sum_f2", "sum_gf")

    def __post_init__(self):
        self.acc = torch.zeros(self.num_layers, len(self.FIELDS), self.num_experts, dtype=torch.float64)

    def add(self, layer: int, expert_ids: torch.Tensor, g: torch.Tensor, fnorm: torch.Tensor):
        ids = expert_ids.reshape(-1).long().cpu()
        gg = g.reshape(-1).double().cpu()
        ff = fnorm.reshape(-1).double().cpu()
        a = self.acc[layer]
        a[0].index_add_(0, ids, torch.ones_like(gg))
        a[1].index_add_(0, ids, gg)
        a[2].index_add_(0, ids, ff)
        a[3].index_add_(0, ids, ff * ff)
        a[4].index_add_(0, ids, gg * ff)


class MoE(nn.Module):
    """Routed SwiGLU experts (``w13`` = gate rows then up rows) plus a sigmoid-gated shared expert."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        H, I, E = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts
        self.gate = nn.Linear(H, E, bias=False)
        self.w13 = nn.Parameter(torch.empty(E, 2 * I, H))
        self.w2 = nn.Parameter(torch.empty(E, H, I))
        Is = cfg.shared_expert_intermediate_size
        self.shared_gate_proj = nn.Linear(H, Is, bias=False)
        self.shared_up_proj = nn.Linear(H, Is, bias=False)
        self.shared_down_proj = nn.Linear(Is, H, bias=False)
        self.shared_expert_gate = nn.Linear(H, 1, bias=False)
        self.layer_index = -1
        self.saliency: SaliencyAccumulator | None = None
        self.expert_override = None  # callable(x_rows, expert) -> rows, e.g. a dequantized INT3 path

    def expert_forward(self, x, e):
        if self.expert_override is not None:
            return self.expert_override(x, e)
        I = self.cfg.moe_intermediate_size
        h = x @ self.w13[e].t()
        return (F.silu(h[:, :I]) * h[:, I:]) @ self.w2[e].t()

    def shared(self, x):
        y = self.shared_down_proj(F.silu(self.shared_gate_proj(x)) * self.shared_up_proj(x))
        return torch.sigmoid(self.shared_expert_gate(x)) * y

    def forward(self, x):
        c = self.cfg
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        w, ids = route(self.gate(xf), c.num_experts_per_tok, c.norm_topk_prob)
        out = torch.zeros_like(xf)
        for e in torch.unique(ids).tolist():
            tok, slot = (ids == e).nonzero(as_tuple=True)
            y = self.expert_forward(xf[tok], e)
            g = w[tok, slot]
            if self.saliency is not None:
                self.saliency.add(self.layer_index, torch.full_like(tok, e), g.detach(), y.detach().float().norm(dim=-1))
            out.index_add_(0, tok, (y * g[:, None].to(y.dtype)).to(out.dtype))
        out = out + self.shared(xf)
        return out.reshape(shape)


class HyperConnection(nn.Module):
    """Hyper-connection read of a residual stream of G branches h [..., G, H] (the reference model's gated residual,
    ``training/work/qwen38fn_lora/hc_mix.py:1-20``):

        zb   = rmsnorm_g(h) * (1 + w)               RMSNorm of every branch (H features), zero-centred weight [G*H]
        du   = zb @ W_down^T, di = zb @ W_inject^T   [.., R], [.., G]
        x    = mean_g(sigmoid(silu(du / 4) @ W_up^T) * zb)    the mixed sub-layer input [..., H]
        gate = 2 sigmoid(di / 4)                    the write-back gate of every branch [..., G]

    The write-back of the sub-layer's output y is ``h + y * gate`` per branch (:func:`hc_inject`). ``inject=False``
    (the final readout) has no gate."""

    def __init__(self, cfg: ModelConfig, inject: bool = True):
        super().__init__()
        G, H, R = cfg.hc_count, cfg.hidden_size, cfg.hc_lowrank
        self.G, self.H, self.R, self.eps = G, H, R, cfg.rms_norm_eps
        self.hc_norm = RMSNorm(G * H, cfg.rms_norm_eps)
        self.w_down = nn.Parameter(torch.zeros(R, G * H))
        self.w_up = nn.Parameter(torch.zeros(G * H, R))
        self.w_inject = nn.Parameter(torch.zeros(G, G * H)) if inject else None

    def forward(self, h):
        G, H = self.G, self.H
        hf = h.float()
        zb = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + self.eps)
        zb = zb.flatten(-2) * (1.0 + self.hc_norm.weight.float())
        s = F.silu((zb @ self.w_down.float().t()) * 0.25)
        pre = s @ self.w_up.float().t()
        x = (torch.sigmoid(pre) * zb).unflatten(-1, (G, H)).mean(-2).to(h.dtype)
        if self.w_inject is None:
            return x, None
        return x, (2.0 * torch.sigmoid((zb @ self.w_inject.float().t()) * 0.25)).to(h.dtype)


def hc_inject(h, y, gate):
    """h [..., G, H] + y [..., H] * gate [..., G] per branch."""
    return (h.float() + y.float()[..., None, :] * gate.float()[..., :, None]).to(h.dtype)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, kind: str, index: int):
        super().__init__()
        self.kind = kind
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.mixer = GatedAttention(cfg) if kind == FULL else GatedDeltaNet(cfg)
        self.mlp = MoE(cfg)
        self.mlp.layer_index = index
        self.hc = cfg.hc_count > 1
        if self.hc:  # hyper-connections: each sub-layer reads a mix of the branches and writes back gated
            self.hc_attn = HyperConnection(cfg)
            self.hc_mlp = HyperConnection(cfg)
        from .ple import PLELayer
        self.ple = PLELayer(cfg) if index in cfg.ple_layer_ids else None

    def _ple(self, x, tokens, cache):
        """Add the per-layer n-gram embedding update (one sequence per batch row; ``cache`` keeps the last n-1 tokens
        and the conv inputs of every row for incremental decoding)."""
        ple = self.ple
        xs = x if self.hc else x.unsqueeze(-2)
        pad = (ple.k - 1) * ple.dil
        hists = cache.get("ple_hist") if cache is not None else None
        states = cache.get("ple_conv") if cache is not None else None
        outs, new_h, new_s = [], [], []
        for b in range(tokens.shape[0]):
            hist = hists[b] if hists is not None else None
            state = states[b] if states is not None else None
            upd, c = ple.mix(xs[b], ple.embed(ple.hash.ids(tokens[b], history=hist)), conv_state=state)
            outs.append(upd)
            if cache is not None:
                ext = tokens[b].long() if hist is None else torch.cat([hist, tokens[b].long()])
                new_h.append(ext[-(ple.hash.n - 1):])
                prev = torch.zeros(pad, c.shape[1], device=c.device) if state is None else state
                new_s.append(torch.cat([prev, c])[-pad:] if pad else prev)
        if cache is not None:
            cache["ple_hist"], cache["ple_conv"] = new_h, new_s
        upd = torch.stack(outs).to(x.dtype)
        return x + (upd if self.hc else upd.squeeze(-2))

    def forward(self, x, positions, cache=None, tokens=None):
        if self.ple is not None:
            if tokens is None:
                raise ValueError("a PLE layer needs the token ids")
            x = self._ple(x, tokens, cache)
        if self.hc:  # x is the branch stream [B, T, G, H]
            a, g = self.hc_attn(x)
            x = hc_inject(x, self.mixer(self.input_layernorm(a), positions, cache), g)
            a, g = self.hc_mlp(x)
            return hc_inject(x, self.mlp(self.post_attention_layernorm(a)), g)
        x = x + self.mixer(self.input_layernorm(x), positions, cache)
        return x + self.mlp(self.post_attention_layernorm(x))


class HybridMoE(nn.Module):
    """The whole model. ``forward(ids, cache)`` returns logits; pass the same ``cache`` list across calls for
    incremental decoding (per layer: attention ``k``/``v``, GDN ``conv``/``ssm``)."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(cfg, t, i) for i, t in enumerate(cfg.layer_types)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        self.hc_final = HyperConnection(cfg, inject=False) if cfg.hc_count > 1 else None

    @torch.no_grad()
    def init_weights(self, seed: int = 0):
        """Random init: every matrix N(0, init_std); norms at their identity; GDN gates in a sane range."""
        gen = torch.Generator().manual_seed(seed)
        std = self.cfg.init_std
        for name, p in self.named_parameters():
            if name.endswith("A_log"):
                p.copy_(torch.log(torch.empty(p.shape).uniform_(1.0, 16.0, generator=gen)))
            elif name.endswith("dt_bias"):
                dt = torch.exp(torch.empty(p.shape).uniform_(math.log(1e-3), math.log(1e-1), generator=gen))
                p.copy_(dt + torch.log(-torch.expm1(-dt)))
            elif name.endswith("mixer.norm"):
                p.fill_(1.0)
            elif "layernorm" in name or name.endswith("norm.weight"):
                p.zero_()
            else:
                p.copy_(torch.randn(p.shape, generator=gen) * std)
        return self

    def new_cache(self):
        return [dict() for _ in self.layers]

    def hidden(self, ids, cache=None, start_pos: int = 0, positions=None, image_features=None, deepstack=None,
               image_token_id: int | None = None):
        """Final hidden states. Multimodal (one sequence, B = 1): ``positions`` three-row [3, T]
        (``models/vision.py`` ``mrope_positions``, with ``cfg.mrope_section``), ``image_features`` [n, H] replace
        the embeddings of the ``image_token_id`` tokens in order, and the i-th ``deepstack`` feature [n, H] is added
        to those tokens' hidden state after decoder layer i (Qwen3-VL's deepstack; in every branch of a
        hyper-connection stream). Decoding after an image continues with 1-D positions offset by the sequence's
        delta (last three-row position + 1 - length)."""
        B, T = ids.shape
        if positions is None:
            positions = torch.arange(start_pos, start_pos + T, device=ids.device)
        elif is_three_row(positions) and self.cfg.mrope_section is None:
            raise ValueError("three-row positions need cfg.mrope_section")
        x = self.embed_tokens(ids)
        mask = None
        if image_features is not None:
            mask = ids == image_token_id
            if int(mask.sum()) != image_features.shape[0]:
                raise ValueError(f"{int(mask.sum())} image tokens for {image_features.shape[0]} image features")
            x = x.clone()
            x[mask] = image_features.to(x.dtype)
        if self.hc_final is not None:  # every branch starts as the embedding
            x = x[..., None, :].expand(*x.shape[:-1], self.cfg.hc_count, x.shape[-1]).contiguous()
        for i, layer in enumerate(self.layers):
            x = layer(x, positions, None if cache is None else cache[i], ids)
            if deepstack is not None and i < len(deepstack):
                add = deepstack[i].to(x.dtype)
                x = x.clone()
                x[mask] = x[mask] + (add[:, None, :] if self.hc_final is not None else add)
        if self.hc_final is not None:
            x = self.hc_final(x)[0]
        return self.norm(x)

    def forward(self, ids, cache=None, start_pos: int = 0):
        return self.lm_head(self.hidden(ids, cache, start_pos))

    @torch.no_grad()
    def greedy_decode(self, prompt: torch.Tensor, steps: int):
        """prompt [B, T] -> generated ids [B, steps] and the logits of every decode step [B, steps, V]."""
        cache = self.new_cache()
        logits = self.forward(prompt, cache, 0)[:, -1]
        pos = prompt.shape[1]
        toks, all_logits = [], []
        for _ in range(steps):
            nxt = logits.argmax(-1)
            toks.append(nxt)
            all_logits.append(logits)
            logits = self.forward(nxt[:, None], cache, pos)[:, -1]
            pos += 1
        return torch.stack(toks, 1), torch.stack(all_logits, 1)

    def moe_layers(self):
        return [layer.mlp for layer in self.layers]


def build_reference(cfg: ModelConfig, seed: int = 0, dtype=torch.float32) -> HybridMoE:
    return HybridMoE(cfg).init_weights(seed).to(dtype)
