"""DFlash drafter training: a differentiable PyTorch twin of the serving drafter (``models/drafter.py``, same
parameters and math), trained on target hidden states, and its export into the serving drafter.

Per training sequence (tokens x[0..T), the target's hidden states h[0..T) -- h[t] after reading x[t]) and a set of
anchor positions a:

* context K/V of every layer come from the fusions ``f_t = E[x_t] + fc(h_t)`` through the layer's ``ctx_norm`` and
  k/v projections (injected context: no trunk pass over the context);
* the block at anchor a is ``[x_a, mask, ..., mask]`` (K slots at positions a..a+K-1), each slot plus
  ``fc(h_{a-1})``; it runs through the layers attending to the context keys before a inside the window and
  causally to the block's own earlier slots (gated attention, q/k RMSNorm, full-dim RoPE);
* slot i predicts x[a+i+1] over the draft vocabulary.

Objectives (the reference's ``training/work/qwen38fn_dflash/objective.py``): ``ce`` (next-token cross-entropy on
every slot) and, with teacher logits, ``kl`` (forward KL to the target's distribution restricted to the draft
vocabulary), mixed by ``kl_weight``; with a candidate selector (``selector_top_k`` > 0) also ``dpace``
(D-PACE-weighted CE, selector CE, early KL), ``acceptance`` (coverage KL + WTV at the serving temperature) and the
OPD terms over recorded verify cycles (``train/drafter_objective.py``).

Two training-only variants (the reference's ``Config.residual`` / ``ffn_type``, ``qwen38fn_dflash/model.py:20-91``,
``:114 GatedResidual``): ``residual="hc"`` keeps G branches of the stream; each sub-layer reads the hyper-connection
mix of the branches in place of its RMSNorm and writes back through per-branch gates, and a final readout mix
replaces the final norm. ``ffn="dense_shared"`` adds a shared SwiGLU scaled by ``sigmoid(y . w_shared_gate)``.
The serving drafter is plain and dense; ``train/drafter_tools.py`` converts the variants.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ..config import DrafterConfig
from ..models.reference import HyperConnection, apply_rope, hc_inject, rms_norm, rope_cos_sin
from .drafter_objective import CandidateSelector, Objective, acceptance_terms, combine, dpace_terms, opd_terms


class DrafterTrain(nn.Module):
    def __init__(self, cfg: DrafterConfig, target_hidden: int, vocab_size: int, draft_vocab: torch.Tensor,
                 device="cpu", seed: int = 0, std: float = 0.02):
        super().__init__()
        self.cfg = cfg
        g = torch.Generator(device=device).manual_seed(seed)
        H, D, Hq, Hkv, I = cfg.hidden_size, cfg.head_dim, cfg.num_attention_heads, cfg.num_kv_heads, cfg.intermediate_size

        def p(*shape):
            return nn.Parameter(torch.randn(*shape, generator=g, device=device) * std)

        def z(*shape):
            return nn.Parameter(torch.zeros(*shape, device=device))
        self.vocab_size, self.mask_id = vocab_size, vocab_size
        self.hc = cfg.residual == "hc"
        if cfg.residual not in ("plain", "hc") or cfg.ffn not in ("dense", "dense_shared"):
            raise ValueError(f"unknown drafter variant residual={cfg.residual!r} ffn={cfg.ffn!r}")

        def hc_mod(inject):  # starts as a single stream in disguise: constant mix, unit gates
            mod = HyperConnection(cfg, inject).to(device)
            with torch.no_grad():
                mod.w_down.copy_(torch.randn(mod.w_down.shape, generator=g, device=device) * std)
            return mod
        self.embed = p(vocab_size + 1, H)
        self.fc = p(H, target_hidden)
        self.layers = nn.ModuleList()
        for _ in range(cfg.num_layers):
            m = nn.Module()
            m.ctx_norm = z(H)
            if self.hc:
                m.hc_attn, m.hc_mlp = hc_mod(True), hc_mod(True)
            else:
                m.in_norm, m.post_norm = z(H), z(H)
            m.w_qkv = p(Hq * 2 * D + 2 * Hkv * D, H)
            m.q_norm, m.k_norm = z(D), z(D)
            m.w_o, m.w13, m.w2 = p(H, Hq * D), p(2 * I, H), p(H, I)
            if cfg.ffn == "dense_shared":
                Is = cfg.shared_intermediate_size
                m.sw13, m.sw2, m.shared_gate = p(2 * Is, H), p(H, Is), p(1, H)
            self.layers.append(m)
        if self.hc:
            self.hc_final = hc_mod(False)
        else:
            self.final_norm = z(H)
        self.register_buffer("draft_vocab", draft_vocab.long().to(device))
        self.lm_head = p(len(draft_vocab), H)
        to_draft = torch.full((vocab_size,), -1, dtype=torch.long)
        to_draft[draft_vocab.long().cpu()] = torch.arange(len(draft_vocab))
        self.register_buffer("to_draft", to_draft.to(device))
        self.selector = (CandidateSelector(len(draft_vocab), H, cfg.selector_top_k, cfg.selector_rank, device, g, std)
                         if cfg.selector_top_k > 0 else None)

    def _rope(self, x, pos):
        cos, sin = rope_cos_sin(pos, self.cfg.head_dim, self.cfg.rope_theta)
        return apply_rope(x, cos, sin)

    def _read(self, site: str, x, norm_w, hc_mod, probe):
        """The sub-layer input at ``site``: RMSNorm of the stream (plain) or the hyper-connection mix (hc)."""
        if hc_mod is not None:
            y, gate = hc_mod(x)
        else:
            y, gate = rms_norm(x, norm_w, self.cfg.rms_norm_eps), None
        if probe is not None:
            probe(site, x, y, gate)
        return y, gate

    def _ffn(self, m, y, i: int, probe):
        I = self.cfg.intermediate_size
        gu = y @ m.w13.t()
        out = (F.silu(gu[..., :I]) * gu[..., I:]) @ m.w2.t()
        if self.cfg.ffn == "dense_shared":
            Is = self.cfg.shared_intermediate_size
            logit = y @ m.shared_gate.t()
            if probe is not None:
                probe(f"shared{i}", None, logit, None)
            sg = y @ m.sw13.t()
            out = out + torch.sigmoid(logit) * ((F.silu(sg[..., :Is]) * sg[..., Is:]) @ m.sw2.t())
        return out

    def block_logits(self, tokens: torch.Tensor, hidden: torch.Tensor, anchors: torch.Tensor, probe=None,
                     return_hidden: bool = False):
        """tokens [T], hidden [T, Ht], anchors [A] (1 <= a, a + K <= T - 1) -> draft-vocab logits [A, K, Vd].
        ``probe(site, stream, sub-layer input, gate)`` is called at every read (sites ``attn<i>``, ``mlp<i>``,
        ``final``; ``shared<i>`` with the shared-gate logits); it may raise to stop the forward early."""
        c = self.cfg
        K, D, Hq, Hkv = c.k, c.head_dim, c.num_attention_heads, c.num_kv_heads
        T, A = tokens.shape[0], anchors.shape[0]
        dev = tokens.device
        fus = self.embed[tokens] + hidden.float() @ self.fc.t()                      # [T, H]
        blk_ids = torch.full((A, K), self.mask_id, dtype=torch.long, device=dev)
        blk_ids[:, 0] = tokens[anchors]
        x = self.embed[blk_ids] + (hidden[anchors - 1].float() @ self.fc.t())[:, None]  # [A, K, H]
        pos_b = anchors[:, None] + torch.arange(K, device=dev)[None]                  # [A, K]
        pos_c = torch.arange(T, device=dev)
        # visibility: context key p for block row (a, i) if p < a and p > a + i - window; block key (a, j) if j <= i
        qpos = pos_b.reshape(-1)
        ctx_ok = (pos_c[None] < anchors.repeat_interleave(K)[:, None]) & (pos_c[None] > qpos[:, None] - c.window)
        same = torch.arange(A, device=dev).repeat_interleave(K)
        blk_ok = (same[:, None] == same[None]) & (torch.arange(K, device=dev).repeat(A)[None] <=
                                                  torch.arange(K, device=dev).repeat(A)[:, None])
        mask = torch.cat([ctx_ok, blk_ok], 1)                                         # [A*K, T + A*K]
        G = c.hc_count
        if self.hc:  # every branch starts as the fusion
            x = x[..., None, :].expand(A, K, G, x.shape[-1]).clone()
        for i, m in enumerate(self.layers):
            kv_c = rms_norm(fus, m.ctx_norm, c.rms_norm_eps) @ m.w_qkv[Hq * 2 * D:].t()
            kc = rms_norm(kv_c[:, :Hkv * D].view(T, Hkv, D), m.k_norm, c.rms_norm_eps)
            kc = self._rope(kc.unsqueeze(0), pos_c[None])[0]
            vc = kv_c[:, Hkv * D:].view(T, Hkv, D)
            y, gate_a = self._read(f"attn{i}", x, getattr(m, "in_norm", None), getattr(m, "hc_attn", None), probe)
            y = y.reshape(A * K, -1)
            qkv = y @ m.w_qkv.t()
            qg = qkv[:, :Hq * 2 * D].view(A * K, Hq, 2 * D)
            q, gate = qg[..., :D], qg[..., D:]
            kb = qkv[:, Hq * 2 * D:Hq * 2 * D + Hkv * D].view(A * K, Hkv, D)
            vb = qkv[:, Hq * 2 * D + Hkv * D:].view(A * K, Hkv, D)
            q = self._rope(rms_norm(q, m.q_norm, c.rms_norm_eps).unsqueeze(0), qpos[None])[0]
            kb = self._rope(rms_norm(kb, m.k_norm, c.rms_norm_eps).unsqueeze(0), qpos[None])[0]
            keys = torch.cat([kc, kb], 0).repeat_interleave(Hq // Hkv, 1)            # [T + A*K, Hq, D]
            vals = torch.cat([vc, vb], 0).repeat_interleave(Hq // Hkv, 1)
            s = torch.einsum("qhd,khd->hqk", q.float(), keys.float()) / math.sqrt(D)
            s = s.masked_fill(~mask[None], float("-inf"))
            o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vals.float())
            o = (o * torch.sigmoid(gate.float())).reshape(A * K, Hq * D)
            o = (o @ m.w_o.t()).view(A, K, -1)
            x = hc_inject(x, o, gate_a) if self.hc else x + o
            y, gate_m = self._read(f"mlp{i}", x, getattr(m, "post_norm", None), getattr(m, "hc_mlp", None), probe)
            f = self._ffn(m, y, i, probe)
            x = hc_inject(x, f, gate_m) if self.hc else x + f
        y, _ = self._read("final", x, getattr(self, "final_norm", None), getattr(self, "hc_final", None), probe)
        logits = y @ self.lm_head.t()
        return (logits, y) if return_hidden else logits

    def _block_targets(self, tokens, anchors, teacher_logits):
        K = self.cfg.k
        tgt_pos = anchors[:, None] + 1 + torch.arange(K, device=tokens.device)[None]
        labels = self.to_draft[tokens[tgt_pos]]
        pred = self.to_draft[tokens[tgt_pos - 1]]
        teacher = None if teacher_logits is None else teacher_logits[tgt_pos - 1][..., self.draft_vocab]
        return labels, pred, teacher

    def objective_terms(self, tokens, hidden, anchors, obj: Objective, teacher_logits=None) -> dict:
        """Additive terms of the ``dpace`` / ``acceptance`` objective for the blocks at ``anchors`` (teacher forcing:
        slot j's predecessor is the data token x[a + j]); ``teacher_logits`` [T, V] are the target's logits."""
        if self.selector is None:
            raise ValueError("the dpace / acceptance objectives need a candidate selector (selector_top_k > 0)")
        logits, y = self.block_logits(tokens, hidden, anchors, return_hidden=True)
        labels, pred, teacher = self._block_targets(tokens, anchors, teacher_logits)
        if obj.name == "dpace":
            return dpace_terms(logits, labels, pred, y, self.selector, teacher, obj.dpace_alpha)
        if teacher is None:
            raise ValueError("the acceptance objective needs the teacher's logits")
        return acceptance_terms(logits, labels, pred, y, self.selector, teacher, obj.temperature, obj.joint)

    def opd_objective_terms(self, tokens, hidden, anchors, drafted, accepted, teacher_logits, obj: Objective,
                            sampler_q=None, sampler_cand=None) -> dict:
        """OPD terms of recorded verify cycles at ``anchors``: drafted [A, K] target ids the drafter proposed there,
        accepted [A], teacher_logits [A, K, V] the target's verify rows on the proposal prefix."""
        if self.selector is None:
            raise ValueError("OPD needs a candidate selector")
        logits, y = self.block_logits(tokens, hidden, anchors, return_hidden=True)
        d = self.to_draft[drafted]
        if (d < 0).any():
            raise ValueError("a recorded draft lies outside the draft vocabulary")
        return opd_terms(logits, d, self.to_draft[tokens[anchors]], y, self.selector,
                         teacher_logits[..., self.draft_vocab], accepted, obj.temperature, obj.joint, sampler_q,
                         None if sampler_cand is None else sampler_cand)

    def objective_loss(self, tokens, hidden, anchors, obj: Objective, teacher_logits=None, opd=None):
        """Loss of one chunk under ``obj``; ``opd``: the keyword arguments of :meth:`opd_objective_terms`."""
        if obj.name == "ce":
            return self.loss(tokens, hidden, anchors, teacher_logits, obj.kl_weight)
        terms = self.objective_terms(tokens, hidden, anchors, obj, teacher_logits)
        o = self.opd_objective_terms(obj=obj, **opd) if (opd is not None and obj.opd_weight) else None
        return combine(obj, terms, o)

    @torch.no_grad()
    def propose_greedy(self, tokens, hidden, anchors) -> torch.Tensor:
        """The serving drafter's greedy proposal chain at ``anchors`` [A] -> target ids [A, K]: the unary argmax
        without a selector; with one, slot j takes the best-scored of its top-k candidates given the token chosen at
        slot j - 1 (the anchor for slot 0)."""
        logits, y = self.block_logits(tokens, hidden, anchors, return_hidden=True)
        if self.selector is None:
            return self.draft_vocab[logits.argmax(-1)]
        unary, cand = logits.float().topk(self.selector.top_k, -1)
        pred = self.to_draft[tokens[anchors]]
        out = []
        for j in range(logits.shape[1]):
            sc = self.selector(cand[:, j], unary[:, j], y[:, j], pred)
            pred = cand[:, j].gather(-1, sc.argmax(-1, keepdim=True)).squeeze(-1)
            out.append(pred)
        return self.draft_vocab[torch.stack(out, 1)]

    def loss(self, tokens, hidden, anchors, teacher_logits=None, kl_weight: float = 0.0):
        """Mean CE of every slot's next token (tokens outside the draft vocabulary are skipped), plus
        ``kl_weight`` x forward KL to ``teacher_logits`` [T, V] of the target at the predicted positions."""
        K = self.cfg.k
        logits = self.block_logits(tokens, hidden, anchors)                           # [A, K, Vd]
        tgt_pos = anchors[:, None] + 1 + torch.arange(K, device=tokens.device)[None]
        tgt = self.to_draft[tokens[tgt_pos]]
        ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), tgt.reshape(-1), ignore_index=-1)
        if teacher_logits is None or kl_weight == 0:
            return ce
        # the target's logits that predict position a+i+1 are those read at a+i
        t = teacher_logits[tgt_pos - 1][..., self.draft_vocab].float()
        kl = F.kl_div(torch.log_softmax(logits.float(), -1), torch.log_softmax(t, -1), log_target=True,
                      reduction="batchmean")
        return ce + kl_weight * kl

    @torch.no_grad()
    def export_to(self, drafter):
        """Copy the trained weights (bf16) into a serving ``models.drafter.Drafter`` of the same shape (plain residual,
        dense FFN; ``train/drafter_tools.py`` converts the other variants first)."""
        if self.hc or self.cfg.ffn != "dense":
            raise ValueError("the serving drafter is plain / dense: convert this variant first (drafter_tools)")
        dt = torch.bfloat16
        drafter.embed.copy_(self.embed.to(dt))
        drafter.fc.copy_(self.fc.to(dt))
        for m, lw in zip(self.layers, drafter.layers):
            for n in ("in_norm", "ctx_norm", "post_norm", "w_qkv", "q_norm", "k_norm", "w_o", "w13", "w2"):
                lw[n].copy_(getattr(m, n).to(dt))
        drafter.final_norm.copy_(self.final_norm.to(dt))
        drafter.lm_head.copy_(self.lm_head.to(dt))
        drafter.draft_vocab.copy_(self.draft_vocab.int())
        drafter.set_selector(None if self.selector is None else dict(
            top_k=self.selector.top_k, pred=self.selector.pred_codebook.float(),
            succ=self.selector.succ_codebook.float(), proj=self.selector.proj.float()))
