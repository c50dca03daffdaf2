"""DFlash-style block drafter on the native kernels.

Contract (``training/work/qwen38fn_dflash/model.py:20-91``: plain residual, ``context="inject"``, window 1024;
the shipped drafter has 8 dense layers and verify width K=4):

* Fusion of a token with the target's hidden state: ``f = E[tok] + fc(h_target)``.
* Context: every committed token's K/V at each layer come from its fusion through the layer's ``ctx_norm`` and
  the layer's own k/v projections ("injected" context, no trunk pass over the context).
* Proposal block: slot 0 is the anchor (the next token already chosen by the target), slots 1..K-1 carry a mask
  embedding; every slot is conditioned on the target hidden state of the last committed position. The block runs
  through the layers with causal attention over [context window | block]; slot i proposes the token at
  anchor position + i + 1, so one forward proposes K tokens.
* The LM head covers a draft-vocabulary subset (``draft_vocab`` maps its rows to target ids).

Attention is gated like the target's (``[q_h | gate_h]`` per head), so the same fused q/k-norm/RoPE/KV-store and
paged-attention kernels serve both models.
"""
from __future__ import annotations

import torch

from ..config import DrafterConfig
from ..ops import C
from ..ops.attention import PAGE, paged_attention
from .reference import rope_cos_sin


class Drafter:
    def __init__(self, cfg: DrafterConfig, target_hidden: int, vocab_size: int, device, seed: int = 1,
                 draft_vocab: int = 32768, std: float = 0.02):
        self.cfg = cfg
        dev = torch.device(device)
        self.device = dev
        gen = torch.Generator(device=dev).manual_seed(seed)
        H, D, Hq, Hkv, I = cfg.hidden_size, cfg.head_dim, cfg.num_attention_heads, cfg.num_kv_heads, cfg.intermediate_size

        def randn(*shape):
            return (torch.randn(*shape, generator=gen, device=dev) * std).to(torch.bfloat16)

        self.vocab_size = vocab_size
        self.mask_id = vocab_size  # extra embedding row for the mask slots
        self.embed = randn(vocab_size + 1, H)
        self.fc = randn(H, target_hidden)
        self.layers = []
        for _ in range(cfg.num_layers):
            self.layers.append(dict(
                in_norm=torch.zeros(H, dtype=torch.bfloat16, device=dev),
                ctx_norm=torch.zeros(H, dtype=torch.bfloat16, device=dev),
                post_norm=torch.zeros(H, dtype=torch.bfloat16, device=dev),
                w_qkv=randn(Hq * 2 * D + 2 * Hkv * D, H),
                q_norm=torch.zeros(D, dtype=torch.bfloat16, device=dev),
                k_norm=torch.zeros(D, dtype=torch.bfloat16, device=dev),
                w_o=randn(H, Hq * D),
                w13=randn(2 * I, H),
                w2=randn(H, I)))
        self.final_norm = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        vd = min(draft_vocab, vocab_size)
        self.draft_vocab = torch.randperm(vocab_size, generator=gen, device=dev)[:vd].sort().values.int()
        self.lm_head = randn(vd, H)
        cos, sin = rope_cos_sin(torch.arange(1 << 17, device=dev), D, cfg.rope_theta)
        self.rope_cos, self.rope_sin = cos.contiguous(), sin.contiguous()
        self.selector = None

    def set_selector(self, sel: dict | None):
        """Candidate selector tensors (fp32): ``pred`` [Vd + 1, r], ``succ`` [Vd, r], ``proj`` [r, H] and ``top_k``;
        None proposes the unary argmax."""
        if sel is not None:
            sel = dict(sel)
            for k in ("pred", "succ", "proj"):
                sel[k] = sel[k].detach().float().to(self.device).contiguous()
            to_draft = torch.full((self.vocab_size,), -1, dtype=torch.long, device=self.device)
            to_draft[self.draft_vocab.long()] = torch.arange(self.draft_vocab.shape[0], device=self.device)
            sel["to_draft"] = to_draft
        self.selector = sel

    def _select(self, logits, y, anchor_ids, num_seqs: int, K: int):
        """Greedy chain through the candidate selector: slot j's predecessor is the token chosen at j - 1 (the
        anchor for slot 0); scores = unary + < P[pred] * (W y), S[c] > over the slot's top-k candidates."""
        sel = self.selector
        unary, cand = logits.float().view(num_seqs, K, -1).topk(sel["top_k"], -1)
        proj = (y.float() @ sel["proj"].t()).view(num_seqs, K, -1)
        succ = sel["succ"][cand]                                                   # [S, K, k, r]
        pred = sel["to_draft"][anchor_ids.long()]
        vd = sel["succ"].shape[0]
        picks = []
        for j in range(K):
            row = torch.where(pred >= 0, pred, torch.full_like(pred, vd))
            ctx = sel["pred"][row] * proj[:, j]
            sc = unary[:, j] + torch.einsum("sr,skr->sk", ctx, succ[:, j])
            pred = cand[:, j].gather(-1, sc.argmax(-1, keepdim=True)).squeeze(-1)
            picks.append(pred)
        return torch.stack(picks, 1)

    @classmethod
    def from_dir(cls, path, device, verify: bool = True) -> "Drafter":
        """Load a drafter directory (``train/drafter_tools.py`` layout: an export, a plain conversion, a layer
        expansion or a deployment copy; block-FP8 linears are dequantised to bf16 for the serving GEMMs)."""
        from ..train.drafter_tools import load_dir
        twin = load_dir(path, verify=verify)
        d = cls(twin.cfg, twin.fc.shape[1], twin.vocab_size, device, draft_vocab=len(twin.draft_vocab))
        twin.export_to(d)
        return d

    @property
    def kv_row_offset(self) -> int:
        c = self.cfg
        return c.num_attention_heads * 2 * c.head_dim

    def new_kv_cache(self, num_pages: int):
        c = self.cfg
        shape = (num_pages, c.num_kv_heads, PAGE, c.head_dim)
        return [(torch.zeros(shape, dtype=torch.bfloat16, device=self.device),
                 torch.zeros(shape, dtype=torch.bfloat16, device=self.device)) for _ in range(c.num_layers)]

    def new_workspace(self, max_rows: int):
        c = self.cfg
        bf = dict(dtype=torch.bfloat16, device=self.device)
        H, D, Hq, Hkv = c.hidden_size, c.head_dim, c.num_attention_heads, c.num_kv_heads
        return dict(
            x=torch.empty(max_rows, H, **bf), y=torch.empty(max_rows, H, **bf), f=torch.empty(max_rows, H, **bf),
            fcv=torch.empty(max_rows, H, **bf), qkv=torch.empty(max_rows, Hq * 2 * D + 2 * Hkv * D, **bf),
            q=torch.empty(max_rows + 8, Hq * D, **bf), attn=torch.empty(max_rows + 8, Hq * D, **bf),
            gu=torch.empty(max_rows, 2 * c.intermediate_size, **bf),
            hmid=torch.empty(max_rows, c.intermediate_size, **bf),
            logits=torch.empty(max_rows, self.lm_head.shape[0], **bf),
            tok=torch.empty(max_rows, dtype=torch.int32, device=self.device),
            dummy_q=torch.empty(1, **bf))

    def inject(self, ids, target_hidden_rows, positions, slots, kv, ws):
        """Write context K/V of ``ids`` (fused with their target hidden rows) at ``positions``/``slots``."""
        c, cC = self.cfg, C()
        N = ids.shape[0]
        f = ws["f"][:N]
        cC.embedding(ids, self.embed, f)
        fcv = ws["fcv"][:N]
        cC.gemm(target_hidden_rows, self.fc, out=fcv, residual=f)  # f + fc(h)
        y = ws["y"][:N]
        off = self.kv_row_offset
        for li, lw in enumerate(self.layers):
            cC.rmsnorm(fcv, None, lw["ctx_norm"], y, c.rms_norm_eps, True)
            kvrow = ws["qkv"][:N, : 2 * c.num_kv_heads * c.head_dim]
            cC.gemm(y, lw["w_qkv"][off:], out=kvrow)
            kc, vc = kv[li]
            cC.qk_norm_rope_store(kvrow, 0, c.num_kv_heads, c.head_dim, c.head_dim, lw["q_norm"], lw["k_norm"],
                                  positions, slots, self.rope_cos, self.rope_sin, c.rms_norm_eps, ws["dummy_q"], kc, vc)

    def propose(self, ids, cond_hidden, positions, slots, block_table, attn_len, kv, ws, out_drafts,
                num_seqs: int, max_pages: int | None = None):
        """ids [S*K] block tokens (anchor, masks); cond_hidden [S, Ht]; writes drafts [S, K] (target ids)."""
        c, cC = self.cfg, C()
        K = c.block_size - 1
        N = ids.shape[0]
        H, D, Hq, Hkv = c.hidden_size, c.head_dim, c.num_attention_heads, c.num_kv_heads
        x = ws["x"][:N]
        cC.embedding(ids, self.embed, x)
        fcv = ws["fcv"][:num_seqs]
        cC.gemm(cond_hidden, self.fc, out=fcv)
        x.view(num_seqs, K, H).add_(fcv[:, None, :])
        y = ws["y"][:N]
        for li, lw in enumerate(self.layers):
            cC.rmsnorm(x, None, lw["in_norm"], y, c.rms_norm_eps, True)
            qkv = ws["qkv"][:N]
            cC.gemm(y, lw["w_qkv"], out=qkv)
            kc, vc = kv[li]
            q = ws["q"][:N]
            cC.qk_norm_rope_store(qkv, Hq, Hkv, D, D, lw["q_norm"], lw["k_norm"], positions, slots, self.rope_cos,
                                  self.rope_sin, c.rms_norm_eps, q, kc, vc)
            attn = ws["attn"][:N]
            paged_attention(q.view(-1, Hq, D), kc, vc, block_table, attn_len, K, attn.view(-1, Hq, D),
                            gate=qkv[:, D:], gate_ld=qkv.shape[1], gate_head_stride=2 * D, window=c.window,
                            max_pages=max_pages)
            cC.gemm(attn, lw["w_o"], out=x, residual=x)
            cC.rmsnorm(x, None, lw["post_norm"], y, c.rms_norm_eps, True)
            gu = ws["gu"][:N]
            cC.gemm(y, lw["w13"], out=gu)
            cC.swiglu(gu, ws["hmid"][:N])
            cC.gemm(ws["hmid"][:N], lw["w2"], out=x, residual=x)
        cC.rmsnorm(x, None, self.final_norm, y, c.rms_norm_eps, True)
        logits = ws["logits"][:N]
        cC.gemm(y, self.lm_head, out=logits)
        if self.selector is not None:
            picks = self._select(logits, y, ids.view(num_seqs, K)[:, 0], num_seqs, K)
            out_drafts.copy_(self.draft_vocab[picks])
            return out_drafts
        tok = ws["tok"][:N]
        cC.select_tokens(logits, logits.shape[1], tok, 0.0, 0, None)
        out_drafts.copy_(self.draft_vocab[tok.long()].view(num_seqs, K))
        return out_drafts
