"""QSA block-sparse verify attention on the native kernels (``csrc/qsa.cu`` + the sparse mode of
``csrc/attention.cu``), plus fp32 PyTorch oracles of every step.

Block = one 64-token KV page. Per full-attention layer:

* ``qsa_prep`` -- index queries (RMSNorm + RoPE, ``Hi`` heads of 128) for this step's tokens, and each token's raw
  index key stored at its KV slot;
* ``qsa_finalize`` -- pooled index keys of pages whose 64 tokens are all committed (mean, RMSNorm, RoPE at the
  page's first position), once per page;
* ``qsa_attention`` -- per session: scores of its W verify rows over its finalised pages, top-K per row, the union
  of the rows' pages plus the local (not yet finalised) pages with a row mask per page, then paged attention over
  that union (one pass for all rows of the session; GQA rows and the output gate as in the dense kernel).

The reference's QSA (``training/work/qwen38fn_lora/sparse_qsa.py:83-153``) scores 4-token blocks with a 4-head
128-dim indexer and keeps 512 of them (2,048 tokens); BASELINE config 5 asks for 64-token blocks and top-32 (the
same 2,048-token budget), which makes a block one page.
"""
from __future__ import annotations

import math

import torch

from ..models.reference import apply_rope
from ._ext import C

PAGE = 64


class QsaWorkspace:
    """Union buffers for up to ``S`` sessions of ``W`` verify rows and top-``K`` (fixed addresses); ``idx_q`` holds
    ``q_rows`` index-query rows (prefill chunks write there too)."""

    def __init__(self, S: int, W: int, K: int, max_pages: int, Hi: int, device, local_pages: int = 3,
                 q_rows: int = 0):
        dev = torch.device(device)
        self.ucap = W * K + local_pages
        i32 = dict(dtype=torch.int32, device=dev)
        self.u_page = torch.zeros(S, self.ucap, **i32)
        self.u_lpage = torch.zeros(S, self.ucap, **i32)
        self.u_mask = torch.zeros(S, self.ucap, dtype=torch.uint8, device=dev)
        self.u_count = torch.zeros(S, **i32)
        self.idx_q = torch.zeros(max(S * W, q_rows), Hi, 128, dtype=torch.bfloat16, device=dev)
        self.W, self.K, self.Hi, self.max_pages = W, K, Hi, max_pages


class QsaState:
    """What a serving engine keeps for QSA: per-layer index caches, finalised pages per session, the workspace."""

    def __init__(self, model, S: int, W: int, num_pages: int, max_pages: int, q_rows: int, splits: int = 1):
        c = model.cfg
        self.cache = model.new_qsa_cache(num_pages, S, max_pages)
        self.fin = torch.zeros(S, dtype=torch.int32, device=model.device)
        self.ws = QsaWorkspace(S, W, c.qsa_topk, max_pages, c.qsa_indexer_heads, model.device, q_rows=q_rows)
        self.k_norms = [lw.qsa_k_norm for lw in model.layers if lw.qsa_k_norm is not None]
        self.model = model
        self.splits = splits
        self.hs = None  # HiSparseState when the KV history lives in host memory
        self.replay = None  # DecisionReplay (record / force the selections; eager engine cycles only)

    def finalize(self, block_table, ctx_len):
        """Pooled keys for every page whose tokens are all committed (ctx_len), in every QSA layer."""
        m = self.model
        C().qsa_finalize([r for r, _ in self.cache], [k for _, k in self.cache], self.k_norms, block_table, self.fin,
                         ctx_len, m.rope_cos, m.rope_sin, m.cfg.rotary_dim, m.cfg.rms_norm_eps)


class DecisionReplay:
    """Record the sparse-attention decisions of every QSA call (the per-session page union, its logical pages and
    row masks) or force recorded ones in place of the selection (the reference's decision replay,
    ``training/work/qwen38fn_lora/decision_replay.py``): kernels and configurations are then compared on identical
    selections. Calls are matched in order; the decisions hold physical pages, so a forced run must allocate pages as
    the recorded one did (same engine, same inputs). Eager execution only (the log grows on the host)."""

    def __init__(self, mode: str = "record", log=None):
        if mode not in ("record", "force"):
            raise ValueError(mode)
        self.mode, self.log, self.cursor = mode, list(log or []), 0

    def record(self, ws: QsaWorkspace, S: int):
        self.log.append(tuple(t[:S].detach().clone() for t in (ws.u_page, ws.u_lpage, ws.u_mask, ws.u_count)))

    def force(self, ws: QsaWorkspace, S: int):
        if self.cursor >= len(self.log):
            raise RuntimeError(f"decision replay: {len(self.log)} recorded calls, call {self.cursor + 1} asked")
        rec = self.log[self.cursor]
        self.cursor += 1
        for dst, src in zip((ws.u_page, ws.u_lpage, ws.u_mask, ws.u_count), rec):
            if src.shape[0] != S:
                raise RuntimeError("decision replay: the forced call has a different number of sessions")
            dst[:S].copy_(src)

    def save(self, path):
        torch.save([tuple(t.cpu() for t in rec) for rec in self.log], path)

    @classmethod
    def load(cls, path, device, mode: str = "force"):
        return cls(mode, [tuple(t.to(device) for t in rec) for rec in torch.load(path, weights_only=True)])


def qsa_attention(q, kcache, vcache, block_table, seq_lens, fin, idx_key, ws: QsaWorkspace, out, gate=None,
                  gate_ld=0, gate_head_stride=0, splits: int = 1, hs=None, layer: int = 0,
                  replay: DecisionReplay | None = None, kv_scales=None):
    """q [S*W, Hq, D] (already normed / RoPE'd), ws.idx_q filled by ``qsa_prep`` for the same rows. With ``hs``
    (a ``HiSparseState``) the selected finalised pages are first made resident from the host pool; ``replay``
    records or forces the selections. ``kv_scales``: (kscale, vscale) of an NVFP4 cache."""
    c = C()
    S = seq_lens.shape[0]
    if replay is not None and replay.mode == "force":
        replay.force(ws, S)
    else:
        c.qsa_select(ws.idx_q, idx_key, block_table, fin, seq_lens, ws.W, ws.K, ws.Hi, ws.u_page[:S],
                     ws.u_lpage[:S], ws.u_mask[:S], ws.u_count[:S])
        if replay is not None:
            replay.record(ws, S)
    if hs is not None:
        hs.ctx.fetch(layer, ws.u_page, ws.u_lpage, ws.u_count, fin)
    D = q.shape[-1]
    pps = math.ceil(ws.ucap / splits)
    c.paged_attention(q, kcache, vcache, ws.u_page[:S], seq_lens, ws.W, 1.0 / math.sqrt(D), out, gate, gate_ld,
                      gate_head_stride, math.ceil(ws.ucap / pps), pps, 0, None, ws.u_count[:S], ws.u_lpage[:S],
                      ws.u_mask[:S], *(kv_scales or (None, None)))
    return out


# ------------------------------------------------------------------------------------------------ oracles
def rms(x, w, eps=1e-6):
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())


def prep_reference(proj_idx, positions, q_norm, cos_t, sin_t, Hi, rot, eps=1e-6):
    """proj_idx [T, (Hi+1)*128] -> (idx_q [T, Hi, 128] fp32, raw [T, 128] fp32)."""
    T = proj_idx.shape[0]
    q = rms(proj_idx[:, :Hi * 128].view(T, Hi, 128), q_norm, eps)
    half = rot // 2
    cos, sin = cos_t[positions.long(), :half], sin_t[positions.long(), :half]
    q = apply_rope(q.unsqueeze(0), cos.unsqueeze(0), sin.unsqueeze(0))[0]
    return q, proj_idx[:, Hi * 128:(Hi + 1) * 128].float()


def pooled_key_reference(raw_page, page_index, k_norm, cos_t, sin_t, rot, eps=1e-6):
    """raw_page [64, 128] (bf16 values) -> the page's index key (fp32)."""
    m = raw_page.float().mean(0).bfloat16().float()
    x = rms(m, k_norm, eps)
    half = rot // 2
    pos = torch.tensor([page_index * PAGE])
    cos, sin = cos_t[pos, :half], sin_t[pos, :half]
    return apply_rope(x.view(1, 1, 128), cos, sin).view(128)


def select_reference(idx_q, keys, fin, seq_len, W, K):
    """One session: idx_q [W, Hi, 128], keys [F, 128] (finalised pages, logical order) -> per row the sorted list
    of logical pages it attends (top-K finalised by score, ties to the lower index, plus local pages)."""
    F = fin
    last = (seq_len - 1) // PAGE
    rows = []
    for r in range(W):
        pos = seq_len - W + r
        if F <= K:
            chosen = list(range(F))
        else:
            sc = torch.relu(idx_q[r].float() @ keys[:F].float().t()).sum(0) / math.sqrt(128)
            # top-K with ties to the lower index: sort by (-score, index)
            order = sorted(range(F), key=lambda b: (-float(sc[b]), b))
            chosen = sorted(order[:K])
        local = [p for p in range(F, last + 1) if pos >= p * PAGE]
        rows.append(chosen + local)
    return rows


def attention_reference(q, kcache, vcache, bt_row, seq_len, W, rows_pages, gate=None):
    """One session's W verify rows: q [W, Hq, D]; each row attends to the keys of its pages up to its position."""
    Hq, D = q.shape[1], q.shape[2]
    Hkv = kcache.shape[1]
    g = Hq // Hkv
    out = torch.zeros(W, Hq, D)
    for r in range(W):
        pos = seq_len - W + r
        toks = [p * PAGE + j for p in rows_pages[r] for j in range(PAGE) if p * PAGE + j <= pos]
        toks = torch.tensor(toks)
        pages = bt_row[(toks // PAGE).long()].long()
        k = kcache[pages, :, (toks % PAGE).long()].float()  # [n, Hkv, D]
        v = vcache[pages, :, (toks % PAGE).long()].float()
        for h in range(Hq):
            s = (k[:, h // g] @ q[r, h].float()) / math.sqrt(D)
            p = torch.softmax(s, 0)
            o = p @ v[:, h // g]
            if gate is not None:
                o = o * torch.sigmoid(gate[r, h].float())
            out[r, h] = o
    return out
