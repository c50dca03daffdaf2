"""QSA block-sparse verify attention on the native kernels (``csrc/qsa.cu`` + the sparse modes of the attention
kernels), plus fp32 PyTorch oracles of every step.

Block = ``B`` tokens, a divisor of the 64-token KV page (4 for the reference's own model, 64 for BASELINE config 5).
Per full-attention layer:

* ``qsa_prep`` -- index queries (RMSNorm + RoPE, ``Hi`` heads of 128) for this step's tokens, and each token's raw
  index key stored at its KV slot;
* ``qsa_finalize`` -- pooled index keys of blocks whose B tokens are all committed (mean, RMSNorm, RoPE at the
  block's first position), once per block;
* ``qsa_attention`` -- per session: each verify row's scores over its complete blocks (blocks completed inside the
  verify window pooled on the fly), top-K per row, the union of the rows' blocks plus each row's own incomplete
  block with a row mask per block, then attention over that union (one pass for all rows of the session; GQA rows
  and the output gate as in the dense kernel): page mode (B = 64) on the paged kernel's sparse mode, sub-page
  blocks gathered into the tcgen05 kernel's shared-memory tiles.

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
    """Union buffers for up to ``S`` sessions of ``W`` verify rows and top-``K`` blocks of ``block`` tokens (fixed
    addresses); ``idx_q`` holds ``q_rows`` index-query rows (prefill chunks write there too); ``sel`` is the
    selection kernels' row-bitmask scratch (all zero between calls)."""

    def __init__(self, S: int, W: int, K: int, max_pages: int, Hi: int, device, block: int = PAGE, q_rows: int = 0,
                 idx_q: torch.Tensor | None = None):
        dev = torch.device(device)
        self.block = block
        self.max_blocks = max_pages * (PAGE // block)
        self.ucap = W * K + W + 2  # every row's top-K, every row's own incomplete block
        i32 = dict(dtype=torch.int32, device=dev)
        self.u_page = torch.zeros(S, self.ucap, **i32)
        self.u_lpage = torch.zeros(S, self.ucap, **i32)
        self.u_mask = torch.zeros(S, self.ucap, dtype=torch.uint8, device=dev)
        self.u_count = torch.zeros(S, **i32)
        self.sel = torch.zeros(S, self.max_blocks + 1, **i32)
        # committed blocks' scores from the tensor-core kernel (all W rows of a set at once; W * Hi <= 32)
        self.scores = (torch.empty(S * W * self.max_blocks, dtype=torch.float32, device=dev) if W * Hi <= 32
                       else None)
        self.idx_q = (idx_q if idx_q is not None else
                      torch.zeros(max(S * W, q_rows), Hi, 128, dtype=torch.bfloat16, device=dev))
        self.W, self.K, self.Hi, self.max_pages = W, K, Hi, max_pages


class QsaState:
    """What a serving engine keeps for QSA: per-layer index caches, finalised pages per session, the workspace."""

    def __init__(self, model, S: int, W: int, num_pages: int, max_pages: int, q_rows: int, splits: int = 1,
                 prefill_sets: int = 0, prefill_rows: int = 8):
        c = model.cfg
        self.cache = model.new_qsa_cache(num_pages, S, max_pages)
        self.fin = torch.zeros(S, dtype=torch.int32, device=model.device)  # finalised blocks per session
        self.ws = QsaWorkspace(S, W, c.qsa_topk, max_pages, c.qsa_indexer_heads, model.device, block=c.qsa_block,
                               q_rows=q_rows)
        # prefill: row sets of prefill_rows consecutive prompt positions, their own unions (same index queries);
        # per chunk the session's blocks are finalised layer by layer into the pooled-key cache first
        self.pf = (QsaWorkspace(prefill_sets, prefill_rows, c.qsa_topk, max_pages, c.qsa_indexer_heads, model.device,
                                block=c.qsa_block, idx_q=self.ws.idx_q) if prefill_sets else None)
        i32 = dict(dtype=torch.int32, device=model.device)
        self.pf_fin0, self.pf_fin, self.pf_ctx = (torch.zeros(S, **i32) for _ in range(3))
        self.k_norms = [lw.qsa_k_norm for lw in model.layers if lw.qsa_k_norm is not None]
        self.model = model
        self.splits = splits
        self.hs = None  # HiSparseState when the KV history lives in host memory
        self.replay = None  # DecisionReplay (record / force the selections; eager engine cycles only)

    def finalize(self, block_table, ctx_len):
        """Pooled keys for every block whose tokens are all committed (ctx_len), in every QSA layer."""
        m = self.model
        C().qsa_finalize([r for r, _ in self.cache], [k for _, k in self.cache], self.k_norms, block_table, self.fin,
                         ctx_len, m.rope_cos, m.rope_sin, m.cfg.rotary_dim, m.cfg.rms_norm_eps, m.cfg.qsa_block)


    def prefill_chunk(self, row: int, done: int, end: int):
        """Before a prefill chunk of session ``row``: blocks below ``done`` tokens already have pooled keys in
        every layer, the chunk's raw keys complete the blocks below ``end``."""
        self.pf_fin0.zero_()
        self.pf_ctx.zero_()
        self.pf_fin0[row] = done // self.ws.block
        self.pf_ctx[row] = end

    def prefill_attention(self, q, kcache, vcache, block_table, seq_lens, bt_row, layer: int, raw, key, k_norm, out,
                          gate=None, gate_ld=0, gate_head_stride=0, kv_scales=None):
        """QSA attention of prefill row sets (``seq_lens`` [n] ends, ``bt_row`` [n] the session): this layer's
        pooled keys of the chunk's complete blocks, then selection and sparse attention as in verify."""
        m = self.model
        self.pf_fin.copy_(self.pf_fin0)
        C().qsa_finalize([raw], [key], [k_norm], block_table, self.pf_fin, self.pf_ctx, m.rope_cos, m.rope_sin,
                         m.cfg.rotary_dim, m.cfg.rms_norm_eps, self.ws.block)
        return qsa_attention(q, kcache, vcache, block_table, seq_lens, self.pf_fin, key, self.pf, out, gate, gate_ld,
                             gate_head_stride, splits=self.splits, kv_scales=kv_scales, raw=raw, k_norm=k_norm,
                             rope=(m.rope_cos, m.rope_sin), rot=m.cfg.rotary_dim, eps=m.cfg.rms_norm_eps,
                             bt_row=bt_row)


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
                  replay: DecisionReplay | None = None, kv_scales=None, raw=None, k_norm=None, rope=None,
                  rot: int = 64, eps: float = 1e-6, bt_row=None):
    """q [S*W, Hq, D] (already normed / RoPE'd), ws.idx_q filled by ``qsa_prep`` for the same rows; ``raw`` /
    ``k_norm`` / ``rope`` = (cos, sin): the layer's raw index keys and key norm (blocks completed inside the verify
    window are pooled from them). With ``hs`` (a ``HiSparseState``) the selected finalised pages are first made
    resident from the host pool; ``replay`` records or forces the selections. ``kv_scales``: (kscale, vscale) of an
    NVFP4 cache. ``bt_row``: the row sets are prefill positions of session ``bt_row[i]`` (``fin``, ``idx_key`` and
    ``block_table`` are then indexed by session)."""
    c = C()
    S = seq_lens.shape[0]
    if replay is not None and replay.mode == "force":
        replay.force(ws, S)
    else:
        c.qsa_select(ws.idx_q, idx_key, raw, k_norm, block_table, fin, seq_lens, ws.W, ws.K, ws.Hi, ws.block, ws.sel,
                     rope[0], rope[1], rot, eps, ws.u_page[:S], ws.u_lpage[:S], ws.u_mask[:S], ws.u_count[:S],
                     bt_row, ws.scores)
        if replay is not None:
            replay.record(ws, S)
    if hs is not None:
        hs.ctx.fetch(layer, ws.u_page, ws.u_lpage, ws.u_count, fin)
    D = q.shape[-1]
    if ws.block == PAGE:  # a block is a page: the paged kernel's sparse mode walks the page union
        pps = math.ceil(ws.ucap / splits)
        c.paged_attention(q, kcache, vcache, ws.u_page[:S], seq_lens, ws.W, 1.0 / math.sqrt(D), out, gate, gate_ld,
                          gate_head_stride, math.ceil(ws.ucap / pps), pps, 0, None, ws.u_count[:S], ws.u_lpage[:S],
                          ws.u_mask[:S], *(kv_scales or (None, None)))
        return out
    if kv_scales is not None:
        raise ValueError("QSA blocks smaller than a page need a bf16 KV cache")
    # sub-page blocks: the tcgen05 kernel gathers each 64-key tile from PAGE / B union entries
    per_tile = PAGE // ws.block
    tiles = math.ceil(ws.ucap / per_tile)
    tps = math.ceil(tiles / splits)
    c.paged_attention(q, kcache, vcache, block_table, seq_lens, ws.W, 1.0 / math.sqrt(D), out, gate, gate_ld,
                      gate_head_stride, math.ceil(tiles / tps), tps, 0, bt_row, ws.u_count[:S], ws.u_lpage[:S],
                      ws.u_mask[:S], None, None, sp_block=ws.block, sp_slot=ws.u_page[:S])
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


def pooled_key_reference(raw_block, block_index, k_norm, cos_t, sin_t, rot, eps=1e-6, block: int = PAGE):
    """raw_block [B, 128] (bf16 values) -> the block's index key (fp32), RoPE at its first position."""
    m = raw_block.float().mean(0).bfloat16().float()
    x = rms(m, k_norm, eps)
    half = rot // 2
    pos = torch.tensor([block_index * block])
    cos, sin = cos_t[pos, :half], sin_t[pos, :half]
    return apply_rope(x.view(1, 1, 128), cos, sin).view(128)


def select_reference(idx_q, keys, seq_len, W, K, block: int = PAGE):
    """One session: idx_q [W, Hi, 128], keys [n, 128] (pooled keys of the session's complete blocks, logical
    order: committed ones and those completed inside the window) -> per row the sorted list of blocks it attends:
    its complete blocks b < (p + 1) / B (the top-K by score, ties to the lower index, when there are more than K)
    and its own incomplete block."""
    rows = []
    for r in range(W):
        pos = seq_len - W + r
        n = (pos + 1) // block
        if n <= K:
            chosen = list(range(n))
        else:
            sc = torch.relu(idx_q[r].float() @ keys[:n].float().t()).sum(0) / math.sqrt(128)
            order = sorted(range(n), key=lambda b: (-float(sc[b]), b))
            chosen = sorted(order[:K])
        if (pos + 1) % block:
            chosen.append(n)
        rows.append(chosen)
    return rows


def attention_reference(q, kcache, vcache, bt_row, seq_len, W, rows_blocks, gate=None, block: int = PAGE):
    """One session's W verify rows: q [W, Hq, D]; each row attends to the keys of its blocks up to its position."""
    Hq, D = q.shape[1], q.shape[2]
    Hkv = kcache.shape[1]
    g = Hq // Hkv
    out = torch.zeros(W, Hq, D)
    for r in range(W):
        pos = seq_len - W + r
        toks = [b * block + j for b in rows_blocks[r] for j in range(block) if b * block + j <= pos]
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
