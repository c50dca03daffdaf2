"""Speculative serving engine on one GPU; under expert parallelism every rank runs one over its own sessions and
the model's MoE layers exchange tokens with the other ranks (``parallel/ep.py``).

One decode cycle for all resident sessions (fixed shapes, no host inputs, CUDA-graph replayable):

1. ``build_window``: verify rows [anchor, d1..dK] at positions ctx..ctx+K, KV slots from the page table;
2. target forward over S*(K+1) rows (GDN layers commit the previous cycle's accepted prefix on the fly);
3. LM head + token selection (argmax or Gumbel-max sampling);
4. ``spec_accept``: accepted prefix (greedy match, or seeded Bernoulli(p) for benchmarks), emitted tokens,
   ctx += m+1, next anchor;
5. drafter: inject the window rows' context K/V, then propose the next K drafts from a block
   [anchor, mask x K-1] conditioned on the target hidden state of the last committed row.

The cycle alternates the GDN pending-buffer parity, so two graphs are captured and replayed in turn. The host
reads back only the emitted tokens of each cycle (pinned, asynchronous) and keeps page allocation one cycle ahead.
Prefill runs the target over the prompt in chunks (attention as virtual rows of 8 queries sharing the page-table
row; GDN in commit-all mode) and injects the prompt tail into the drafter cache.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import torch

from ..config import ServeConfig
from ..models.drafter import Drafter
from ..models.hybrid import HybridModel, StepBatch
from ..ops import C
from ..ops.attention import PAGE
from ..ops.gdn import GdnScratch

PREFILL_CHUNK = 2048


@dataclass
class Session:
    sid: int
    row: int
    prompt: list[int]
    max_new_tokens: int
    generated: list[int] = field(default_factory=list)
    done: bool = False
    emitted: list[int] = field(default_factory=list)  # every token the target emitted (generated is capped)
    last_used: float = 0.0


@dataclass
class Parked:
    """An idle session whose slot was given away: its committed recurrent state in pinned host memory (GDN conv and
    SSM rows, PLE history and conv rows, the drafter's ring pages, the QSA finalisation mark). Its KV pages stay
    allocated on the device."""
    sess: Session
    committed: int
    gdn: list
    ple: list
    dkv: list
    qsa_fin: int | None


class SpecEngine:
    def __init__(self, model: HybridModel, drafter: Drafter | None, scfg: ServeConfig, max_sessions: int,
                 max_context: int, num_pages: int | None = None):
        self.model, self.drafter, self.scfg = model, drafter, scfg
        dev = model.device
        self.device = dev
        S = self.S = max_sessions
        K = self.K = scfg.spec_k if drafter is not None else 0
        W = self.W = K + 1
        self.max_context = max_context
        self.maxp = math.ceil((max_context + 2 * W + 8) / PAGE)
        # prefill attention runs virtual sequences of this many consecutive queries (x the GQA group <= 64 rows)
        self.prefill_rows = max(1, min(8, 64 // (model.cfg.num_attention_heads // model.cfg.num_kv_heads)))
        self.hs_slots = 0
        if scfg.hisparse:  # GPU pages: per-session caches and rings, prefill staging, scratch (the host holds history)
            if not model.cfg.qsa_topk:
                raise ValueError("HiSparse offload needs QSA attention (cfg.qsa_topk > 0)")
            from ..ops.hisparse import gpu_pages
            self.hs_slots = scfg.hisparse_hot_blocks or W * model.cfg.qsa_topk + 32
            num_pages = gpu_pages(S, self.maxp, self.hs_slots, 4) - 1
        num_pages = (num_pages or S * self.maxp) + 1
        # the last page is a scratch sink: rows without a session point at it, so their (ignored) window
        # writes never land in another session's pages
        self.scratch_page = num_pages - 1
        self.alloc = C().PageAllocator(num_pages - 1, PAGE)
        if scfg.hisparse and model.cfg.qsa_block != 64:
            raise ValueError("HiSparse moves whole KV pages: it needs 64-token QSA blocks (qsa_block=64)")
        if scfg.kv_dtype == "nvfp4" and model.cfg.qsa_topk and model.cfg.qsa_block != 64:
            raise ValueError("QSA blocks smaller than a page run on the bf16 KV cache")
        if scfg.kv_dtype == "nvfp4" and scfg.hisparse:
            raise ValueError("the HiSparse host pool holds bf16 / e4m3 pages: use kv_dtype='bf16' with hisparse")
        self.kv = model.new_kv_cache(num_pages, scfg.kv_dtype)
        self.gdn = model.new_gdn_states(S, W)
        self.ple = model.new_ple_states(S, W) if model.cfg.ple_layer_ids else None
        i32 = dict(dtype=torch.int32, device=dev)
        self.block_table = torch.full((S, self.maxp), self.scratch_page, **i32)
        self.bt_host = torch.full((S, self.maxp), self.scratch_page, dtype=torch.int32).pin_memory()
        self.ctx_len = torch.zeros(S, **i32)
        self.anchor = torch.zeros(S, **i32)
        self.drafts = torch.zeros(S, max(K, 1), **i32)
        self.win_ids = torch.zeros(S * W, **i32)
        self.win_pos = torch.zeros(S * W, **i32)
        self.win_slots = torch.zeros(S * W, **i32)
        self.attn_len = torch.zeros(S, **i32)
        self.seq_slot = torch.arange(S, **i32)
        self.n_commit = torch.zeros(S, **i32)
        self.tgt_tok = torch.zeros(S * W, **i32)
        self.out_tokens = torch.zeros(S, W, **i32)
        self.out_count = torch.zeros(S, **i32)
        self.last_row = torch.zeros(S, **i32)
        self.step_ctr = torch.zeros(1, **i32)
        self.total = torch.zeros(1, dtype=torch.int64, device=dev)
        self.active = torch.zeros(S, **i32)
        self.ws = model.new_workspace(max(S * W, PREFILL_CHUNK))
        self.logits = torch.empty(max(S * W, 8), model.cfg.vocab_size, dtype=torch.bfloat16, device=dev)
        self.parity = 0
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.sessions: dict[int, Session] = {}
        self.parked: dict[int, Parked] = {}
        self.prefilled_tokens = 0  # tokens run through prefill (continuations prefill only their new tokens)
        self.free_rows = list(range(S))
        self.out_host = torch.zeros(S, W, dtype=torch.int32).pin_memory()
        self.cnt_host = torch.zeros(S, dtype=torch.int32).pin_memory()
        if drafter is not None:
            dc = drafter.cfg
            self.ring = dc.window // PAGE + 3
            dpages = S * self.ring
            self.dkv = drafter.new_kv_cache(dpages)
            p = torch.arange(self.maxp, device=dev)
            self.d_block_table = (torch.arange(S, device=dev)[:, None] * self.ring + p[None, :] % self.ring).int()
            self.dws = drafter.new_workspace(max(S * W, PREFILL_CHUNK))
            self.d_ids = torch.zeros(S * K, **i32)
            self.d_pos = torch.zeros(S * K, **i32)
            self.d_slots = torch.zeros(S * K, **i32)
            self.d_attn_len = torch.zeros(S, **i32)
            self.win_dslots = torch.zeros(S * W, **i32)
            self.scratch_ids = torch.zeros(S * W, **i32)
            self.scratch_pos = torch.zeros(S * W, **i32)
            self.scratch_len = torch.zeros(S, **i32)
            self.cond = torch.empty(S, model.cfg.hidden_size, dtype=torch.bfloat16, device=dev)
        self.mode = {"greedy": 0, "rejection": 0, "bernoulli": 1}[scfg.accept_mode]
        self.gdn_scratch = GdnScratch(model.gdn_shape, 1, PREFILL_CHUNK, dev)
        self.qsa = None
        if model.cfg.qsa_topk:
            from ..ops.qsa import QsaState
            # index-query rows: a verify step's S * W, or a prefill chunk rounded up to whole row sets
            self.qsa = QsaState(model, S, W, num_pages, self.maxp, max(S * W, PREFILL_CHUNK + 8), splits=scfg.qsa_splits,
                                prefill_sets=math.ceil(PREFILL_CHUNK / self.prefill_rows),
                                prefill_rows=self.prefill_rows)
        self.hs = None
        if scfg.hisparse:
            from ..ops.hisparse import HiSparseState
            self.hs = HiSparseState(self.kv, self.qsa.cache, S, self.maxp, self.hs_slots, 4, fp8=scfg.hisparse_fp8)
            self.qsa.hs = self.hs

    # ------------------------------------------------------------------ one cycle (device only)
    def _cycle(self, parity: int):
        cC, m = C(), self.model
        S, K, W = self.S, self.K, self.W
        if self.hs is not None:  # ring pages for this window; pages the last cycle completed go to the host pool
            self.hs.ctx.cycle_start(self.block_table, self.ctx_len, W)
            self.hs.ctx.writeback(self.block_table, self.qsa.fin, self.ctx_len)
        if self.qsa is not None:  # pooled index keys of the pages the last cycle completed
            self.qsa.finalize(self.block_table, self.ctx_len)
        cC.build_window(self.anchor, self.drafts if K else None, 0, self.ctx_len, self.block_table, self.win_ids,
                        self.win_pos, self.win_slots, self.attn_len, self.step_ctr, W, 0)
        b = StepBatch(self.win_ids, self.win_pos, self.win_slots, self.block_table, self.attn_len, self.seq_slot,
                      self.n_commit, W, parity, max_pages=self.maxp)
        hidden = m.forward(b, self.kv, self.gdn, self.ws, qsa=self.qsa, ple=self.ple)
        logits = self.logits[: S * W]
        m.logits(hidden, out=logits)
        cC.select_tokens(logits, m.cfg.vocab_size, self.tgt_tok, float(self.scfg.temperature), self.scfg.seed,
                         self.step_ctr)
        if self.drafter is not None:  # drafter slots of the window positions (before ctx advances)
            cC.build_window(self.anchor, self.drafts, 0, self.ctx_len, self.d_block_table, self.scratch_ids,
                            self.scratch_pos, self.win_dslots, self.scratch_len, None, W, 0)
        cC.spec_accept(self.win_ids.view(S, W), self.tgt_tok.view(S, W), self.seq_slot, self.active, self.ctx_len,
                       self.n_commit, self.out_tokens, self.out_count, self.anchor, self.last_row, self.step_ctr,
                       self.total, self.mode, float(self.scfg.accept_prob), self.scfg.seed)
        if self.drafter is not None:
            d = self.drafter
            d.inject(self.win_ids, hidden, self.win_pos, self.win_dslots, self.dkv, self.dws)
            cC.build_window(self.anchor, None, d.mask_id, self.ctx_len, self.d_block_table, self.d_ids, self.d_pos,
                            self.d_slots, self.d_attn_len, None, K, 0)
            cC.gather_rows(hidden, self.last_row, self.cond)
            d.propose(self.d_ids, self.cond, self.d_pos, self.d_slots, self.d_block_table, self.d_attn_len,
                      self.dkv, self.dws, self.drafts, S, max_pages=self.maxp)

    def capture(self):
        """Capture one graph per GDN parity (warm-up runs first so every lazy allocation happens outside)."""
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            for p in (0, 1):
                self._cycle(p)
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        for p in (0, 1):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._cycle(p)
            self.graphs[p] = g
        torch.cuda.synchronize()

    def run_cycle(self):
        if self.graphs:
            self.graphs[self.parity].replay()
        else:
            self._cycle(self.parity)
        self.parity ^= 1

    # ------------------------------------------------------------------ host side
    def _sync_pages(self, rows=None):
        """Refresh the page-table rows of live sessions (host, native allocator) and upload the table."""
        rows = set(range(self.S) if rows is None else rows)
        for s in self.sessions.values():
            if s.row in rows:
                self.alloc.fill_row(s.sid, self.bt_host, s.row)
                n = len(self.alloc.pages(s.sid))
                self.bt_host[s.row, n:] = self.scratch_page
        self.block_table.copy_(self.bt_host, non_blocking=True)

    # ------------------------------------------------------------------ session continuation and parking
    @property
    def free_slots(self) -> int:
        """Rows a new session can take now: free rows plus idle sessions that can be parked to make room."""
        return len(self.free_rows) + (0 if self.hs is not None else len(self._idle()))

    def has_session(self, sid: int) -> bool:
        return sid in self.sessions or sid in self.parked

    def _idle(self):
        return [s for s in self.sessions.values() if s.done]

    def _make_room(self):
        if self.free_rows:
            return
        idle = self._idle() if self.hs is None else []
        if not idle:
            raise RuntimeError("no free session slot")
        self.park(min(idle, key=lambda s: s.last_used).sid)

    def _committed(self, r: int) -> int:
        """Tokens of row r whose recurrent state is committed (the last cycle's accepted rows are still pending)."""
        return int(self.ctx_len[r]) - int(self.n_commit[r])

    @torch.no_grad()
    def park(self, sid: int):
        """Move an idle session's committed state to pinned host memory and free its row (the reference parks one
        GDN snapshot per idle session in host memory; its KV stays where it is)."""
        sess = self.sessions[sid]
        if not sess.done:
            raise RuntimeError(f"session {sid} is decoding; only idle sessions park")
        if self.hs is not None:
            raise NotImplementedError("parking with the HiSparse host pool")
        r = sess.row
        torch.cuda.synchronize(self.device)

        def host(t):
            return torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t)
        gdn = [(host(st.conv[r]), host(st.ssm[r])) for st in self.gdn]
        ple = [(host(st.hist[r]), host(st.hist_len[r]), host(st.conv[r])) for st in (self.ple or ())]
        dkv = []
        if self.drafter is not None:
            pages = slice(r * self.ring, (r + 1) * self.ring)
            dkv = [(host(k[pages]), host(v[pages])) for k, v in self.dkv]
        fin = int(self.qsa.fin[r]) if self.qsa is not None else None
        self.parked[sid] = Parked(sess, self._committed(r), gdn, ple, dkv, fin)
        del self.sessions[sid]
        self.active[r] = 0
        self.n_commit[r] = 0
        self.bt_host[r] = self.scratch_page
        self.block_table[r].copy_(self.bt_host[r])
        sess.row = -1
        self.free_rows.append(r)

    @torch.no_grad()
    def _unpark(self, sid: int) -> Session:
        self._make_room()
        pk = self.parked.pop(sid)
        sess = pk.sess
        r = sess.row = self.free_rows.pop(0)
        for st, (conv, ssm) in zip(self.gdn, pk.gdn):
            st.conv[r].copy_(conv)
            st.ssm[r].copy_(ssm)
        for st, (hist, hl, conv) in zip(self.ple or (), pk.ple):
            st.hist[r].copy_(hist)
            st.hist_len[r].copy_(hl)
            st.conv[r].copy_(conv)
        if pk.dkv:
            pages = slice(r * self.ring, (r + 1) * self.ring)
            for (k, v), (hk, hv) in zip(self.dkv, pk.dkv):
                k[pages].copy_(hk)
                v[pages].copy_(hv)
        if pk.qsa_fin is not None:
            self.qsa.fin[r] = pk.qsa_fin
        self.ctx_len[r] = pk.committed
        self.n_commit[r] = 0
        self.sessions[sid] = sess
        self._sync_pages([r])
        return sess

    @torch.no_grad()
    def continue_session(self, sid: int, tokens: list[int], max_new_tokens: int, on_chunk=None) -> Session:
        """Next turn of an idle (or parked) session: ``tokens`` is its whole transcript so far plus the new input.
        Only the part after the committed state is prefilled; a transcript that differs from what the engine
        committed (or the HiSparse pool) falls back to prefilling it all."""
        if len(tokens) + max_new_tokens + 2 * self.W > self.max_context:
            raise ValueError("prompt + max_new_tokens exceed max_context")
        if sid in self.parked:
            self._unpark(sid)
        sess = self.sessions[sid]
        if not sess.done:
            raise RuntimeError(f"session {sid} is still decoding")
        r = sess.row
        torch.cuda.synchronize(self.device)
        committed = self._committed(r)
        known = (sess.prompt + sess.emitted)[:committed]
        if self.hs is not None or len(tokens) <= committed or list(tokens[:committed]) != known:
            self.release(sid)
            return self.add_session(sid, list(tokens), max_new_tokens, on_chunk)
        sess.prompt, sess.generated, sess.emitted = list(tokens), [], []
        sess.max_new_tokens, sess.done = max_new_tokens, False
        self.alloc.ensure(sid, len(tokens) + 2 * self.W + 8)
        self._sync_pages([r])
        self.ctx_len[r] = committed
        self.n_commit[r] = 0  # the last window's accepted rows are prefilled again below
        self._prefill(sess, on_chunk, start=committed)
        return sess

    def add_session(self, sid: int, prompt: list[int], max_new_tokens: int, on_chunk=None):
        self._make_room()
        if len(prompt) + max_new_tokens + 2 * self.W > self.max_context:
            raise ValueError("prompt + max_new_tokens exceed max_context")
        row = self.free_rows.pop(0)
        sess = Session(sid, row, list(prompt), max_new_tokens)
        self.sessions[sid] = sess
        if self.hs is not None:  # the prompt is prefilled into the staging pages
            self.bt_host[row] = torch.arange(self.hs.staging_base, self.hs.staging_base + self.maxp, dtype=torch.int32)
            self.block_table[row].copy_(self.bt_host[row])
        else:
            self.alloc.ensure(sid, len(prompt) + 2 * self.W + 8)
            self._sync_pages([row])
        self._prefill(sess, on_chunk)
        return sess

    @torch.no_grad()
    def score(self, tokens: list[int], fn):
        """Run ``tokens`` through the target model as one temporary session, chunk by chunk, calling
        ``fn(hidden_rows [T, H], start)`` with the final-normed hidden states of every chunk (teacher scoring)."""
        sid = -(1 << 30)
        sess = self.add_session(sid, tokens, 1, on_chunk=fn)
        self.release(sess.sid)

    @torch.no_grad()
    def _prefill(self, sess: Session, on_chunk=None, start: int = 0):
        """Prefill ``sess.prompt[start:]`` (``start`` > 0: the recurrent state holds the first ``start`` tokens)."""
        cC, m = C(), self.model
        if m.ep is not None and m.ep.world > 1:
            raise NotImplementedError("prefill under expert parallelism needs every rank in the same forward; "
                                      "this engine prefills one rank's session alone")
        dev = self.device
        L = len(sess.prompt)
        ids_all = torch.tensor(sess.prompt, dtype=torch.int32, device=dev)
        pages = (self.block_table[sess.row].long() if self.hs is not None else
                 torch.tensor(self.alloc.pages(sess.sid), dtype=torch.int64, device=dev))
        slot_row = torch.tensor([sess.row], dtype=torch.int32, device=dev)
        if start == 0:
            for st in self.gdn:  # fresh recurrent state for this row
                st.conv[sess.row].zero_()
                st.ssm[sess.row].zero_()
            for st in self.ple or ():
                st.reset(sess.row)
        hidden_last = None
        self.prefilled_tokens += L - start
        for c0 in range(start, L, PREFILL_CHUNK):
            T = min(PREFILL_CHUNK, L - c0)
            pos = torch.arange(c0, c0 + T, device=dev, dtype=torch.int32)
            slots = (pages[pos.long() // PAGE] * PAGE + (pos.long() % PAGE)).int()
            qp = self.prefill_rows
            nv = (T + qp - 1) // qp
            vlen = torch.arange(1, nv + 1, device=dev, dtype=torch.int32) * qp + c0
            if self.qsa is not None:  # this chunk's QSA bookkeeping: the blocks its raw keys complete
                self.qsa.prefill_chunk(sess.row, c0 if c0 > start else 0, c0 + T)
            b = StepBatch(ids_all[c0:c0 + T].contiguous(), pos, slots, self.block_table, None, slot_row,
                          self.n_commit, T, 0, commit_current=True, max_pages=self.maxp,
                          attn_bt_row=torch.full((nv,), sess.row, dtype=torch.int32, device=dev),
                          attn_seq_lens=vlen, attn_q_per_seq=qp)
            hidden = m.forward(b, self.kv, self.gdn, self.ws, self.gdn_scratch, qsa=self.qsa, ple=self.ple)
            if on_chunk is not None:
                on_chunk(hidden[:T], c0)
            if self.drafter is not None:
                keep = max(0, T - (self.drafter.cfg.window + 64))
                dslots = (self.d_block_table[sess.row, (pos.long() // PAGE)] * PAGE + pos.long() % PAGE).int()
                self.drafter.inject(ids_all[c0 + keep:c0 + T].contiguous(), hidden[keep:T], pos[keep:].contiguous(),
                                    dslots[keep:].contiguous(), self.dkv, self.dws)
            hidden_last = hidden[T - 1:T]
        logits = self.logits[:1]
        m.logits(hidden_last, out=logits)
        tok = torch.empty(1, dtype=torch.int32, device=dev)
        cC.select_tokens(logits, m.cfg.vocab_size, tok, 0.0, 0, None)
        r = sess.row
        self.ctx_len[r] = L
        if self.qsa is not None:  # the prompt's complete pages get their pooled index keys now
            self.qsa.fin[r] = 0
            self.qsa.finalize(self.block_table, self.ctx_len)
        if self.hs is not None:  # complete pages -> host pool, the partial page -> its ring page
            full, part = L // PAGE, L % PAGE
            self.hs.ctx.after_prefill(self.block_table, r, 0, full, full + (1 if part else 0))
            self.bt_host[r] = self.scratch_page
            if part:
                self.bt_host[r, full] = self.hs.ring_page(r, full)
            self.block_table[r].copy_(self.bt_host[r])
            self.hs.reset_session(r)
        self.anchor[r] = tok[0]
        self.n_commit[r] = 0
        self.active[r] = 1
        if self.drafter is not None:  # first drafts: propose from the prefill's last hidden state
            self.drafts[r].fill_(0)
        sess.generated.append(int(tok.item()))
        sess.emitted.append(sess.generated[-1])

    def update_weights(self, pkg_dir) -> dict:
        """Swap in the weights of a deploy package between steps (in place: the captured graphs stay valid)."""
        torch.cuda.synchronize(self.model.device)
        return self.model.update_from_package(pkg_dir)

    def release(self, sid: int):
        if sid in self.parked:  # its KV pages only
            self.parked.pop(sid)
            if self.hs is None:
                self.alloc.release(sid)
            return
        sess = self.sessions.pop(sid)
        self.active[sess.row] = 0
        if self.hs is None:
            self.alloc.release(sid)
        self.bt_host[sess.row] = self.scratch_page
        if self.hs is not None:
            self.block_table[sess.row].copy_(self.bt_host[sess.row])
        self.free_rows.append(sess.row)

    def step(self) -> dict[int, list[int]]:
        """One cycle for every session + host bookkeeping; returns the tokens emitted per session."""
        if self.hs is None:  # pages for this cycle's window (at most W new tokens); HiSparse maps them on device
            for s in self.sessions.values():
                self.alloc.ensure(s.sid, len(s.prompt) + len(s.generated) + 2 * self.W + 8)
            self._sync_pages()
        self.run_cycle()
        self.out_host.copy_(self.out_tokens, non_blocking=True)
        self.cnt_host.copy_(self.out_count, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        emitted = {}
        for s in list(self.sessions.values()):
            n = int(self.cnt_host[s.row])
            toks = self.out_host[s.row, :n].tolist()
            room = s.max_new_tokens - len(s.generated)
            if not s.done and n > room:
                # the turn ends inside this window: commit only the rows of the delivered tokens, so the state
                # matches the transcript a later turn continues (the other accepted rows are dropped)
                self.ctx_len[s.row] -= n - room
                self.n_commit[s.row] -= n - room
            toks = toks[:room]
            if not s.done:
                s.emitted.extend(toks)
            s.generated.extend(toks)
            emitted[s.sid] = toks
            if len(s.generated) >= s.max_new_tokens and not s.done:
                s.done = True
                s.last_used = time.monotonic()
                self.active[s.row] = 0
        return emitted

    def generate(self, prompts: list[list[int]], max_new_tokens: int) -> list[list[int]]:
        for i, p in enumerate(prompts):
            self.add_session(i, p, max_new_tokens)
        while any(not s.done for s in self.sessions.values()):
            self.step()
        outs = [self.sessions[i].generated[:max_new_tokens] for i in range(len(prompts))]
        for i in range(len(prompts)):
            self.release(i)
        return outs
