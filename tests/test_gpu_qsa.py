"""QSA kernels against their fp32 oracles: index prep, pooled block keys, per-row top-K block selection (blocks
completed inside the verify window pooled on the fly) with the per-session union, and block-sparse verify attention
over that union: 64-token blocks (a block is a page) and sub-page blocks (4 tokens: the reference model's QSA)
gathered into the tcgen05 kernel's tiles."""
import math

import pytest
import torch

from arc_forge_2026_b200.models.reference import rope_cos_sin
from arc_forge_2026_b200.ops import C, check_status
from arc_forge_2026_b200.ops.qsa import (PAGE, QsaWorkspace, attention_reference, pooled_key_reference,
                                         prep_reference, qsa_attention, select_reference)

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _tables(rot=64, n=8192):
    cos, sin = rope_cos_sin(torch.arange(n), rot, 1.0e7)
    return cos.contiguous(), sin.contiguous()


class _Case:
    """Sessions with random KV pages, raw index keys per slot, stored pooled keys of the committed blocks (random)
    and index queries; ``keys_of(s)`` gives the logical keys the selection scores (stored, then pooled on the fly
    for blocks completed inside the window)."""

    def __init__(self, lens, W, Hq, Hkv, D, block, seed, Hi=4, rot=64):
        g = torch.Generator().manual_seed(seed)
        self.lens, self.W, self.block, self.Hi, self.rot = lens, W, block, Hi, rot
        S = self.S = len(lens)
        self.maxp = max((L + PAGE - 1) // PAGE for L in lens)
        P = S * self.maxp + 3
        self.bt = torch.randperm(P, generator=g)[:S * self.maxp].view(S, self.maxp).int()
        self.kc = torch.randn(P, Hkv, PAGE, D, generator=g).bfloat16()
        self.vc = torch.randn(P, Hkv, PAGE, D, generator=g).bfloat16()
        self.raw = torch.randn(P * PAGE, 128, generator=g).bfloat16()
        self.kn = (torch.randn(128, generator=g) * 0.1).bfloat16()
        self.mb = self.maxp * (PAGE // block)
        self.keys = torch.randn(S * self.mb, 128, generator=g).bfloat16()  # pooled keys by (session, block)
        self.idx_q = torch.randn(S * W, Hi, 128, generator=g).bfloat16()
        self.q = torch.randn(S * W, Hq, D, generator=g).bfloat16()
        self.gate = torch.randn(S * W, Hq, D, generator=g).bfloat16()
        self.seq_lens = torch.tensor(lens, dtype=torch.int32)
        self.fin = torch.tensor([(L - W) // block for L in lens], dtype=torch.int32)  # committed blocks
        self.cos, self.sin = _tables(rot)

    def keys_of(self, s):
        F, n = int(self.fin[s]), self.lens[s] // self.block
        out = [self.keys[s * self.mb + b].float() for b in range(F)]
        for b in range(F, n):
            toks = torch.arange(b * self.block, (b + 1) * self.block)
            slots = self.bt[s][toks // PAGE].long() * PAGE + toks % PAGE
            out.append(pooled_key_reference(self.raw[slots], b, self.kn, self.cos, self.sin, self.rot,
                                            block=self.block).bfloat16().float())
        return torch.stack(out) if out else torch.zeros(0, 128)

    def run(self, K, ws=None, splits=1, replay=None, kv=None, idx_q=None):
        ws = ws or QsaWorkspace(self.S, self.W, K, self.maxp, self.Hi, dev, block=self.block)
        ws.idx_q[:self.S * self.W].copy_(self.idx_q if idx_q is None else idx_q)
        Hq, D = self.q.shape[1], self.q.shape[2]
        out = torch.zeros(self.S * self.W, Hq, D, dtype=torch.bfloat16, device=dev)
        kc, vc, scales = kv or (self.kc.to(dev), self.vc.to(dev), None)
        qsa_attention(self.q.to(dev), kc, vc, self.bt.to(dev), self.seq_lens.to(dev), self.fin.to(dev),
                      self.keys.to(dev), ws, out, self.gate.to(dev), Hq * D, D, splits=splits, replay=replay,
                      kv_scales=scales, raw=self.raw.to(dev), k_norm=self.kn.to(dev),
                      rope=(self.cos.to(dev), self.sin.to(dev)), rot=self.rot, eps=1e-6)
        return out, ws


@pytest.mark.parametrize("block", [64, 4])
def test_prep_and_finalize_match_oracles(block):
    g = torch.Generator().manual_seed(0)
    Hi, rot, T, P = 4, 64, 130, 6
    cos, sin = _tables(rot)
    off = 64  # index columns start after some other projection columns
    proj = torch.randn(T, off + (Hi + 1) * 128, generator=g).bfloat16()
    pos = torch.arange(T, dtype=torch.int32)
    perm = torch.randperm(P, generator=g)
    slots = (perm[pos.long() // PAGE] * PAGE + pos.long() % PAGE).int()
    qn = (torch.randn(128, generator=g) * 0.1).bfloat16()
    kn = (torch.randn(128, generator=g) * 0.1).bfloat16()
    idx_q = torch.zeros(T, Hi, 128, dtype=torch.bfloat16, device=dev)
    raw = torch.zeros(P * PAGE, 128, dtype=torch.bfloat16, device=dev)
    C().qsa_prep(proj.to(dev), off, pos.to(dev), slots.to(dev), qn.to(dev), cos.to(dev), sin.to(dev), 1e-6, Hi, rot,
                 idx_q, raw)
    q_ref, raw_ref = prep_reference(proj[:, off:], pos, qn, cos, sin, Hi, rot)
    assert _rel(idx_q.cpu(), q_ref) < 1e-2
    assert torch.equal(raw.cpu()[slots.long()], raw_ref.bfloat16())
    # pooled keys of the complete blocks (130 tokens committed)
    bt = perm.int().view(1, P).to(dev)
    nb = T // block
    key = torch.zeros(P * (PAGE // block), 128, dtype=torch.bfloat16, device=dev)  # (session 0, block) rows
    fin = torch.zeros(1, dtype=torch.int32, device=dev)
    ctx = torch.tensor([T], dtype=torch.int32, device=dev)
    C().qsa_finalize([raw], [key], [kn.to(dev)], bt, fin, ctx, cos.to(dev), sin.to(dev), rot, 1e-6, block)
    torch.cuda.synchronize()
    assert int(fin.item()) == nb
    for b in range(nb):
        toks = torch.arange(b * block, (b + 1) * block)
        ref = pooled_key_reference(raw.cpu()[(perm[toks // PAGE] * PAGE + toks % PAGE).long()], b, kn, cos, sin, rot,
                                   block=block)
        assert _rel(key.cpu()[b], ref) < 1e-2, b
    assert not key.cpu()[nb:].any()  # the incomplete block has no key yet


@pytest.mark.parametrize("block,K,splits,Hq,Hkv,D,W", [
    (64, 8, 1, 16, 2, 256, 5), (64, 8, 3, 16, 2, 256, 5),      # page blocks (BASELINE config 5 shape)
    (4, 64, 1, 32, 8, 128, 5), (4, 64, 2, 32, 8, 128, 5),      # 4-token blocks, GQA 4, D 128
    (4, 48, 2, 24, 2, 256, 5),                                 # the reference model's heads: GQA 12, D 256
    (4, 48, 2, 24, 2, 256, 8),                                 # 8 verify rows x 12 heads: two row runs per KV head
    (16, 16, 1, 32, 8, 128, 3), (64, 8, 2, 16, 2, 256, 8)])
def test_select_and_sparse_attention_match_oracle(block, K, splits, Hq, Hkv, D, W):
    lens = [300, 3000, 2050, 200, 64 * 20 + 3, 7]   # tokens incl. the W verify rows
    cs = _Case(lens, W, Hq, Hkv, D, block, seed=1)
    out, ws = cs.run(K, splits=splits)
    torch.cuda.synchronize()
    check_status()
    for s in range(cs.S):
        rows = select_reference(cs.idx_q[s * W:(s + 1) * W], cs.keys_of(s), lens[s], W, K, block=block)
        n = int(ws.u_count[s])
        lp, m = ws.u_lpage[s, :n].cpu().tolist(), ws.u_mask[s, :n].cpu().tolist()
        got_rows = [sorted(p for p, mm in zip(lp, m) if mm >> r & 1) for r in range(W)]
        assert got_rows == rows, (s, got_rows, rows)
        assert lp == sorted(lp) and len(set(lp)) == n
        ref = attention_reference(cs.q[s * W:(s + 1) * W], cs.kc, cs.vc, cs.bt[s], lens[s], W, rows,
                                  cs.gate[s * W:(s + 1) * W], block=block)
        assert _rel(out[s * W:(s + 1) * W].cpu(), ref) < 1e-2, s
    assert not ws.sel.any()  # the union cleared its marks
    # the per-row CUDA-core scoring (no tensor-core scores) selects the same blocks
    ws2 = QsaWorkspace(cs.S, W, K, cs.maxp, cs.Hi, dev, block=block)
    ws2.scores = None
    cs.run(K, ws=ws2, splits=splits)
    torch.cuda.synchronize()
    for s in range(cs.S):
        n = int(ws.u_count[s])
        assert int(ws2.u_count[s]) == n
        assert torch.equal(ws2.u_lpage[s, :n], ws.u_lpage[s, :n]) and torch.equal(ws2.u_mask[s, :n], ws.u_mask[s, :n])


def test_decision_replay_forces_recorded_selections(tmp_path):
    """A recorded run's block unions, forced into a second run with different index queries, reproduce the first
    run's output exactly; the log survives a save / load."""
    from arc_forge_2026_b200.ops.qsa import DecisionReplay
    cs = _Case([900, 2000, 1500], 5, 16, 2, 256, 64, seed=5)
    outs = []
    rec = DecisionReplay("record")
    ws = None
    for i, mode in enumerate((rec, None, "forced")):
        iq = torch.randn(cs.S * cs.W, cs.Hi, 128, generator=torch.Generator().manual_seed(10 + min(i, 1))).bfloat16()
        rp = mode
        if mode == "forced":
            rec.save(tmp_path / "dec.pt")
            rp = DecisionReplay.load(tmp_path / "dec.pt", dev)
        out, ws = cs.run(8, ws=ws, replay=rp, idx_q=iq)
        outs.append(out)
    torch.cuda.synchronize()
    check_status()
    assert len(rec.log) == 1
    assert not torch.equal(outs[0], outs[1])   # other index queries select other blocks
    assert torch.equal(outs[0], outs[2])       # forced: the recorded selection, bit for bit


def test_sparse_attention_over_an_nvfp4_cache():
    """QSA sparse verify attention reading an NVFP4 cache equals the same selection over the dequantised bf16
    pages."""
    from arc_forge_2026_b200.ops.attention import nvfp4_dequant
    cs = _Case([300, 3000, 2050], 5, 16, 2, 256, 64, seed=5)
    g = torch.Generator().manual_seed(6)
    P, Hkv, D = cs.kc.shape[0], 2, 256
    codes = [torch.randint(0, 256, (P, Hkv, PAGE, D // 2), generator=g, dtype=torch.uint8).to(dev) for _ in range(2)]
    scales = [(torch.rand(P, Hkv, PAGE, D // 16, generator=g) * 0.75 + 0.25).to(torch.float8_e4m3fn)
              .view(torch.uint8).to(dev) for _ in range(2)]
    kd, vd = (nvfp4_dequant(c, s).bfloat16() for c, s in zip(codes, scales))
    outs = []
    for kv in ((codes[0], codes[1], (scales[0], scales[1])), (kd, vd, None)):
        out, _ = cs.run(8, splits=2, kv=kv)
        outs.append(out)
    torch.cuda.synchronize()
    check_status()
    assert _rel(outs[0], outs[1]) < 1e-2


@pytest.mark.parametrize("W", [5, 8])
def test_dense_attention_with_more_than_64_rows(W):
    """24 query heads over 2 KV heads (GQA 12) with 8 verify positions = 96 rows per KV head: the tcgen05 kernel runs
    them as two CTAs of <= 64 rows and matches the fp32 oracle."""
    from arc_forge_2026_b200.ops.attention import paged_attention, paged_attention_reference
    g = torch.Generator().manual_seed(9)
    lens = [700, 1500, 64 * 3 + W]
    S, Hq, Hkv, D = len(lens), 24, 2, 256
    maxp = max((L + PAGE - 1) // PAGE for L in lens)
    P = S * maxp + 1
    bt = torch.randperm(P, generator=g)[:S * maxp].view(S, maxp).int()
    kc = torch.randn(P, Hkv, PAGE, D, generator=g).bfloat16()
    vc = torch.randn(P, Hkv, PAGE, D, generator=g).bfloat16()
    q = torch.randn(S * W, Hq, D, generator=g).bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32)
    for splits in (1, 3):
        out = torch.zeros(S * W, Hq, D, dtype=torch.bfloat16, device=dev)
        paged_attention(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), sl.to(dev), W, out, splits=splits)
        torch.cuda.synchronize()
        check_status()
        ref = paged_attention_reference(q, kc, vc, bt, sl, W)
        assert _rel(out.cpu(), ref) < 1e-2, splits


def test_sub_page_blocks_match_page_mode_when_every_block_is_kept():
    """With K above every row's block count, 4-token blocks select everything: the gathered attention equals the
    dense tcgen05 kernel's causal verify output."""
    from arc_forge_2026_b200.ops.attention import paged_attention
    cs = _Case([300, 700, 64 * 5 + 3], 5, 32, 8, 128, 4, seed=7)
    out, _ = cs.run(4096, splits=2)
    ref = torch.zeros_like(out)
    paged_attention(cs.q.to(dev), cs.kc.to(dev), cs.vc.to(dev), cs.bt.to(dev), cs.seq_lens.to(dev), cs.W, ref,
                    gate=cs.gate.to(dev), gate_ld=32 * 128, gate_head_stride=128)
    torch.cuda.synchronize()
    check_status()
    assert _rel(out, ref) < 5e-3
