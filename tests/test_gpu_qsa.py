"""QSA kernels against their fp32 oracles: index prep, pooled page keys, per-row top-K page selection with the
page union, and block-sparse verify attention over that union."""
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


def test_prep_and_finalize_match_oracles():
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
    # pooled keys of the two complete pages (130 tokens committed -> pages 0, 1)
    bt = perm.int().view(1, P).to(dev)
    key = torch.zeros(P, 128, dtype=torch.bfloat16, device=dev)  # (session 0, page) rows
    fin = torch.zeros(1, dtype=torch.int32, device=dev)
    ctx = torch.tensor([T], dtype=torch.int32, device=dev)
    C().qsa_finalize([raw], [key], [kn.to(dev)], bt, fin, ctx, cos.to(dev), sin.to(dev), rot, 1e-6)
    torch.cuda.synchronize()
    assert int(fin.item()) == 2
    for p in range(2):
        ref = pooled_key_reference(raw.cpu()[perm[p] * PAGE:(perm[p] + 1) * PAGE], p, kn, cos, sin, rot)
        assert _rel(key.cpu()[p], ref) < 1e-2


@pytest.mark.parametrize("splits", [1, 3])
def test_select_and_sparse_attention_match_oracle(splits):
    g = torch.Generator().manual_seed(1)
    Hi, W, K, Hq, Hkv, D = 4, 5, 8, 16, 2, 256
    lens = [300, 3000, 2050, 700, 64 * 20 + 3]   # tokens incl. the W verify rows
    S = len(lens)
    maxp = max((L + PAGE - 1) // PAGE for L in lens)
    P = S * maxp + 3
    bt = torch.randperm(P, generator=g)[:S * maxp].view(S, maxp).int()
    kc = torch.randn(P, Hkv, PAGE, D, generator=g).bfloat16()
    vc = torch.randn(P, Hkv, PAGE, D, generator=g).bfloat16()
    keys = torch.randn(S * maxp, 128, generator=g).bfloat16()  # pooled keys by (session, page)
    idx_q = torch.randn(S * W, Hi, 128, generator=g).bfloat16()
    q = torch.randn(S * W, Hq, D, generator=g).bfloat16()
    gate = torch.randn(S * W, Hq, D, generator=g).bfloat16()
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    fin = torch.tensor([(L - W) // PAGE for L in lens], dtype=torch.int32)  # committed pages are finalised
    ws = QsaWorkspace(S, W, K, maxp, Hi, dev)
    ws.idx_q.copy_(idx_q)
    out = torch.zeros(S * W, Hq, D, dtype=torch.bfloat16, device=dev)
    qsa_attention(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), seq_lens.to(dev), fin.to(dev), keys.to(dev), ws,
                  out, gate.to(dev), Hq * D, D, splits=splits)
    torch.cuda.synchronize()
    check_status()
    for s in range(S):
        F = int(fin[s])
        logical_keys = keys[s * maxp:s * maxp + F]
        rows = select_reference(idx_q[s * W:(s + 1) * W], logical_keys, F, lens[s], W, K)
        n = int(ws.u_count[s])
        lp, m = ws.u_lpage[s, :n].cpu().tolist(), ws.u_mask[s, :n].cpu().tolist()
        got_rows = [sorted(p for p, mm in zip(lp, m) if mm >> r & 1) for r in range(W)]
        assert got_rows == rows, (s, got_rows, rows)
        assert lp == sorted(lp) and len(set(lp)) == n
        ref = attention_reference(q[s * W:(s + 1) * W], kc, vc, bt[s], lens[s], W, rows, gate[s * W:(s + 1) * W])
        assert _rel(out[s * W:(s + 1) * W].cpu(), ref) < 1e-2


def test_decision_replay_forces_recorded_selections(tmp_path):
    """A recorded run's page unions, forced into a second run with different index queries, reproduce the first
    run's output exactly; the log survives a save / load."""
    from arc_forge_2026_b200.ops.qsa import DecisionReplay
    g = torch.Generator().manual_seed(5)
    Hi, W, K, Hq, Hkv, D = 4, 5, 8, 16, 2, 256
    lens = [900, 2000, 1500]
    S = len(lens)
    maxp = max((L + PAGE - 1) // PAGE for L in lens)
    P = S * maxp + 3
    bt = torch.randperm(P, generator=g)[:S * maxp].view(S, maxp).int().to(dev)
    kc = torch.randn(P, Hkv, PAGE, D, generator=g).bfloat16().to(dev)
    vc = torch.randn(P, Hkv, PAGE, D, generator=g).bfloat16().to(dev)
    keys = torch.randn(S * maxp, 128, generator=g).bfloat16().to(dev)
    q = torch.randn(S * W, Hq, D, generator=g).bfloat16().to(dev)
    seq_lens = torch.tensor(lens, dtype=torch.int32).to(dev)
    fin = torch.tensor([(L - W) // PAGE for L in lens], dtype=torch.int32).to(dev)
    ws = QsaWorkspace(S, W, K, maxp, Hi, dev)
    outs = []
    rec = DecisionReplay("record")
    for i, mode in enumerate((rec, None, "forced")):
        ws.idx_q.copy_(torch.randn(S * W, Hi, 128, generator=torch.Generator().manual_seed(10 + min(i, 1))).bfloat16())
        out = torch.zeros(S * W, Hq, D, dtype=torch.bfloat16, device=dev)
        rp = mode
        if mode == "forced":
            rec.save(tmp_path / "dec.pt")
            rp = DecisionReplay.load(tmp_path / "dec.pt", dev)
        qsa_attention(q, kc, vc, bt, seq_lens, fin, keys, ws, out, replay=rp)
        outs.append(out)
    torch.cuda.synchronize()
    check_status()
    assert len(rec.log) == 1
    assert not torch.equal(outs[0], outs[1])   # other index queries select other pages
    assert torch.equal(outs[0], outs[2])       # forced: the recorded selection, bit for bit


def test_sparse_attention_over_an_nvfp4_cache():
    """QSA sparse verify attention reading an NVFP4 cache equals the same selection over the dequantised bf16
    pages."""
    from arc_forge_2026_b200.ops.attention import nvfp4_dequant
    g = torch.Generator().manual_seed(5)
    Hi, W, K, Hq, Hkv, D = 4, 5, 8, 16, 2, 256
    lens = [300, 3000, 2050]
    S = len(lens)
    maxp = max((L + PAGE - 1) // PAGE for L in lens)
    P = S * maxp + 3
    bt = torch.randperm(P, generator=g)[:S * maxp].view(S, maxp).int().to(dev)
    codes = [torch.randint(0, 256, (P, Hkv, PAGE, D // 2), generator=g, dtype=torch.uint8).to(dev) for _ in range(2)]
    scales = [(torch.rand(P, Hkv, PAGE, D // 16, generator=g) * 0.75 + 0.25).to(torch.float8_e4m3fn)
              .view(torch.uint8).to(dev) for _ in range(2)]
    kd, vd = (nvfp4_dequant(c, s).bfloat16() for c, s in zip(codes, scales))
    keys = torch.randn(S * maxp, 128, generator=g).bfloat16().to(dev)
    idx_q = torch.randn(S * W, Hi, 128, generator=g).bfloat16().to(dev)
    q = torch.randn(S * W, Hq, D, generator=g).bfloat16().to(dev)
    seq_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    fin = torch.tensor([(L - W) // PAGE for L in lens], dtype=torch.int32, device=dev)
    outs = []
    for kv in ((codes[0], codes[1], (scales[0], scales[1])), (kd, vd, None)):
        ws = QsaWorkspace(S, W, K, maxp, Hi, dev)
        ws.idx_q.copy_(idx_q)
        out = torch.zeros(S * W, Hq, D, dtype=torch.bfloat16, device=dev)
        qsa_attention(q, kv[0], kv[1], bt, seq_lens, fin, keys, ws, out, None, 0, 0, splits=2, kv_scales=kv[2])
        outs.append(out)
    torch.cuda.synchronize()
    check_status()
    assert _rel(outs[0], outs[1]) < 1e-2
