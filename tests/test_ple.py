"""Per-layer n-gram embeddings on CPU: the hash contract (64-bit wrapping arithmetic, primes, offsets), history
rules (EOS, packed segments, incremental decoding), the reference layer's incremental decoding, hot tables and the
QAD student against the reference."""
import numpy as np
import pytest
import torch

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.models import ple as P
from arc_forge_2026_b200.models.reference import build_reference


def _cfg(**kw):
    return preset("tiny_cpu", ple_layer_ids=(1,), ngram_vocab_size_base=997, ple_embed_dim=256, **kw)


def _wrap(x):  # Python int -> signed 64-bit
    x &= (1 << 64) - 1
    return x - (1 << 64) if x >> 63 else x


def _ids_python(h, toks):
    """Row ids of one sequence by the contract, with Python integers."""
    out = []
    for t in range(len(toks)):
        prev, ok = [], True
        for s in range(1, h.n):
            ok = ok and t - s >= 0 and toks[t - s] != h.eos
            prev.append(toks[t - s] if ok else h.eos)
        row, mix = [], _wrap(toks[t] * h.mult[0])
        for order in range(2, h.n + 1):
            mix = _wrap(mix ^ _wrap(prev[order - 2] * h.mult[order - 1]))
            for j in range(h.hpn):
                hh = (order - 2) * h.hpn + j
                row.append(mix % h.moduli[hh] + h.offsets[hh])
        out.append(row)
    return out


def test_hash_contract_constants():
    mult = P.ngram_multipliers(248320, 3, 1234)
    assert all(m % 2 == 1 and m * (248320 - 1) < 2**63 for m in mult)
    mods = P.ngram_moduli(20_000_000, 16)
    assert mods[0] > 19_999_999 and all(P._is_prime(p) for p in mods) and mods == sorted(set(mods))
    # no prime is skipped between consecutive moduli
    assert not any(P._is_prime(q) for q in range(mods[0] + 1, mods[1]))
    assert [P._is_prime(n) for n in (1, 2, 97, 561, 7919, 2**61 - 1, 2**61 + 1)] == \
        [False, True, True, False, True, True, False]


def test_ngram_ids_match_python_integers_and_history_rules():
    cfg = _cfg(vocab_size=248320)
    h = P.NgramHash(cfg)
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, cfg.vocab_size, (40,), generator=g)
    toks[[5, 6, 20]] = cfg.eos_token_id
    ids = h.ids(toks)
    assert ids.tolist() == _ids_python(h, toks.tolist())
    # a packed row: every segment hashes like a sequence of its own
    lens = [13, 9, 18]
    starts = torch.repeat_interleave(torch.tensor([0, 13, 22]), torch.tensor(lens))
    packed = h.ids(toks, starts)
    alone = torch.cat([h.ids(toks[s:s + n]) for s, n in zip([0, 13, 22], lens)])
    assert torch.equal(packed, alone)
    # incremental: the last n-1 tokens of the history give the same rows as the whole sequence
    for cut in (1, 2, 6, 7, 21, 30):
        hist = toks[max(0, cut - (cfg.ngram_size - 1)):cut]
        assert torch.equal(h.ids(toks[cut:], history=hist), ids[cut:]), cut


@pytest.mark.parametrize("hc", [1, 4])
def test_reference_ple_layer_incremental_decoding_equals_full_forward(hc):
    cfg = _cfg(hc_count=hc, hc_lowrank=32, ple_conv_dilation=2)
    ref = build_reference(cfg, seed=1)
    ids = torch.randint(0, cfg.vocab_size, (2, 21), generator=torch.Generator().manual_seed(1))
    ids[0, 8] = cfg.eos_token_id
    with torch.no_grad():
        full = ref(ids)
        cache = ref.new_cache()
        inc = torch.cat([ref(ids[:, a:b], cache, a) for a, b in ((0, 11), (11, 16), (16, 17), (17, 21))], 1)
        assert (inc - full).abs().max() < 1e-4
        saved = ref.layers[1].ple.table.clone()
        ref.layers[1].ple.table.zero_()
        off = ref(ids)
        ref.layers[1].ple.table.copy_(saved)
    assert (off - full).abs().max() > 1e-3  # the layer does contribute


def test_causal_conv_segments_and_state():
    g = torch.Generator().manual_seed(3)
    x, w = torch.randn(12, 5, generator=g), torch.randn(5, 4, generator=g)
    starts = torch.tensor([0] * 7 + [7] * 5)
    y = P.causal_conv(x, w, 2, starts)
    assert torch.allclose(y[7:], P.causal_conv(x[7:], w, 2)) and torch.allclose(y[:7], P.causal_conv(x[:7], w, 2))
    full = P.causal_conv(x, w, 2)
    assert torch.allclose(P.causal_conv(x[9:], w, 2, state=x[3:9]), full[9:], atol=1e-6)


def test_hot_table_keeps_the_most_used_buckets():
    cfg = _cfg()
    h = P.NgramHash(cfg)
    g = torch.Generator().manual_seed(4)
    common = torch.randint(0, cfg.vocab_size, (30,), generator=g).repeat(12)  # a repeated phrase: frequent n-grams
    seqs = [common.numpy()] + [torch.randint(0, cfg.vocab_size, (60,), generator=g).numpy() for _ in range(3)]
    hot = P.build_hot(h, seqs, {2: 0.1, 3: 0.1})
    assert all(len(hot[k]) == int(h.moduli[k] * 0.1) and np.all(np.diff(hot[k]) > 0) for k in hot)
    ids = h.ids(torch.as_tensor(seqs[0]))
    rows = P.hot_rows(h, hot, ids)
    hit = rows >= 0
    assert hit[2:].all()  # every n-gram of the phrase is among the most used buckets
    base = np.concatenate([[0], np.cumsum([len(hot[k]) for k in range(len(hot))])[:-1]])
    for k in range(ids.shape[1]):
        sel = hit[:, k]
        assert torch.equal(torch.as_tensor(hot[k])[rows[sel, k] - base[k]], ids[sel, k] - h.offsets[k])
    with pytest.raises(ValueError):
        P.build_hot(h, seqs[:1], {2: 0.9, 3: 0.9})


def test_student_with_ple_follows_reference():
    from arc_forge_2026_b200.quant.gptq import rtn_quantize
    from arc_forge_2026_b200.train.student import QADStudent
    cfg = _cfg()
    ref = build_reference(cfg, seed=2)
    cs = []
    with torch.no_grad():
        for moe in ref.moe_layers():
            c13, s13 = rtn_quantize(moe.w13.float())
            c2, s2 = rtn_quantize(moe.w2.float())
            s13, s2 = s13.bfloat16().float(), s2.bfloat16().float()
            moe.w13.copy_((c13.float() - 4) * s13.repeat_interleave(128, -1))
            moe.w2.copy_((c2.float() - 4) * s2.repeat_interleave(128, -1))
            cs.append((c13, s13, c2, s2))
        ref.layers[1].ple.table.mul_(30.0)  # a visible contribution
    st = QADStudent(cfg, ref, cs, compute_dtype=torch.float32, checkpoint_layers=False)
    assert st.layers[1].ple is not None and st.layers[0].ple is None
    ids = torch.randint(0, cfg.vocab_size, (2, 30), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        rel = ((st.hidden(ids) - ref.hidden(ids)).norm() / ref.hidden(ids).norm()).item()
    assert rel < 0.2, rel
    st.hidden(ids).pow(2).mean().backward()
    assert st.layers[0].moe.w13_scales.grad is not None


def _shard_worker(rank, world, port, out):
    import os
    import torch.distributed as dist
    from arc_forge_2026_b200.parallel.ple_shard import ShardedPleTable, shard_rows
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    cfg = _cfg()
    h = P.NgramHash(cfg)
    w = torch.randn(h.rows, 16, generator=torch.Generator().manual_seed(9))
    per = shard_rows(h.rows, world)
    t = ShardedPleTable(h, w[rank * per:(rank + 1) * per], rank, world, "cpu", fp8=True, group=None)
    toks = torch.randint(0, cfg.vocab_size, (20 + 7 * rank,), generator=torch.Generator().manual_seed(rank))
    got = t.lookup_tokens(toks)
    # the unsharded table quantised per shard: every 128-row scale block lies inside one shard
    full = torch.cat([w, w.new_zeros(per * world - h.rows, 16)])
    from arc_forge_2026_b200.quant.fp8 import dequant_weight_block, quantize_weight_block
    q, s = quantize_weight_block(full)
    dense = dequant_weight_block(q, s)
    want = dense[h.ids(toks)].flatten(-2)
    torch.save({"err": (got - want).abs().max().item()}, f"{out}/r{rank}.pt")
    dist.destroy_process_group()


def test_row_sharded_table_over_gloo_ranks(tmp_path):
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_shard_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert torch.load(tmp_path / f"r{r}.pt")["err"] < 1e-6


def test_serving_side_state_commit_matches_the_reference(monkeypatch):
    """``ops.ple.ple_serve`` (prefill, then verify windows with partial acceptance and the deferred commit) gives
    every accepted row the reference layer's update; the native GEMM and lookup are replaced by torch here."""
    import arc_forge_2026_b200.ops as ops_pkg
    from arc_forge_2026_b200.ops import ple as OP

    class FakeC:
        @staticmethod
        def gemm(a, b):
            return (a.float() @ b.float().t()).to(torch.bfloat16)

    def fake_lookup(self, ext, pos, seg, ids_out=None):
        rows = []
        for p, s in zip(pos.tolist(), seg.tolist()):
            rows.append(self.hash.ids(ext[s:p + 1].long())[-1])
        ids = torch.stack(rows)
        return self.dense_rows()[ids].flatten(-2).to(torch.bfloat16)
    monkeypatch.setattr(ops_pkg, "C", lambda: FakeC())
    monkeypatch.setattr(OP.PleTable, "lookup", fake_lookup)
    cfg = _cfg(hc_count=2, hc_lowrank=32, ple_conv_dilation=1)
    ref = build_reference(cfg, seed=5)
    mod = ref.layers[1].ple
    with torch.no_grad():
        mod.table.mul_(20.0)
    w = OP.PleServeWeights.from_module(mod, "cpu", fp8=False)
    W, slots = 3, 2
    st = OP.PleServeState(w, slots, W, "cpu")
    g = torch.Generator().manual_seed(6)
    T = 40
    toks = torch.randint(0, cfg.vocab_size, (T,), generator=g)
    toks[17] = cfg.eos_token_id
    stream = torch.randn(T, 2, cfg.hidden_size, generator=g).bfloat16()
    with torch.no_grad():
        want = mod(stream.float(), toks)                        # [T, G, H] update of every position
    got = torch.zeros(T, 2, cfg.hidden_size)
    slot = torch.tensor([1])
    n_commit = torch.zeros(slots, dtype=torch.int32)
    # prefill 11 tokens
    x = stream[:11].float()
    OP.ple_serve(x, toks[:11].int(), w, st, slot, n_commit, 11, 0, True)
    got[:11] = (x.float() - stream[:11].float())
    pos, parity = 11, 0
    while pos + W <= T:
        x = stream[pos:pos + W].float()
        OP.ple_serve(x, toks[pos:pos + W].int(), w, st, slot, n_commit, W, parity, False)
        acc = int(torch.randint(1, W + 1, (1,), generator=g))  # rows accepted this cycle, committed by the next
        got[pos:pos + acc] = (x.float() - stream[pos:pos + W].float())[:acc]
        n_commit[1] = acc
        pos += acc
        parity ^= 1
    rel = ((got[:pos] - want[:pos]).norm() / want[:pos].norm()).item()
    assert rel < 1e-2, rel
    # committing every row of a window (instead of the accepted ones) breaks the history: the check sees it
    st2 = OP.PleServeState(w, slots, W, "cpu")
    x = stream[:11].float()
    OP.ple_serve(x, toks[:11].int(), w, st2, slot, torch.zeros(slots, dtype=torch.int32), 11, 0, True)
    x = stream[11:14].float()
    OP.ple_serve(x, torch.tensor([5, 6, 7], dtype=torch.int32), w, st2, slot, n_commit, W, 0, False)
    x = stream[11:14].float()
    OP.ple_serve(x, toks[11:14].int(), w, st2, slot, torch.tensor([0, 3], dtype=torch.int32), W, 1, False)
    bad = (x - stream[11:14].float())
    assert ((bad - want[11:14]).norm() / want[11:14].norm()).item() > 5e-2
