"""The native PLE lookup (hash + gather + dequantisation in one kernel) against the torch contract: e4m3 and bf16
tables, packed segments, EOS resets, decode-style history, hot tables, row shards and the bounds check."""
import pytest
import torch

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.models.ple import NgramHash, build_hot
from arc_forge_2026_b200.ops import check_status
from arc_forge_2026_b200.ops.ple import PleTable

pytestmark = pytest.mark.gpu
dev = "cuda"


def _setup(head_dim=160, base=4001, seed=0):
    cfg = preset("tiny_cpu", vocab_size=248320, ple_layer_ids=(1,), ngram_vocab_size_base=base,
                 ple_embed_dim=16 * head_dim)
    h = NgramHash(cfg)
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(h.rows, head_dim, generator=g)
    toks = torch.randint(0, cfg.vocab_size, (300,), generator=g)
    toks[[3, 4, 100, 250]] = cfg.eos_token_id
    return cfg, h, w, toks


@pytest.mark.parametrize("fp8", [True, False])
def test_lookup_matches_the_contract(fp8):
    cfg, h, w, toks = _setup()
    t = PleTable.from_weight(h, w, dev, fp8=fp8)
    lens = [120, 64, 116]
    seg = torch.repeat_interleave(torch.tensor([0, 120, 184]), torch.tensor(lens))
    got = t.lookup_tokens(toks.to(dev), seg.to(dev))
    torch.cuda.synchronize()
    check_status()
    want = t.lookup_reference(toks, seg)
    assert torch.equal(got.float().cpu(), want.bfloat16().float())


def test_lookup_with_decode_history_hot_table_and_shards():
    cfg, h, w, toks = _setup(head_dim=32, base=2003, seed=1)
    # decode layout: per session [last n-1 tokens | step tokens]
    hist, step = toks[40:42], toks[42:47]
    ext = torch.cat([hist, step, toks[90:91], toks[91:95]]).int()   # session 2 has one history token
    pos = torch.tensor([2, 3, 4, 5, 6, 8, 9, 10, 11])
    seg = torch.tensor([0] * 5 + [7] * 4)
    full = PleTable.from_weight(h, w, dev, fp8=True)
    ids_out = torch.empty(9, 16, dtype=torch.int64, device=dev)
    got = full.lookup(ext.to(dev), pos.to(dev), seg.to(dev), ids_out=ids_out)
    want_ids = torch.cat([h.ids(step, history=hist), h.ids(toks[91:95], history=toks[90:91])])
    assert torch.equal(ids_out.cpu(), want_ids)
    dense = full.dense_rows().cpu()
    assert torch.equal(got.float().cpu(), dense[want_ids].flatten(-2).bfloat16().float())
    # hot table: kept buckets read their rows, the rest zeros
    hot = build_hot(h, [toks.numpy()], {2: 0.05, 3: 0.05})
    ht = PleTable.from_weight(h, w, dev, fp8=False, hot=hot)
    assert torch.equal(ht.lookup_tokens(toks.to(dev)).float().cpu(), ht.lookup_reference(toks).bfloat16().float())
    # the same table split into 3 row shards (pointers in row order) reads the same rows
    bf = w.to(dev, torch.bfloat16)
    rps = 128 * ((h.rows + 3 * 128 - 1) // (3 * 128))
    parts = [bf[i * rps:(i + 1) * rps].contiguous() for i in range(3)]
    sharded = PleTable(h, parts[0], None, shards=[(p.data_ptr(), 0) for p in parts], rows_per_shard=rps,
                       table_rows=h.rows)
    one = PleTable(h, bf, None)
    assert torch.equal(sharded.lookup_tokens(toks.to(dev)), one.lookup_tokens(toks.to(dev)))
    torch.cuda.synchronize()
    check_status()


def test_lookup_bounds_check_reports_and_reads_zeros():
    cfg, h, w, toks = _setup(head_dim=32, base=2003, seed=2)
    t = PleTable.from_weight(h, w, dev, fp8=False)
    ext = toks[:10].int().to(dev)
    out = t.lookup(ext, torch.tensor([3, 40], device=dev), torch.tensor([0, 0], device=dev))
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="out of bounds"):
        check_status()
    assert out[1].abs().max() == 0 and out[0].abs().max() > 0
