"""End-to-end GPU tests of the hybrid model and the speculative engine (tiny shape)."""
import dataclasses

import pytest
import torch

from arc_forge_2026_b200.config import FULL, ServeConfig, drafter_preset, preset
from arc_forge_2026_b200.models.drafter import Drafter
from arc_forge_2026_b200.models.hybrid import HybridModel
from arc_forge_2026_b200.models.reference import build_reference
from arc_forge_2026_b200.ops import check_status
from arc_forge_2026_b200.quant.gptq import rtn_quantize
from arc_forge_2026_b200.serve.engine import SpecEngine

pytestmark = pytest.mark.gpu
dev = "cuda"


def _models(seed=0, name="tiny_gpu", **over):
    cfg = preset(name, **over)
    ref = build_reference(cfg, seed=seed)
    with torch.no_grad():
        ref.lm_head.weight.mul_(40.0)  # peaky logits: argmax far from ties
        for L in ref.layers:
            if L.ple is not None:
                L.ple.table.mul_(50.0)  # a PLE layer that visibly moves the stream
        qs = []
        for moe in ref.moe_layers():  # INT3 experts in both models
            c13, s13 = rtn_quantize(moe.w13.float())
            c2, s2 = rtn_quantize(moe.w2.float())
            s13, s2 = s13.bfloat16(), s2.bfloat16()
            moe.w13.copy_((c13.float() - 4) * s13.float().repeat_interleave(128, -1))
            moe.w2.copy_((c2.float() - 4) * s2.float().repeat_interleave(128, -1))
            qs.append((c13, s13, c2, s2))
    return cfg, ref, HybridModel.from_reference(ref, dev, qs)


def test_prefill_logits_match_reference():
    cfg, ref, model = _models()
    eng = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy"), 2, 1024)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (300,), generator=g).tolist()
    eng.add_session(0, prompt, 4)
    torch.cuda.synchronize()
    check_status()
    ref_logits = ref(torch.tensor([prompt]))[0, -1]
    first = int(ref_logits.argmax())
    assert eng.sessions[0].generated[0] == first


def test_spec_greedy_equals_plain_greedy():
    cfg, ref, model = _models(1)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 130, 9)]
    plain = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy"), 4, 1024)
    out_plain = plain.generate(prompts, 40)
    drafter = Drafter(drafter_preset("tiny"), cfg.hidden_size, cfg.vocab_size, dev, draft_vocab=4096)
    spec = SpecEngine(model, drafter, ServeConfig(spec_k=4, accept_mode="greedy"), 4, 1024)
    out_spec = spec.generate(prompts, 40)
    torch.cuda.synchronize()
    check_status()
    for a, b in zip(out_plain, out_spec):
        assert a == b
    # reference greedy decode of the first prompt agrees with the engine on the leading tokens
    toks, _ = ref.greedy_decode(torch.tensor([prompts[0]]), 8)
    assert toks[0].tolist()[:4] == out_plain[0][:4]


@pytest.mark.parametrize("spec_k", [0, 4])
def test_qwen38fn_qsa_decode_matches_reference(spec_k):
    """The reference model's own shape (24Q/2KV x 256 attention, 16/48-head GDN, 4 hyper-connection branches, PLE at
    layer 2, QSA over 4-token blocks) at reduced width, depth and n-gram table, top-16 blocks so decoding runs past the dense range (64
    tokens). Teacher-forced against the fp32 reference with its QSA selection: every token the engine emits (plain
    decode, or speculative verify of 5 rows) is the reference's argmax up to a near-tie, and the engine's QSA prefill
    of the whole sequence gives the reference's logits."""
    cfg, ref, model = _models(4, "qwen38fn", num_layers=4, hidden_size=512, vocab_size=4096, num_experts=16,
                              qsa_topk=16, ngram_vocab_size_base=4096, ple_embed_dim=512)
    assert cfg.qsa_block == 4 and cfg.hc_count == 4
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, cfg.vocab_size, (50,), generator=g).tolist()
    drafter = (Drafter(drafter_preset("tiny"), cfg.hidden_size, cfg.vocab_size, dev, draft_vocab=4096)
               if spec_k else None)
    eng = SpecEngine(model, drafter, ServeConfig(spec_k=spec_k, accept_mode="greedy"), 2, 1024)
    assert eng.qsa is not None and eng.qsa.ws.block == 4
    out = eng.generate([prompt], 60)[0]
    torch.cuda.synchronize()
    check_status()
    seq = prompt + out
    with torch.no_grad():
        ref_logits = ref(torch.tensor([seq]))[0].float()
        dense_cfg = dataclasses.replace(cfg, qsa_topk=1 << 20)  # same weights, every block kept
        for lay in ref.layers:
            if lay.kind == FULL:
                lay.mixer.cfg = dense_cfg
        dense_logits = ref(torch.tensor([seq]))[0].float()
    L = len(prompt)
    # decode: each emitted token is the reference's best up to a near-tie (a few flips of near-tied block scores
    # between the bf16 engine and the fp32 reference are expected: a bf16 copy of the reference shows them too)
    far = [i for i, t in enumerate(out)
           if float(ref_logits[L - 1 + i].max() - ref_logits[L - 1 + i][t]) >
           0.03 * float(ref_logits[L - 1 + i].max() - ref_logits[L - 1 + i].median())]
    assert len(far) <= len(out) // 10, far
    # prefill of the whole sequence through the engine (QSA row sets past 64 tokens) against both references:
    # close to the QSA one (bf16-level error), far from the dense one past the dense range
    rows = []
    eng.score(seq, lambda h, s: rows.append(model.logits(h, fp32=True).float().cpu()))
    torch.cuda.synchronize()
    check_status()
    got = torch.cat(rows)[:len(seq)]

    def rel(x, y):
        return (x - y).norm(dim=-1) / y.norm(dim=-1)
    e_qsa, e_dense = rel(got, ref_logits), rel(got, dense_logits)
    # (the engine's own bf16 / INT3 error is ~4 % already in the dense range; a flipped near-tie adds an outlier)
    assert e_qsa.median() < 0.06 and e_qsa[70:].median() < 0.06, e_qsa
    assert e_qsa[70:].median() < 0.4 * e_dense[70:].median(), (e_qsa[70:], e_dense[70:])
    assert (got.argmax(-1) == ref_logits.argmax(-1)).float().mean() > 0.85


def test_qwen38fn_full_width_constructs_and_decodes():
    """preset('qwen38fn') at full width (hidden 2560, 512 experts x 640 INT3, vocab 248,320, the full n-gram table
    of the PLE layer in e4m3, top-512 of 4-token blocks), 4 of its 48 layers: random init on the GPU, prefill (one
    prompt past the 2,048-token dense range) and speculative decode through the engine."""
    cfg = preset("qwen38fn", num_layers=4)
    model = HybridModel.random(cfg, dev, seed=5)
    drafter = Drafter(drafter_preset("tiny"), cfg.hidden_size, cfg.vocab_size, dev, draft_vocab=4096)
    eng = SpecEngine(model, drafter, ServeConfig(spec_k=4, accept_mode="greedy"), 2, 4096)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (300, 2100)]
    out = eng.generate(prompts, 16)
    torch.cuda.synchronize()
    check_status()
    assert [len(o) for o in out] == [16, 16]
    assert all(0 <= t < cfg.vocab_size for o in out for t in o)


def test_bernoulli_acceptance_and_graph_replay():
    cfg, ref, model = _models(2)
    drafter = Drafter(drafter_preset("tiny"), cfg.hidden_size, cfg.vocab_size, dev, draft_vocab=4096)
    scfg = ServeConfig(spec_k=4, accept_mode="bernoulli", accept_prob=0.7, seed=3)
    eng = SpecEngine(model, drafter, scfg, 8, 2048)
    g = torch.Generator().manual_seed(2)
    for i in range(8):
        eng.add_session(i, torch.randint(0, cfg.vocab_size, (50 + 10 * i,), generator=g).tolist(), 1000)
    eng.capture()
    emitted = 0
    for _ in range(40):
        emitted += sum(len(v) for v in eng.step().values())
    torch.cuda.synchronize()
    check_status()
    per_cycle = emitted / (40 * 8)
    expected = 1 + 0.7 + 0.7**2 + 0.7**3 + 0.7**4
    assert abs(per_cycle - expected) < 0.25, per_cycle


def test_qsa_engine_equals_dense_while_all_pages_fit_and_runs_sparse_beyond():
    cfg = preset("tiny_gpu", qsa_block=64, qsa_topk=4)
    model = HybridModel.random(cfg, dev, seed=3)
    with torch.no_grad():
        model.lm_head.mul_(40.0)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (100, 150)]
    scfg = ServeConfig(spec_k=0, accept_mode="greedy")
    dense = SpecEngine(model, None, scfg, 2, 1024)
    dense.qsa = None
    out_dense = dense.generate(prompts, 30)
    sparse = SpecEngine(model, None, scfg, 2, 1024)
    assert sparse.qsa is not None
    out_qsa = sparse.generate(prompts, 30)  # <= 3 finalised pages < top-4: QSA selects everything
    torch.cuda.synchronize()
    check_status()
    # same attention up to the order of the split-KV sums (the QSA union is split in 4, the dense path by its plan):
    # greedy decoding agrees until a near-tie of two logits, which sets in late if at all
    for a, b in zip(out_qsa, out_dense):
        same = next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), len(a))
        assert same >= 16, (same, a, b)
    long_prompt = torch.randint(0, cfg.vocab_size, (700,), generator=g).tolist()  # 10 pages > top-4: sparse
    out = sparse.generate([long_prompt], 20)
    torch.cuda.synchronize()
    check_status()
    assert len(out[0]) == 20 and all(0 <= t < cfg.vocab_size for t in out[0])
    assert int(sparse.qsa.fin[0]) >= 10


@pytest.mark.parametrize("fp8", [False, True])
def test_hisparse_offload_equals_on_device_qsa(fp8):
    """Same QSA engine with the KV history in pinned host memory (bf16: exact; e4m3 pool: runs, close)."""
    cfg = preset("tiny_gpu", qsa_block=64, qsa_topk=2)
    model = HybridModel.random(cfg, dev, seed=4)
    with torch.no_grad():
        model.lm_head.mul_(40.0)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (700, 450)]
    base = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy"), 2, 1024)
    out_base = base.generate(prompts, 80)  # crosses page boundaries: write-back and fetch both run
    off = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy", hisparse=True, hisparse_fp8=fp8,
                                              hisparse_hot_blocks=4), 2, 1024)
    out_off = off.generate(prompts, 80)
    torch.cuda.synchronize()
    check_status()
    assert int(off.hs.cycle.item()) >= 79  # the first token comes from the prefill
    if not fp8:
        assert out_off == out_base
    else:
        agree = sum(a == b for x, y in zip(out_off, out_base) for a, b in zip(x, y)) / (2 * 80)
        assert agree > 0.5
    off.hs.close()


def test_trained_drafter_export_matches_serving_proposals():
    """The PyTorch drafter twin and the serving drafter (native kernels) propose the same block after export."""
    from arc_forge_2026_b200.train.drafter_train import DrafterTrain
    dcfg = drafter_preset("tiny")
    V, Ht, Lc = 4096, 256, 70
    g = torch.Generator().manual_seed(7)
    serving = Drafter(dcfg, Ht, V, dev, draft_vocab=V)
    twin = DrafterTrain(dcfg, Ht, V, serving.draft_vocab.long().cpu(), seed=3)
    with torch.no_grad():
        twin.lm_head.mul_(50.0)  # peaky logits: argmax far from bf16 ties
    twin.export_to(serving)
    tokens = torch.randint(0, V, (Lc + dcfg.k + 1,), generator=g)
    hidden = torch.randn(Lc + dcfg.k + 1, Ht, generator=g) * 0.5
    with torch.no_grad():
        want = twin.draft_vocab[twin.block_logits(tokens, hidden.bfloat16().float(),
                                                  torch.tensor([Lc])).argmax(-1)[0]].tolist()
    kv = serving.new_kv_cache(4)
    ws = serving.new_workspace(128)
    i32 = dict(dtype=torch.int32, device=dev)
    pos = torch.arange(Lc, **i32)
    serving.inject(tokens[:Lc].int().to(dev), hidden[:Lc].bfloat16().to(dev), pos, pos.clone(), kv, ws)
    blk = torch.full((dcfg.k,), serving.mask_id, **i32)
    blk[0] = int(tokens[Lc])
    bpos = torch.arange(Lc, Lc + dcfg.k, **i32)
    out = torch.zeros(1, dcfg.k, **i32)
    serving.propose(blk, hidden[Lc - 1:Lc].bfloat16().to(dev), bpos, bpos.clone(), torch.arange(4, **i32).view(1, 4),
                    torch.tensor([Lc + dcfg.k], **i32), kv, ws, out, 1, max_pages=4)
    torch.cuda.synchronize()
    check_status()
    assert out[0].tolist() == want


def test_drafter_with_candidate_selector_export_matches_serving_proposals(tmp_path):
    """A drafter with a trained-looking candidate selector (non-zero successor codebook, so the selector reorders
    the unary top-k): published through a drafter directory, the serving drafter's greedy chain equals the twin's."""
    from arc_forge_2026_b200.train.drafter_tools import save_dir
    from arc_forge_2026_b200.train.drafter_train import DrafterTrain
    dcfg = drafter_preset("tiny", selector_top_k=8, selector_rank=16)
    V, Ht, Lc = 4096, 256, 70
    g = torch.Generator().manual_seed(11)
    twin = DrafterTrain(dcfg, Ht, V, torch.randperm(V, generator=g)[:2048].sort().values, seed=5)
    with torch.no_grad():
        twin.lm_head.mul_(50.0)
        twin.selector.succ_codebook.normal_(0, 2.0, generator=g)
        twin.selector.pred_codebook.normal_(0, 2.0, generator=g)
        twin.selector.proj.normal_(0, 0.5, generator=g)
    serving = Drafter.from_dir(save_dir(twin, tmp_path / "d", kind="export"), dev)
    tokens = torch.randint(0, V, (Lc + dcfg.k + 1,), generator=g)
    hidden = torch.randn(Lc + dcfg.k + 1, Ht, generator=g) * 0.5
    with torch.no_grad():
        want = twin.propose_greedy(tokens, hidden.bfloat16().float(), torch.tensor([Lc]))[0].tolist()
        plain = twin.draft_vocab[twin.block_logits(tokens, hidden.bfloat16().float(),
                                                   torch.tensor([Lc])).argmax(-1)[0]].tolist()
    kv = serving.new_kv_cache(4)
    ws = serving.new_workspace(128)
    i32 = dict(dtype=torch.int32, device=dev)
    pos = torch.arange(Lc, **i32)
    serving.inject(tokens[:Lc].int().to(dev), hidden[:Lc].bfloat16().to(dev), pos, pos.clone(), kv, ws)
    blk = torch.full((dcfg.k,), serving.mask_id, **i32)
    blk[0] = int(tokens[Lc])
    bpos = torch.arange(Lc, Lc + dcfg.k, **i32)
    out = torch.zeros(1, dcfg.k, **i32)
    serving.propose(blk, hidden[Lc - 1:Lc].bfloat16().to(dev), bpos, bpos.clone(), torch.arange(4, **i32).view(1, 4),
                    torch.tensor([Lc + dcfg.k], **i32), kv, ws, out, 1, max_pages=4)
    torch.cuda.synchronize()
    check_status()
    assert out[0].tolist() == want
    assert want != plain  # the selector changed the chain, so the test exercises it


def test_model_from_package_equals_model_from_reference(tmp_path):
    from arc_forge_2026_b200.formats.int3_package import package_tensors, write_package
    from arc_forge_2026_b200.quant.int3_tiles import tiles_to_codes, tiles_to_scales
    cfg, ref, model = _models(5)
    cs = [(tiles_to_codes(lw.bank.w13_codes.cpu()), tiles_to_scales(lw.bank.w13_scales.cpu()),
           tiles_to_codes(lw.bank.w2_codes.cpu()), tiles_to_scales(lw.bank.w2_scales.cpu())) for lw in model.layers]
    d = write_package(package_tensors(ref, cs, dense_fp8=False), cfg, tmp_path / "pkg", dense_fp8=False)
    loaded = HybridModel.from_package(d, dev)
    prompt = torch.randint(0, cfg.vocab_size, (90,), generator=torch.Generator().manual_seed(5)).tolist()
    outs = []
    for m in (model, loaded):
        eng = SpecEngine(m, None, ServeConfig(spec_k=0, accept_mode="greedy"), 1, 1024)
        outs.append(eng.generate([prompt], 12))
    torch.cuda.synchronize()
    check_status()
    assert outs[0] == outs[1]


def test_update_weights_in_place_matches_fresh_load(tmp_path):
    """A running engine swaps to another package's weights in place (same tensor addresses) and then decodes what
    an engine built on that package decodes."""
    from arc_forge_2026_b200.formats.int3_package import package_tensors, write_package
    from arc_forge_2026_b200.quant.int3_tiles import tiles_to_codes, tiles_to_scales
    cfg, ref, model = _models(6)
    cs = [(tiles_to_codes(lw.bank.w13_codes.cpu()), tiles_to_scales(lw.bank.w13_scales.cpu()),
           tiles_to_codes(lw.bank.w2_codes.cpu()), tiles_to_scales(lw.bank.w2_scales.cpu())) for lw in model.layers]
    d = write_package(package_tensors(ref, cs, dense_fp8=False), cfg, tmp_path / "pkg", dense_fp8=False)
    _, _, other = _models(9)
    ptrs = [t.data_ptr() for _, t in other.tensors()]
    prompt = torch.randint(0, cfg.vocab_size, (70,), generator=torch.Generator().manual_seed(6)).tolist()
    eng = SpecEngine(other, None, ServeConfig(spec_k=0, accept_mode="greedy"), 1, 1024)
    assert eng.update_weights(d)["tensors"] == len(ptrs)
    assert [t.data_ptr() for _, t in other.tensors()] == ptrs
    got = eng.generate([prompt], 10)
    want = SpecEngine(HybridModel.from_package(d, dev), None, ServeConfig(spec_k=0, accept_mode="greedy"), 1,
                      1024).generate([prompt], 10)
    torch.cuda.synchronize()
    check_status()
    assert got == want


def test_hyper_connection_model_decodes_like_reference(tmp_path):
    """A 4-branch hyper-connection model: the engine's greedy decode (plain and speculative) follows the reference,
    and a deploy package carries the hyper-connection weights."""
    from arc_forge_2026_b200.formats.int3_package import package_tensors, write_package
    from arc_forge_2026_b200.quant.int3_tiles import tiles_to_codes, tiles_to_scales
    cfg, ref, model = _models(7, hc_count=4, hc_lowrank=64)
    assert model.hc_final is not None and model.layers[0].hc_attn is not None
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (90, 33)]
    plain = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy"), 2, 1024).generate(prompts, 16)
    drafter = Drafter(drafter_preset("tiny"), cfg.hidden_size, cfg.vocab_size, dev, draft_vocab=4096)
    spec = SpecEngine(model, drafter, ServeConfig(spec_k=4, accept_mode="greedy"), 2, 1024).generate(prompts, 16)
    torch.cuda.synchronize()
    check_status()
    assert plain == spec
    # the serving read (tcgen05 GEMMs around the HC kernels) against the fp32 module
    from arc_forge_2026_b200.models.reference import hc_inject
    from arc_forge_2026_b200.ops.hc import HCWeights, hc_inject_, hc_read
    hs = torch.randn(90, 4, cfg.hidden_size, generator=g).bfloat16()
    mod = ref.layers[0].hc_attn
    x, gate = hc_read(hs.to(dev), HCWeights.from_module(mod, dev), 4)
    xr, gr = mod(hs.float())
    y = torch.randn(90, cfg.hidden_size, generator=g).bfloat16()
    h2 = hs.to(dev)
    hc_inject_(h2, y.to(dev), gate)
    hr = hc_inject(hs.float(), y.float(), gate.float().cpu())
    for a, b in ((x, xr), (gate, gr), (h2, hr)):
        assert ((a.float().cpu() - b).norm() / b.norm()).item() < 1e-2
    # first tokens: among the reference's best (a random INT3 model has near ties that bf16 may flip)
    with torch.no_grad():
        for p, out in zip(prompts, plain):
            lg = ref(torch.tensor([p]))[0, -1]
            assert out[0] in lg.topk(3).indices.tolist()
    cs = [(tiles_to_codes(lw.bank.w13_codes.cpu()), tiles_to_scales(lw.bank.w13_scales.cpu()),
           tiles_to_codes(lw.bank.w2_codes.cpu()), tiles_to_scales(lw.bank.w2_scales.cpu())) for lw in model.layers]
    d = write_package(package_tensors(ref, cs, dense_fp8=False), cfg, tmp_path / "pkg", dense_fp8=False)
    loaded = HybridModel.from_package(d, dev)
    again = SpecEngine(loaded, None, ServeConfig(spec_k=0, accept_mode="greedy"), 2, 1024).generate(prompts, 16)
    assert again == plain


def test_converted_drafter_directory_serves(tmp_path):
    """An HC dense-shared drafter converted to plain, expanded and written as a block-FP8 deployment copy loads into
    the serving drafter (``Drafter.from_dir``); greedy speculative decoding with it equals plain greedy decoding."""
    from arc_forge_2026_b200.train import drafter_tools as dtl
    from arc_forge_2026_b200.train.drafter_train import DrafterTrain
    cfg, ref, model = _models(3)
    dcfg = drafter_preset("tiny", residual="hc", hc_count=4, hc_lowrank=16, ffn="dense_shared",
                          shared_intermediate_size=128)
    src = DrafterTrain(dcfg, cfg.hidden_size, cfg.vocab_size, torch.arange(cfg.vocab_size), seed=4)
    g = torch.Generator().manual_seed(4)
    calib = [(torch.randint(0, cfg.vocab_size, (80,), generator=g), torch.randn(80, cfg.hidden_size, generator=g),
              torch.arange(1, 70, 7)) for _ in range(2)]
    plain, _ = dtl.convert_plain(src, calib)
    big = dtl.expand_layers(plain, [0, 1, 1])
    d = dtl.save_dir(big, tmp_path / "dep", "deploy", fp8=("attn", "mlp"))
    drafter = Drafter.from_dir(d, dev)
    assert drafter.cfg.num_layers == 3 and drafter.cfg.intermediate_size == dcfg.intermediate_size + 128
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (60, 17)]
    out_plain = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy"), 2, 1024).generate(prompts, 24)
    out_spec = SpecEngine(model, drafter, ServeConfig(spec_k=4, accept_mode="greedy"), 2, 1024).generate(prompts, 24)
    torch.cuda.synchronize()
    check_status()
    assert out_plain == out_spec


def test_ple_model_speculative_decoding_commits_side_state(tmp_path):
    """A model with a PLE layer: greedy speculative decoding (partial acceptance: the n-gram history and conv inputs
    of rejected rows must not be committed) equals plain greedy decoding; the first token follows the reference; a
    deploy package carries the PLE layer."""
    from arc_forge_2026_b200.formats.int3_package import package_tensors, write_package
    from arc_forge_2026_b200.quant.int3_tiles import tiles_to_codes, tiles_to_scales
    cfg, ref, model = _models(8, ple_layer_ids=(1,), ngram_vocab_size_base=4001, ple_embed_dim=256)
    assert model.layers[1].ple is not None
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 21, 5)]
    prompts[0][30] = cfg.eos_token_id
    plain = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy"), 3, 1024).generate(prompts, 30)
    drafter = Drafter(drafter_preset("tiny"), cfg.hidden_size, cfg.vocab_size, dev, draft_vocab=4096)
    spec_eng = SpecEngine(model, drafter, ServeConfig(spec_k=4, accept_mode="greedy"), 3, 1024)
    spec = spec_eng.generate(prompts, 30)
    torch.cuda.synchronize()
    check_status()
    assert plain == spec
    with torch.no_grad():
        for p, out in zip(prompts, plain):
            assert out[0] in ref(torch.tensor([p]))[0, -1].topk(3).indices.tolist()
    cs = [(tiles_to_codes(lw.bank.w13_codes.cpu()), tiles_to_scales(lw.bank.w13_scales.cpu()),
           tiles_to_codes(lw.bank.w2_codes.cpu()), tiles_to_scales(lw.bank.w2_scales.cpu())) for lw in model.layers]
    d = write_package(package_tensors(ref, cs, dense_fp8=False), cfg, tmp_path / "pkg", dense_fp8=False)
    loaded = HybridModel.from_package(d, dev)
    again = SpecEngine(loaded, None, ServeConfig(spec_k=0, accept_mode="greedy"), 3, 1024).generate(prompts, 30)
    assert again == plain


def test_session_continuation_and_parking_match_fresh_prefill():
    """Multi-turn sessions on 2 rows: a turn continues from the committed GDN / PLE state (only new tokens are
    prefilled); a third session parks the least recently used idle one (its state to pinned host memory, its row
    freed) and the parked session later resumes from the snapshot. Greedy outputs equal fresh sessions prefilling
    the whole transcript."""
    cfg, ref, model = _models(9, ple_layer_ids=(1,), ngram_vocab_size_base=4001, ple_embed_dim=256)
    drafter = Drafter(drafter_preset("tiny"), cfg.hidden_size, cfg.vocab_size, dev, draft_vocab=4096)
    scfg = ServeConfig(spec_k=4, accept_mode="greedy")
    eng = SpecEngine(model, drafter, scfg, 2, 1024)
    g = torch.Generator().manual_seed(9)

    def rnd(n):
        return torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist()

    def run(sess_id, tokens, n, cont):
        s = eng.continue_session(sess_id, tokens, n) if cont else eng.add_session(sess_id, tokens, n)
        while not s.done:
            eng.step()
        return list(s.prompt) + s.generated[:n]

    def fresh(tokens, n):
        e = SpecEngine(model, drafter, scfg, 1, 1024)
        return tokens + e.generate([tokens], n)[0]

    ta = run(1, rnd(60), 12, False)
    tb = run(2, rnd(45), 9, False)
    assert eng.free_slots == 2 and not eng.free_rows
    ta2 = ta + rnd(7)
    before = eng.prefilled_tokens
    assert run(1, ta2, 10, True) == fresh(ta2, 10)          # continuation in place
    assert eng.prefilled_tokens - before <= 7 + eng.W       # the new tokens and the uncommitted tail only
    tc = run(3, rnd(33), 8, False)                           # parks session 2 (the least recently used)
    assert 2 in eng.parked and 3 in eng.sessions
    tb2 = tb + rnd(5)
    before = eng.prefilled_tokens
    got = run(2, tb2, 11, True)                              # restores 2, parks 1
    assert 1 in eng.parked and got == fresh(tb2, 11)
    assert eng.prefilled_tokens - before <= 5 + eng.W
    assert tc == fresh(tc[:33], 8)
    for sid in (1, 2, 3):
        eng.release(sid)
    assert not eng.parked and len(eng.free_rows) == 2
    torch.cuda.synchronize()
    check_status()


def test_nvfp4_kv_engine_speculative_equals_plain():
    """The engine with an NVFP4 target KV cache: greedy speculative decoding equals plain greedy decoding, and the
    first token is among the reference's best."""
    cfg, ref, model = _models(10)
    g = torch.Generator().manual_seed(10)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (150, 40)]
    plain = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy", kv_dtype="nvfp4"), 2,
                       1024).generate(prompts, 24)
    drafter = Drafter(drafter_preset("tiny"), cfg.hidden_size, cfg.vocab_size, dev, draft_vocab=4096)
    spec = SpecEngine(model, drafter, ServeConfig(spec_k=4, accept_mode="greedy", kv_dtype="nvfp4"), 2,
                      1024).generate(prompts, 24)
    torch.cuda.synchronize()
    check_status()
    assert plain == spec
    with torch.no_grad():
        for p, out in zip(prompts, plain):
            assert out[0] in ref(torch.tensor([p]))[0, -1].topk(3).indices.tolist()
