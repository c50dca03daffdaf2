"""CPU tests of the oracle model and the formats (tiny hybrid MoE, fp32, seed 0)."""
import pytest
import torch

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.models.reference import build_reference
from arc_forge_2026_b200.quant import fp8, gptq, saliency, uint3
from arc_forge_2026_b200.quant.pipeline import collect_hessians
from arc_forge_2026_b200.train.kl import teacher_topk, topk_tail_kl, topk_tail_kl_autograd


def _bit_pack(codes):
    """Independent bit-by-bit packer (the LSB-first 3-bit stream, 32 codes per 3 words)."""
    flat = codes.reshape(-1, codes.shape[-1]).tolist()
    out = []
    for row in flat:
        words = []
        for g in range(0, len(row), 32):
            acc = 0
            for i, c in enumerate(row[g:g + 32]):
                acc |= int(c) << (3 * i)
            for w in range(3):
                v = (acc >> (32 * w)) & 0xFFFFFFFF
                words.append(v - (1 << 32) if v >= (1 << 31) else v)
        out.append(words)
    return torch.tensor(out, dtype=torch.int32).reshape(*codes.shape[:-1], -1)


def test_uint3_roundtrip_and_bit_layout():
    g = torch.Generator().manual_seed(0)
    codes = torch.randint(0, 8, (3, 5, 256), generator=g, dtype=torch.uint8)
    packed = uint3.pack_uint3(codes)
    assert packed.shape == (3, 5, 24) and packed.dtype == torch.int32
    assert torch.equal(packed, _bit_pack(codes))
    assert torch.equal(uint3.unpack_uint3(packed, 256), codes)
    # codes 10 and 21 straddle words: set only them and check both words carry bits
    c = torch.zeros(1, 32, dtype=torch.uint8)
    c[0, 10] = 7
    p = uint3.pack_uint3(c)
    assert int(p[0, 0]) < 0 and int(p[0, 1]) == 1  # bits 30,31 of word 0 and bit 0 of word 1


def test_dequant_matches_bf16_product():
    g = torch.Generator().manual_seed(1)
    codes = torch.randint(0, 8, (4, 256), generator=g, dtype=torch.uint8)
    scales = (torch.randn(4, 2, generator=g) * 0.01).to(torch.bfloat16)
    w = uint3.dequant_uint3(uint3.pack_uint3(codes), scales, 256)
    ref = ((codes.to(torch.bfloat16) - 4) * scales.repeat_interleave(128, -1)).to(torch.bfloat16)
    assert torch.equal(w, ref)


def test_gptq_beats_rtn_and_scales_are_bf16():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2048, 256, generator=g) @ (torch.eye(256) + 0.3 * torch.randn(256, 256, generator=g))
    w = torch.randn(64, 256, generator=g) * 0.02
    H = gptq.hessian(x)
    codes, scales = gptq.gptq_quantize(w, H)
    assert codes.max() <= 7 and scales.shape == (64, 2)
    assert torch.equal(scales, scales.to(torch.bfloat16).float())
    rcodes, rscales = gptq.rtn_quantize(w)
    err = lambda c, s: ((x @ (gptq.dequant(c, s) - w).t()) ** 2).sum()  # noqa: E731
    assert err(codes, scales) < err(rcodes, rscales)


def test_fp8_block_roundtrip():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(300, 260, generator=g)
    q, s = fp8.quantize_weight_block(w)
    assert s.shape == (3, 3)
    back = fp8.dequant_weight_block(q, s)
    assert (back - w).abs().max() < 0.07 * w.abs().max()
    x = torch.randn(5, 256, generator=g)
    xq, xs = fp8.quantize_act_groups(x)
    assert (fp8.dequant_act_groups(xq, xs) - x).abs().max() < 0.07 * x.abs().max()


def test_incremental_decode_matches_full_forward():
    cfg = preset("tiny_cpu")
    m = build_reference(cfg, seed=0)
    ids = torch.randint(0, cfg.vocab_size, (2, 12), generator=torch.Generator().manual_seed(4))
    full = m(ids)
    cache = m.new_cache()
    a = m(ids[:, :7], cache, 0)
    b = m(ids[:, 7:], cache, 7)
    torch.testing.assert_close(torch.cat([a, b], 1), full, rtol=1e-4, atol=1e-5)


def _kl_autograd(z, ids, t_lp, t_tail, direction):
    z = z.clone().requires_grad_(True)
    lq = torch.log_softmax(z.double(), -1)
    lq_k = lq.gather(1, ids)
    lq_r = lq.scatter(1, ids, float("-inf")).logsumexp(-1)
    LQ = torch.cat([lq_k, lq_r[:, None]], 1)
    LP = torch.cat([t_lp.double(), t_tail.double()[:, None]], 1)
    if direction == "forward":
        loss = (LP.exp() * (LP - LQ)).sum(-1)
    else:
        loss = (LQ.exp() * (LQ - LP)).sum(-1)
    loss.sum().backward()
    return loss.float(), z.grad.float()


def test_topk_tail_kl_matches_autograd():
    g = torch.Generator().manual_seed(5)
    zt = torch.randn(6, 300, generator=g) * 3
    ids, lp, tail = teacher_topk(zt, 16)
    zs = torch.randn(6, 300, generator=g) * 3
    zs[0, :] = torch.where(torch.arange(300) % 3 == 0, 80.0, -80.0)  # a peaked row: some classes underflow
    tail[1] = float("-inf")  # a teacher row with no mass outside its top-k
    lp[1] = lp[1] - lp[1].logsumexp(-1)
    for direction in ("forward", "reverse"):
        loss, dz = topk_tail_kl(zs, ids, lp, tail, direction)
        # the fp64 oracle (0 log 0 = 0) covers every row; the plain one here leaves 0 * inf = nan on row 1
        for rl, rg, every_row in ((*topk_tail_kl_autograd(zs, ids, lp, tail, direction), True),
                                  (*_kl_autograd(zs, ids, lp, tail, direction), False)):
            fin = torch.isfinite(rl)
            if every_row:
                assert torch.equal(torch.isfinite(loss), fin)
            torch.testing.assert_close(loss[fin], rl[fin], rtol=1e-4, atol=1e-5)
            rows = fin & torch.isfinite(rg).all(-1)
            torch.testing.assert_close(dz[rows], rg[rows], rtol=1e-4, atol=1e-6)


def test_config1_pipeline_prune_quantize_decode():
    """prune 32->20 by saliency on 512 calibration tokens, GPTQ INT3 g128 pack round trip,
    greedy-decode 64 tokens from a 256-token prompt, logits of the packed model == the dequantized model."""
    torch.manual_seed(0)
    cfg = preset("tiny_cpu")
    model = build_reference(cfg, seed=0)
    g = torch.Generator().manual_seed(0)
    calib = torch.randint(0, cfg.vocab_size, (2, 256), generator=g)
    acc = saliency.collect_saliency(model, [calib])
    assert int(acc.acc[:, 0].sum()) == 512 * cfg.num_experts_per_tok * cfg.num_layers
    scores = saliency.reap_scores(acc.acc)
    drop = saliency.keep_mask(scores, 20)
    mass = saliency.retained_mass(scores, drop)
    assert 0.6 < mass["min"] <= mass["mean"] <= 1.0
    source = build_reference(cfg, seed=0)
    saliency.prune_experts(model, drop)
    assert model.cfg.num_experts == 20 and model.layers[0].mlp.w13.shape[0] == 20
    manifest = {"keep": [(~drop[i]).nonzero().flatten().tolist() for i in range(drop.shape[0])]}
    got = saliency.verify_pruned(model, source, manifest)
    assert got["experts"] == 20 * cfg.num_layers and got["other_tensors"] > 0
    bad = {"keep": [list(reversed(k)) for k in manifest["keep"]]}
    with pytest.raises(ValueError):
        saliency.verify_pruned(model, source, bad)

    # GPTQ every expert of every layer with Hessians from its routed calibration rows (the pruned model re-run on
    # the calibration tokens; experts that saw few rows lean on the pooled prior)
    packs = []
    hessians = collect_hessians(model, [calib])
    for moe, (h13, h2, _, _) in zip(model.moe_layers(), hessians):
        c13, s13 = gptq.gptq_quantize(moe.w13.data, h13)
        c2, s2 = gptq.gptq_quantize(moe.w2.data, h2)
        pack = uint3.pack_experts(c13, s13, c2, s2)
        assert torch.equal(uint3.unpack_uint3(pack["w13_qweight"], cfg.hidden_size), c13)
        packs.append(pack)
    # dequantized twin vs the packed path (expert_override unpacks on the fly)
    twin = build_reference(preset("tiny_cpu"), seed=0)
    saliency.prune_experts(twin, drop)
    twin.load_state_dict(model.state_dict())
    for moe_t, moe_p, pack in zip(twin.moe_layers(), model.moe_layers(), packs):
        w13, w2 = uint3.dequant_experts(pack, cfg.hidden_size, cfg.moe_intermediate_size, torch.float32)
        moe_t.w13.data.copy_(w13)
        moe_t.w2.data.copy_(w2)

        def override(x, e, pack=pack):
            a = uint3.dequant_uint3(pack["w13_qweight"][e], pack["w13_scales"][e], cfg.hidden_size, torch.float32)
            b = uint3.dequant_uint3(pack["w2_qweight"][e], pack["w2_scales"][e], cfg.moe_intermediate_size,
                                    torch.float32)
            h = x @ a.t()
            I = cfg.moe_intermediate_size
            return (torch.nn.functional.silu(h[:, :I]) * h[:, I:]) @ b.t()
        moe_p.expert_override = override
    prompt = torch.randint(0, cfg.vocab_size, (1, 256), generator=g)
    toks_p, logits_p = model.greedy_decode(prompt, 64)
    toks_t, logits_t = twin.greedy_decode(prompt, 64)
    assert toks_p.shape == (1, 64)
    torch.testing.assert_close(logits_p, logits_t, rtol=1e-4, atol=1e-5)
    assert torch.equal(toks_p, toks_t)


def _emulate_kernel_decode(tiles):
    """Bit-exact emulation of the kernel's byte-permute decode: tile words -> e4m3 bytes of (code - 4)."""
    table = [0xC8, 0xC4, 0xC0, 0xB8, 0x00, 0x38, 0x40, 0x44]
    w = tiles.reshape(-1, 3).to(torch.int64) & 0xFFFFFFFF
    out = []
    for L0, L1, H in w.tolist():
        m3, m4 = 0x33333333, 0x44444444
        sels = [(L0 & m3) | (H & m4), ((L0 >> 2) & m3) | ((H >> 1) & m4),
                (L1 & m3) | ((H << 2) & m4 & 0xFFFFFFFF), ((L1 >> 2) & m3) | ((H << 1) & m4 & 0xFFFFFFFF)]
        for s in sels:
            for nib in range(8):
                out.append(table[(s >> (4 * nib)) & 7])
    return torch.tensor(out, dtype=torch.uint8)


def test_int3_tile_layout_roundtrip_and_kernel_decode():
    from arc_forge_2026_b200.quant import int3_tiles
    g = torch.Generator().manual_seed(9)
    codes = torch.randint(0, 8, (2, 256, 384), generator=g, dtype=torch.uint8)
    tiles = int3_tiles.codes_to_tiles(codes)
    assert tiles.shape == (2, 2, 3, 128, 12)
    assert torch.equal(int3_tiles.tiles_to_codes(tiles), codes)
    # Humming pack -> tiles path
    packed = uint3.pack_uint3(codes)
    scales = torch.randn(2, 256, 3, generator=g).to(torch.bfloat16)
    t2, s2 = int3_tiles.pack_to_tiles(packed, scales, 384)
    assert torch.equal(t2, tiles) and torch.equal(int3_tiles.tiles_to_scales(s2), scales)
    # the kernel decode of one tile row equals e4m3(code - 4) in code order
    row = tiles[0, 1, 2, 5]  # expert 0, row block 1, group 2, row 5
    dec = _emulate_kernel_decode(row)
    ref = (codes[0, 128 + 5, 256:384].to(torch.float32) - 4).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(dec, ref)
