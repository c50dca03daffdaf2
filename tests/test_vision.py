"""Vision tower on CPU: the fp32 statement of the tower against Hugging Face's Qwen3-VL vision model with the same
weights (the reference runs the checkpoint's tower through that model family), the position-table resampling and the
rotary angles against its helpers, and the three-row text positions against its ``get_rope_index``."""
import types

import pytest
import torch

from arc_forge_2026_b200.models.vision import (VisionConfig, VisionTower, merge_image_features, mrope_positions,
                                              vit_interp)

hf = pytest.importorskip("transformers.models.qwen3_vl_moe.modeling_qwen3_vl_moe")
hfc = pytest.importorskip("transformers.models.qwen3_vl_moe.configuration_qwen3_vl_moe")

CFG = VisionConfig(depth=3, hidden_size=64, num_heads=4, intermediate_size=96, patch_size=4, out_hidden_size=48,
                   num_position_embeddings=64, deepstack_visual_indexes=(0, 2))
GRIDS = [(1, 6, 8), (2, 4, 4), (1, 2, 10)]


def _hf_model(cfg: VisionConfig):
    c = hfc.Qwen3VLMoeVisionConfig(depth=cfg.depth, hidden_size=cfg.hidden_size, num_heads=cfg.num_heads,
                                   intermediate_size=cfg.intermediate_size, patch_size=cfg.patch_size,
                                   temporal_patch_size=cfg.temporal_patch_size, in_channels=cfg.in_channels,
                                   spatial_merge_size=cfg.spatial_merge_size, out_hidden_size=cfg.out_hidden_size,
                                   num_position_embeddings=cfg.num_position_embeddings,
                                   deepstack_visual_indexes=list(cfg.deepstack_visual_indexes))
    c._attn_implementation = "eager"
    return hf.Qwen3VLMoeVisionModel(c).float().eval()


def test_tower_matches_hf_vision_model_with_the_same_weights():
    ours = VisionTower.random(CFG, seed=3)
    theirs = _hf_model(CFG)
    theirs.load_state_dict(ours.state_dict(), strict=True)  # the checkpoint's names load as they are
    grid = torch.tensor(GRIDS)
    P = sum(t * h * w for t, h, w in GRIDS)
    pixels = torch.randn(P, CFG.patch_dim, generator=torch.Generator().manual_seed(4))
    merged, ds = ours.forward_reference(pixels, grid)
    with torch.no_grad():
        ref = theirs(pixels, grid_thw=grid)
    assert merged.shape == (P // 4, CFG.out_hidden_size)
    torch.testing.assert_close(merged, ref.pooler_output, rtol=1e-4, atol=1e-5)
    assert len(ds) == len(ref.deepstack_features) == 2
    for a, b in zip(ds, ref.deepstack_features):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)


def test_position_resampling_matches_hf_and_rounds_weights_like_the_server():
    cfg = VisionConfig(depth=1, hidden_size=32, num_heads=2, intermediate_size=32, out_hidden_size=16,
                       num_position_embeddings=2304, deepstack_visual_indexes=())
    m = _hf_model(cfg)
    grids = [(1, 20, 34), (2, 48, 48), (1, 2, 2)]
    with torch.no_grad():
        ref = m.fast_pos_embed_interpolate(torch.tensor(grids))
    idx, w = vit_interp(grids, cfg.grid_side, cfg.spatial_merge_size, torch.float32)
    got = (m.pos_embed.weight[idx] * w[..., None]).sum(1)
    torch.testing.assert_close(got, ref, rtol=1e-6, atol=1e-6)
    idx16, w16 = vit_interp(grids, cfg.grid_side, cfg.spatial_merge_size, torch.bfloat16)
    assert torch.equal(idx16, idx) and w16.dtype == torch.bfloat16 and torch.equal(w16, w.bfloat16())


def test_rotary_angles_match_hf():
    m = _hf_model(CFG)
    grids = torch.tensor(GRIDS)
    from arc_forge_2026_b200.models.vision import vision_rope_angles
    got = vision_rope_angles(GRIDS, CFG.head_dim, CFG.spatial_merge_size)
    torch.testing.assert_close(got, m.rot_pos_emb(grids).float(), rtol=0, atol=0)


def test_multimodal_positions_match_hf_rope_index():
    merge = 2
    grids = torch.tensor([[1, 6, 8], [1, 4, 10]])
    n0, n1 = 6 * 8 // 4, 4 * 10 // 4
    types_ = torch.tensor([0] * 5 + [1] * n0 + [0] * 3 + [1] * n1 + [0] * 4)
    ids = torch.where(types_ == 1, 99, 7)
    host = types.SimpleNamespace(config=types.SimpleNamespace(vision_config=types.SimpleNamespace(
        spatial_merge_size=merge)))
    host.get_vision_position_ids = types.MethodType(hf.Qwen3VLMoeModel.get_vision_position_ids, host)
    ref, _ = hf.Qwen3VLMoeModel.get_rope_index(host, ids[None], types_[None].int(), image_grid_thw=grids)
    got = mrope_positions(types_, grids, merge)
    assert torch.equal(got, ref[:, 0])
    emb = torch.randn(len(ids), 8)
    feats = torch.randn(n0 + n1, 8)
    out = merge_image_features(emb, ids, 99, feats)
    assert torch.equal(out[ids == 99], feats) and torch.equal(out[ids != 99], emb[ids != 99])


def test_interleaved_mrope_angles_match_hf_text_rotary():
    from arc_forge_2026_b200.models.vision import mrope_angles
    cfg = hfc.Qwen3VLMoeTextConfig(head_dim=128, rope_parameters={"rope_type": "default", "rope_theta": 5e5,
                                                                   "mrope_section": [24, 20, 20],
                                                                   "mrope_interleaved": True})
    rope = hf.Qwen3VLMoeTextRotaryEmbedding(cfg)
    types_ = torch.tensor([0] * 3 + [1] * 12 + [0] * 2)
    pos3 = mrope_positions(types_, torch.tensor([[1, 6, 8]]), 2)
    cos, sin = rope(torch.zeros(1, dtype=torch.float32), pos3[:, None, :])
    ang = mrope_angles(pos3, 128, 5e5, (24, 20, 20))
    torch.testing.assert_close(torch.cat([ang, ang], -1).cos(), cos[0], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(torch.cat([ang, ang], -1).sin(), sin[0], rtol=1e-6, atol=1e-6)


def _mm_ref(seed=0):
    from arc_forge_2026_b200.config import preset
    from arc_forge_2026_b200.models.reference import build_reference
    cfg = preset("tiny_cpu", mrope_section=(4, 2, 2))
    return cfg, build_reference(cfg, seed=seed)


def test_multimodal_rope_reduces_to_text_rope_on_text_tokens():
    cfg, ref = _mm_ref()
    ids = torch.randint(0, cfg.vocab_size, (1, 40), generator=torch.Generator().manual_seed(1))
    pos3 = torch.arange(40).expand(3, 40)
    with torch.no_grad():
        torch.testing.assert_close(ref.hidden(ids, positions=pos3), ref.hidden(ids), rtol=0, atol=0)


def test_decode_after_an_image_continues_with_the_position_delta():
    """Prefill text + image + text with three-row positions and image features, then decode one token at
    1-D position index + delta: the same hidden state as the whole sequence in one pass."""
    cfg, ref = _mm_ref(seed=2)
    img_id = 7
    g = torch.Generator().manual_seed(3)
    grid = torch.tensor([[1, 4, 6]])
    ids = torch.randint(10, cfg.vocab_size, (1, 16), generator=g)
    ids[0, 5:11] = img_id  # 4 x 6 patches -> 6 merged tokens
    feats = torch.randn(6, cfg.hidden_size, generator=g) * 0.02
    ds = [torch.randn(6, cfg.hidden_size, generator=g) * 0.02]
    pos3 = mrope_positions((ids[0] == img_id).long(), grid, 2)
    with torch.no_grad():
        full = ref.hidden(ids, positions=pos3, image_features=feats, deepstack=ds, image_token_id=img_id)
        cache = ref.new_cache()
        ref.hidden(ids[:, :15], cache, positions=pos3[:, :15], image_features=feats, deepstack=ds,
                   image_token_id=img_id)
        delta = int(pos3[:, :15].max()) + 1 - 15
        step = ref.hidden(ids[:, 15:], cache, start_pos=15 + delta)
    torch.testing.assert_close(step[0, -1], full[0, -1], rtol=1e-4, atol=1e-5)
    assert delta < 0  # the image took fewer positions than tokens


def test_sft_reads_image_examples(tmp_path):
    import json

    import numpy as np

    from arc_forge_2026_b200.train import sft
    np.save(tmp_path / "a.npy", np.zeros((64, 1536), dtype=np.float32))
    rows = [{"ids": [1, 2, 3, 4]}, {"ids": [5] + [9] * 16 + [6], "images": [{"pixels": "a.npy", "grid_thw": [1, 8, 8]}]}]
    (tmp_path / "d.jsonl").write_text("\n".join(json.dumps(r) for r in rows))
    media = []
    seqs, masks = sft.load_examples(tmp_path / "d.jsonl", media)
    assert len(seqs) == 2 and media[0] is None and media[1][0]["grid_thw"] == [1, 8, 8]
    assert media[1][0]["pixels"] == tmp_path / "a.npy"
    with pytest.raises(ValueError):
        sft.load_examples(tmp_path / "d.jsonl")


def test_reference_rope_tables_agree_with_the_vision_module_angles():
    """The text model's three-row RoPE tables (models/reference.py) and models/vision.py's angles are one rule."""
    from arc_forge_2026_b200.models.reference import rope_cos_sin
    from arc_forge_2026_b200.models.vision import mrope_angles
    types_ = torch.tensor([0] * 4 + [1] * 30 + [0] * 6)
    pos3 = mrope_positions(types_, torch.tensor([[1, 10, 12]]), 2)
    cos, sin = rope_cos_sin(pos3, 32, 1.0e7, (6, 5, 5))
    ang = mrope_angles(pos3, 32, 1.0e7, (6, 5, 5))
    torch.testing.assert_close(cos, ang.double().cos().float(), rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(sin, ang.double().sin().float(), rtol=1e-6, atol=1e-6)
    text = rope_cos_sin(torch.arange(40), 32, 1.0e7, (6, 5, 5))  # 1-D positions: plain RoPE
    torch.testing.assert_close(text[0], rope_cos_sin(torch.arange(40), 32, 1.0e7)[0], rtol=0, atol=0)


def test_cpu_engine_serves_an_image_prompt():
    """The CPU serving engine with a vision tower: greedy tokens after an image prompt equal a full recompute of the
    whole sequence (three-row positions over prompt + generated text) at every step."""
    from arc_forge_2026_b200.serve.cpu_engine import CPUEngine
    cfg, ref = _mm_ref(seed=4)
    vcfg = VisionConfig(depth=2, hidden_size=64, num_heads=4, intermediate_size=96, out_hidden_size=cfg.hidden_size,
                        num_position_embeddings=64, deepstack_visual_indexes=(0,))
    tower = VisionTower.random(vcfg, seed=5)
    img = 7
    g = torch.Generator().manual_seed(6)
    pixels = torch.randn(4 * 6, vcfg.patch_dim, generator=g)
    prompt = [11, 12, 13] + [img] * 6 + [14, 15]
    eng = CPUEngine(ref, vision=tower, image_token_id=img)
    s = eng.add_session(0, prompt, 5, images=[(pixels, (1, 4, 6))])
    while not s.done:
        eng.step()
    merged, ds = tower.forward_reference(pixels, torch.tensor([[1, 4, 6]]))
    seq = list(prompt)
    for tok in s.generated:
        ids = torch.tensor([seq])
        pos3 = mrope_positions((ids[0] == img).long(), torch.tensor([[1, 4, 6]]), 2)
        with torch.no_grad():
            h = ref.hidden(ids, positions=pos3, image_features=merged, deepstack=ds, image_token_id=img)
        assert int(ref.lm_head(h)[0, -1].argmax()) == tok
        seq.append(tok)
