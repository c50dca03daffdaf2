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
