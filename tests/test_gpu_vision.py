"""Vision tower on the B200 path (tcgen05 GEMMs, bidirectional tcgen05 attention with padded heads, csrc/vision.cu)
against its fp32 statement and against Hugging Face's bf16 vision model with the same weights."""
import pytest
import torch

from arc_forge_2026_b200.models.vision import VisionConfig, VisionTower
from arc_forge_2026_b200.ops import check_status

pytestmark = pytest.mark.gpu
dev = "cuda"

CFG = VisionConfig(depth=3, deepstack_visual_indexes=(0, 2))  # full-width blocks, three of them
GRIDS = [(1, 32, 40), (1, 16, 16), (2, 8, 12)]


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _inputs():
    P = sum(t * h * w for t, h, w in GRIDS)
    return torch.randn(P, CFG.patch_dim, generator=torch.Generator().manual_seed(5)).to(dev), torch.tensor(GRIDS)


def test_native_tower_matches_fp32_statement():
    tower = VisionTower.random(CFG, seed=1).to(dev)
    pixels, grid = _inputs()
    merged, ds = tower(pixels, grid)
    torch.cuda.synchronize()
    check_status()
    ref, ref_ds = tower.forward_reference(pixels, grid)
    assert merged.shape == ref.shape and merged.dtype == torch.bfloat16
    assert _rel(merged, ref) < 2e-2
    assert len(ds) == 2
    for a, b in zip(ds, ref_ds):
        assert _rel(a, b) < 2e-2
    # deterministic: the same inputs give the same bits
    again, _ = tower(pixels, grid)
    assert torch.equal(merged, again)


def test_native_tower_tracks_hf_bf16_model():
    hf = pytest.importorskip("transformers.models.qwen3_vl_moe.modeling_qwen3_vl_moe")
    hfc = pytest.importorskip("transformers.models.qwen3_vl_moe.configuration_qwen3_vl_moe")
    c = hfc.Qwen3VLMoeVisionConfig(depth=CFG.depth, out_hidden_size=CFG.out_hidden_size,
                                   deepstack_visual_indexes=list(CFG.deepstack_visual_indexes))
    c._attn_implementation = "sdpa"
    tower = VisionTower.random(CFG, seed=2)
    model = hf.Qwen3VLMoeVisionModel(c)
    model.load_state_dict(tower.state_dict(), strict=True)
    model = model.to(dev, torch.bfloat16).eval()
    tower = tower.to(dev)
    pixels, grid = _inputs()
    merged, ds = tower(pixels, grid)
    with torch.no_grad():
        ref = model(pixels.bfloat16(), grid_thw=grid.to(dev))
    torch.cuda.synchronize()
    check_status()
    fp32, _ = tower.forward_reference(pixels, grid)
    # the native path is at least as close to fp32 as the bf16 library model is
    assert _rel(merged, ref.pooler_output) < 2e-2
    assert _rel(merged, fp32) <= 1.5 * _rel(ref.pooler_output, fp32) + 1e-3
