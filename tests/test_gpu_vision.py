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


def _student_and_reference(cfg, seed=6):
    from arc_forge_2026_b200.config import FULL
    from arc_forge_2026_b200.models.reference import build_reference
    from arc_forge_2026_b200.quant import fp8 as fp8q
    from arc_forge_2026_b200.quant.gptq import rtn_quantize
    from arc_forge_2026_b200.train.student import QADStudent
    ref = build_reference(cfg, seed=seed)
    cs = []
    with torch.no_grad():
        for moe in ref.moe_layers():
            c13, s13 = rtn_quantize(moe.w13.float())
            c2, s2 = rtn_quantize(moe.w2.float())
            s13, s2 = s13.bfloat16().float(), s2.bfloat16().float()
            moe.w13.copy_((c13.float() - 4) * s13.repeat_interleave(128, -1))
            moe.w2.copy_((c2.float() - 4) * s2.repeat_interleave(128, -1))
            cs.append((c13, s13, c2, s2))
        for lay in ref.layers:  # dense projections on the FP8 grid: the student's QAT forward is then exact
            for name in (("q_proj", "k_proj", "v_proj") if lay.kind == FULL else ("in_proj_qkvz", "out_proj")):
                w = getattr(lay.mixer, name).weight
                qv, sv = fp8q.quantize_weight_block(w.bfloat16().float())
                w.copy_(fp8q.dequant_weight_block(qv, sv).bfloat16().float())
    return ref, QADStudent(cfg, ref, cs, checkpoint_layers=False).to(dev)


def test_student_multimodal_rows_follow_the_reference():
    """A packed multimodal row in the student (image features over the image tokens, deepstack additions, three-row
    multimodal RoPE through the native attention) against the fp32 reference model given the same inputs."""
    from arc_forge_2026_b200.config import preset
    from arc_forge_2026_b200.models.vision import mrope_positions
    from arc_forge_2026_b200.train.packing import pack
    cfg = preset("tiny_gpu", mrope_section=(6, 5, 5))
    ref, st = _student_and_reference(cfg)
    g = torch.Generator().manual_seed(8)
    img = 9
    seq = torch.randint(10, cfg.vocab_size, (150,), generator=g)
    seq[20:20 + 48] = img  # a 12 x 16 patch grid -> 48 merged tokens
    grid = torch.tensor([[1, 12, 16]])
    feats = torch.randn(48, cfg.hidden_size, generator=g) * 0.05
    ds = [torch.randn(48, cfg.hidden_size, generator=g) * 0.05]
    (b,) = pack([seq.tolist()], 512)
    b = b.to(dev)
    args = b.forward_args()
    args["pos3"] = mrope_positions((b.ids == img).long().cpu(), grid, 2).to(dev)
    with torch.no_grad():
        h = st.hidden(b.ids[None], pack=args, image_features=feats.to(dev), deepstack=[d.to(dev) for d in ds],
                      image_token_id=img)[0, :150].float().cpu()
        h_text = st.hidden(b.ids[None], pack=b.forward_args(), image_features=feats.to(dev),
                           deepstack=[d.to(dev) for d in ds], image_token_id=img)[0, :150].float().cpu()
        r = ref.hidden(seq[None], positions=args["pos3"][:, :150].cpu(), image_features=feats, deepstack=ds,
                       image_token_id=img)[0].float()
    torch.cuda.synchronize()
    check_status()
    e = ((h - r).norm(dim=-1) / r.norm(dim=-1))[68:]  # the text after the image
    e_text = ((h_text - r).norm(dim=-1) / r.norm(dim=-1))[68:]
    assert e.median() < 0.06, (e.median(), e_text.median())
    assert e.median() < 0.5 * e_text.median(), (e.median(), e_text.median())


def test_sft_trains_on_an_image_example(tmp_path):
    import json

    import numpy as np

    from arc_forge_2026_b200.train import sft
    np.save(tmp_path / "a.npy", np.random.default_rng(0).standard_normal((64, 1536)).astype(np.float32))
    rows = [{"ids": list(range(20, 80))},
            {"prompt_ids": [11, 12] + [9] * 16 + [13], "completion_ids": list(range(30, 60)),
             "images": [{"pixels": "a.npy", "grid_thw": [1, 8, 8]}]}]
    (tmp_path / "d.jsonl").write_text("\n".join(json.dumps(r) for r in rows))
    sft.main(["--data", str(tmp_path / "d.jsonl"), "--preset", "tiny_gpu", "--mrope-section", "6,5,5",
              "--vision-random", "--vision-depth", "2", "--image-token-id", "9", "--steps", "3",
              "--bins-per-step", "4", "--max-len", "256", "--out", str(tmp_path / "run")])
    torch.cuda.synchronize()
    check_status()
    assert (tmp_path / "run" / "trainer_state.pt").exists()
