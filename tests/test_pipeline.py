"""Compression pipeline CLI on the tiny CPU model: saliency pruning, routed-row Hessians with the pooled prior,
GPTQ INT3 beating RTN on the Hessian-weighted error, and a loadable deploy package."""
import json

import torch

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.formats.int3_package import expert_codes, read_package
from arc_forge_2026_b200.models.reference import build_reference
from arc_forge_2026_b200.quant import gptq
from arc_forge_2026_b200.quant.pipeline import collect_hessians, main


def test_pipeline_cli_writes_package(tmp_path, capsys):
    path = main(["--preset", "tiny_cpu", "--keep", "20", "--calib-tokens", "512", "--out", str(tmp_path / "pkg")])
    rec = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert 0.6 < rec["retained_mass_mean"] <= 1.0
    cfg, t = read_package(path)
    assert cfg.num_experts == 20
    c13, s13, c2, s2 = expert_codes(t, 0, cfg)
    assert c13.shape == (20, 2 * cfg.moe_intermediate_size, cfg.hidden_size) and int(c13.max()) <= 7


def test_hessian_gptq_beats_rtn():
    cfg = preset("tiny_cpu")
    model = build_reference(cfg, seed=0)
    g = torch.Generator().manual_seed(0)
    batches = [torch.randint(0, cfg.vocab_size, (1, 256), generator=g) for _ in range(2)]
    h13, h2, n, tot = collect_hessians(model, batches)[0]
    assert tot == 512 * cfg.num_experts_per_tok and torch.isfinite(h13).all()
    moe = model.moe_layers()[0]
    W = moe.w13.detach().float()

    def err(codes, scales):
        dw = gptq.dequant(codes, scales.to(torch.bfloat16)) - W
        return float(torch.einsum("eok,ekl,eol->", dw, h13, dw))
    e_gptq = err(*gptq.gptq_quantize(W, h13))
    e_rtn = err(*gptq.rtn_quantize(W))
    assert e_gptq < e_rtn
