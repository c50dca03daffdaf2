"""INT3 deploy package on CPU: write / verify / read round trip of the uint3 expert packs, block-FP8 dense modules
and config; tampering is detected."""
import json

import pytest
import torch

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.formats.int3_package import (dense_weight, expert_codes, package_tensors, read_package,
                                                       write_package)
from arc_forge_2026_b200.models.reference import build_reference
from arc_forge_2026_b200.quant.gptq import rtn_quantize


def _pkg(tmp_path, dense_fp8=True):
    cfg = preset("tiny_cpu")
    ref = build_reference(cfg, seed=0)
    cs = []
    for moe in ref.moe_layers():
        c13, s13 = rtn_quantize(moe.w13.detach().float())
        c2, s2 = rtn_quantize(moe.w2.detach().float())
        cs.append((c13, s13.bfloat16(), c2, s2.bfloat16()))
    t = package_tensors(ref, cs, dense_fp8)
    return cfg, ref, cs, write_package(t, cfg, tmp_path / "pkg", shard_bytes=1 << 20, dense_fp8=dense_fp8)


def test_package_round_trip(tmp_path):
    cfg, ref, cs, d = _pkg(tmp_path)
    assert (d / "DONE").exists() and len(list(d.glob("model-*.safetensors"))) > 1  # sharded
    cfg2, t = read_package(d)
    assert cfg2.num_experts == cfg.num_experts and cfg2.layer_types == cfg.layer_types
    q = json.loads((d / "config.json").read_text())["quantization_config"]["arc_int3"]
    assert q["layout"] == "humming_uint3_g128_nozp" and q["w13_rows"] == "gate_then_up"
    for i in range(cfg.num_layers):
        c13, s13, c2, s2 = expert_codes(t, i, cfg)
        assert torch.equal(c13, cs[i][0]) and torch.equal(c2, cs[i][2])
        assert torch.equal(s13, cs[i][1]) and torch.equal(s2, cs[i][3])
    w = dense_weight(t, "model.layers.0.linear_attn.in_proj_qkvz").float()
    ref_w = ref.layers[0].mixer.in_proj_qkvz.weight.detach().float()
    assert t["model.layers.0.linear_attn.in_proj_qkvz.weight"].dtype == torch.float8_e4m3fn
    assert ((w - ref_w).norm() / ref_w.norm()).item() < 0.05  # e4m3 block quantisation error
    assert torch.equal(dense_weight(t, "model.layers.0.linear_attn.in_proj_ba"),
                       ref.layers[0].mixer.in_proj_ba.weight.detach().bfloat16())


def test_package_detects_tampering(tmp_path):
    _, _, _, d = _pkg(tmp_path)
    f = sorted(d.glob("model-*.safetensors"))[0]
    data = bytearray(f.read_bytes())
    data[-1] ^= 0xFF
    f.write_bytes(bytes(data))
    with pytest.raises(RuntimeError, match="sha256"):
        read_package(d)


def test_package_round_trip_of_hyper_connections_and_ple(tmp_path):
    """A model with 2 hyper-connection branches and a PLE layer: the package carries the HC projections (bf16), the
    PLE table (block FP8) and the PLE projections / norms / conv, and the serving model loaded from it (on the CPU:
    loading runs no kernel) holds the reference's values."""
    import torch
    from arc_forge_2026_b200.config import preset
    from arc_forge_2026_b200.formats.int3_package import package_tensors, write_package
    from arc_forge_2026_b200.models.hybrid import HybridModel
    from arc_forge_2026_b200.models.reference import build_reference
    from arc_forge_2026_b200.quant.fp8 import dequant_weight_block, quantize_weight_block
    from arc_forge_2026_b200.quant.gptq import rtn_quantize
    cfg = preset("tiny_cpu", hc_count=2, hc_lowrank=32, ple_layer_ids=(1,), ngram_vocab_size_base=997,
                 ple_embed_dim=256)
    ref = build_reference(cfg, seed=3)
    cs = []
    for moe in ref.moe_layers():
        c13, s13 = rtn_quantize(moe.w13.detach().float())
        c2, s2 = rtn_quantize(moe.w2.detach().float())
        cs.append((c13, s13, c2, s2))
    d = write_package(package_tensors(ref, cs, dense_fp8=False), cfg, tmp_path / "pkg", dense_fp8=False)
    m = HybridModel.from_package(d, "cpu")
    assert m.cfg.hc_count == 2 and m.cfg.ple_layer_ids == (1,)
    hc = ref.layers[0].hc_attn
    R = hc.w_down.shape[0]
    assert torch.equal(m.layers[0].hc_attn.wcat[:R], hc.w_down.detach().bfloat16())
    assert torch.equal(m.layers[0].hc_attn.wcat[R:R + 2], hc.w_inject.detach().bfloat16())
    assert m.layers[0].hc_attn.wcat.shape[0] % 8 == 0 and m.hc_final is not None and not m.hc_final.inject
    lw = m.layers[1].ple
    assert lw is not None and m.layers[0].ple is None
    q, s = quantize_weight_block(ref.layers[1].ple.table.detach().float())
    assert torch.equal(dequant_weight_block(lw.table.rows, lw.table.scale), dequant_weight_block(q, s))
    assert torch.equal(lw.conv, ref.layers[1].ple.conv.detach().float())
    assert torch.equal(lw.key_proj, ref.layers[1].ple.key_proj.detach().bfloat16())
