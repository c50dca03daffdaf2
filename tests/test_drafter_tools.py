"""Drafter conversions on CPU: HC -> plain (exact for a single stream in disguise), layer expansion with zeroed
repeats (exact), the block-FP8 deployment copy, the directory layout (atomic publish, sha256 verification) and the
CLI."""
import json

import pytest
import torch

from arc_forge_2026_b200.config import drafter_preset
from arc_forge_2026_b200.train import drafter_tools as dt
from arc_forge_2026_b200.train.drafter_train import DrafterTrain

V, HT = 300, 48


def _cfg(**kw):
    return drafter_preset("tiny", hidden_size=128, num_attention_heads=2, num_kv_heads=1, head_dim=64,
                          intermediate_size=96, **kw)


def _calib(n=3, T=120, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        tokens = torch.randint(0, V, (T,), generator=g)
        hidden = torch.randn(T, HT, generator=g)
        anchors = torch.randint(1, T - 6, (24,), generator=g).unique()
        out.append((tokens, hidden, anchors))
    return out


def _hc_source(disguise: bool, seed=0):
    cfg = _cfg(residual="hc", hc_count=4, hc_lowrank=8, ffn="dense_shared", shared_intermediate_size=32)
    src = DrafterTrain(cfg, HT, V, torch.arange(0, V, 2), seed=seed, std=0.05)
    g = torch.Generator().manual_seed(seed + 10)
    with torch.no_grad():
        for mod in [m for L in src.layers for m in (L.hc_attn, L.hc_mlp)] + [src.hc_final]:
            mod.hc_norm.weight.copy_(torch.randn(mod.hc_norm.weight.shape, generator=g) * 0.2)
            if not disguise:
                mod.w_up.copy_(torch.randn(mod.w_up.shape, generator=g) * 0.05)
                if mod.w_inject is not None:
                    mod.w_inject.copy_(torch.randn(mod.w_inject.shape, generator=g) * 0.05)
        for L in src.layers:
            for n in ("ctx_norm", "q_norm", "k_norm"):
                getattr(L, n).copy_(torch.randn(getattr(L, n).shape, generator=g) * 0.1)
            if disguise:
                L.shared_gate.zero_()
    return src


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


def test_hc_to_plain_is_exact_for_a_single_stream_in_disguise():
    src = _hc_source(disguise=True)
    calib = _calib()
    plain, report = dt.convert_plain(src, calib)
    assert plain.cfg.residual == "plain" and plain.cfg.ffn == "dense" and plain.cfg.intermediate_size == 96 + 32
    for tokens, hidden, anchors in _calib(2, seed=5):
        with torch.no_grad():
            assert _rel(plain.block_logits(tokens, hidden, anchors), src.block_logits(tokens, hidden, anchors)) < 1e-4
    assert all(f["relative_residual"] < 1e-4 for f in report["fits"].values()), report["fits"]
    assert all(abs(s["shared_sigmoid_mean"] - 0.5) < 1e-6 and abs(s["mlp_gate_mean"] - 1) < 1e-6
               for s in report["layers"])


def test_hc_to_plain_general_source_fits_and_publishes(tmp_path):
    src = _hc_source(disguise=False, seed=1)
    src_dir = dt.save_dir(src, tmp_path / "hc", "export")
    torch.save([{"tokens": t, "hidden": h, "anchors": a} for t, h, a in _calib()], tmp_path / "calib.pt")
    out = dt.main(["plain", "--source", str(src_dir), "--calibration", str(tmp_path / "calib.pt"),
                   "--out", str(tmp_path / "plain")])
    assert dt.manifest_of(out)["kind"] == "plain-conversion"
    rep = json.loads((out / "calibration.json").read_text())
    assert all(f["relative_residual"] <= f["relative_residual_unit_gain"] + 1e-9 for f in rep["fits"].values())
    plain = dt.load_dir(out)
    tokens, hidden, anchors = _calib(1, seed=7)[0]
    with torch.no_grad():
        a, b = plain.block_logits(tokens, hidden, anchors), src.block_logits(tokens, hidden, anchors)
    assert torch.isfinite(a).all() and _rel(a, b) < 0.5


def test_expand_layers_with_zeroed_repeats_keeps_the_function(tmp_path):
    src = DrafterTrain(_cfg(), HT, V, torch.arange(V), seed=2, std=0.05)
    d = dt.save_dir(src, tmp_path / "src", "export")
    out = dt.main(["expand", "--source", str(d), "--order", "0,1,0,1,1", "--out", str(tmp_path / "x")])
    big = dt.load_dir(out)
    assert big.cfg.num_layers == 5 and dt.manifest_of(out)["order"] == [0, 1, 0, 1, 1]
    assert torch.equal(big.layers[2].w_qkv, src.layers[0].w_qkv) and big.layers[3].w_o.abs().max() == 0
    for tokens, hidden, anchors in _calib(2, seed=3):
        with torch.no_grad():
            assert torch.allclose(big.block_logits(tokens, hidden, anchors), src.block_logits(tokens, hidden, anchors),
                                  rtol=1e-5, atol=1e-6)
    copied = dt.expand_layers(src, [0, 1, 0], zero_repeats=False)
    assert torch.equal(copied.layers[2].w_o, src.layers[0].w_o)
    with pytest.raises(ValueError):
        dt.expand_layers(_hc_source(True), [0, 0])


def test_deploy_copy_block_fp8_and_verification(tmp_path):
    from safetensors.torch import load_file
    from arc_forge_2026_b200.quant.fp8 import dequant_weight_block, quantize_weight_block
    src = DrafterTrain(_cfg(), HT, V, torch.arange(V), seed=4, std=0.05)
    d = dt.save_dir(src, tmp_path / "src", "export")
    out = dt.main(["deploy", "--source", str(d), "--fp8", "attn", "--out", str(tmp_path / "dep")])
    t = load_file(str(out / "layer-0.safetensors"))
    assert t["w_qkv"].dtype == torch.float8_e4m3fn and "w_o_scale_inv" in t and t["w13"].dtype == torch.float32
    back = dt.load_dir(out)
    q, s = quantize_weight_block(src.layers[0].w_o.detach())
    assert torch.equal(back.layers[0].w_o, dequant_weight_block(q, s))
    assert torch.equal(back.layers[1].w2, src.layers[1].w2.detach())
    assert not list(tmp_path.glob("*.tmp-*"))
    raw = bytearray((out / "layer-1.safetensors").read_bytes())
    raw[-1] ^= 0xFF
    (out / "layer-1.safetensors").write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="sha256"):
        dt.load_dir(out)


def test_export_of_a_trainer_checkpoint_loads_back(tmp_path):
    src = DrafterTrain(_cfg(), HT, V, torch.arange(V), seed=5, std=0.05)
    d = dt.save_dir(src, tmp_path / "init", "export")
    with torch.no_grad():
        src.layers[0].w_o.mul_(2.0)
    torch.save(src.state_dict(), tmp_path / "ckpt.pt")
    out = dt.main(["export", "--checkpoint", str(tmp_path / "ckpt.pt"), "--config", str(d),
                   "--out", str(tmp_path / "exp")])
    assert torch.equal(dt.load_dir(out).layers[0].w_o, src.layers[0].w_o.detach())
    with pytest.raises(ValueError, match="plain / dense"):
        _hc_source(True).export_to(None)
