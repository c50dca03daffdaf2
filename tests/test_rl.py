"""RL / LoRA pieces on CPU: adapters (identity at init, gradients, exact merge), fn-lora-merged-v2 export, the
delta-only weight patch, routing replay, and the HTTP trainer service taking optimizer steps."""
import json
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.formats import weight_patch as wp
from arc_forge_2026_b200.train.lora import attach_lora, export_merged, merged_tensors
from arc_forge_2026_b200.train.routing_replay import RoutingReplay
from arc_forge_2026_b200.train.student import random_student


def _student(seed=0):
    return random_student(preset("tiny_cpu"), "cpu", seed=seed, checkpoint_layers=False)


def test_lora_identity_gradients_and_merge():
    st = _student()
    ids = torch.randint(0, st.cfg.vocab_size, (1, 24), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        h0 = st.hidden(ids)
    params = attach_lora(st, r=4, alpha=8.0)
    assert all(not p.requires_grad for n, p in st.named_parameters() if ".lora." not in n)
    h1 = st.hidden(ids)
    assert torch.equal(h0, h1.detach())  # B = 0: adapters start as the identity
    h1.pow(2).mean().backward()
    assert any(p.grad is not None and p.grad.abs().sum() > 0 for p in params)
    # merge of a bf16-served projection equals base + scale * B A
    layer = st.layers[0]
    ad = layer.lora["in_proj_ba"]
    with torch.no_grad():
        ad.B.normal_(0, 0.01)
    x = torch.randn(5, layer.in_proj_ba.shape[1])
    y = layer._lin("in_proj_ba", x, False)
    ref = F.linear(x, layer.in_proj_ba + ad.delta())
    assert torch.allclose(y, ref, atol=1e-5)
    tensors, info = merged_tensors(st)
    key = "model.layers.0.linear_attn.in_proj_ba.weight"
    assert tensors[key].dtype == torch.bfloat16 and info[key]["changed_elements"] > 0
    assert info[key]["format"] == "bf16"
    fk = "model.layers.0.linear_attn.in_proj_qkvz.weight"
    assert tensors[fk].dtype == torch.float8_e4m3fn and info[fk]["format"] == "fp8_e4m3_block128"
    assert info[fk]["scale_key"] == "model.layers.0.linear_attn.in_proj_qkvz.weight_scale_inv"
    assert info[info[fk]["scale_key"]]["format"] == "fp32_scale_inv"


def _package(tmp_path, seed=0):
    from arc_forge_2026_b200.formats.int3_package import package_tensors, write_package
    from arc_forge_2026_b200.models.reference import build_reference
    from arc_forge_2026_b200.quant.gptq import rtn_quantize
    from arc_forge_2026_b200.train.student import QADStudent
    cfg = preset("tiny_cpu")
    ref = build_reference(cfg, seed=seed)
    cs = []
    for moe in ref.moe_layers():
        c13, s13 = rtn_quantize(moe.w13.detach().float())
        c2, s2 = rtn_quantize(moe.w2.detach().float())
        cs.append((c13, s13.bfloat16(), c2, s2.bfloat16()))
    pkg = write_package(package_tensors(ref, cs), cfg, tmp_path / "pkg", shard_bytes=1 << 20)
    return pkg, QADStudent(cfg, ref, cs, checkpoint_layers=False)


def test_merged_export_overlay_and_weight_patch_in_the_reference_layout(tmp_path):
    """A merged RL version -> overlay (arcforge.kaggle.model_overlay.v1) -> weight patch
    (arcforge.kaggle.weight_patch.v1, per-shard patch-<shard> + patch.json): reading the package with the patch gives
    exactly the merged tensors, the untouched tensors stay the package's, and a tampered base is refused."""
    from arc_forge_2026_b200.formats.int3_package import read_package
    pkg, st = _package(tmp_path)
    attach_lora(st, r=4, alpha=8.0)
    with torch.no_grad():
        for layer in st.layers:
            for ad in layer.lora.values():
                ad.B.normal_(0, 0.05)
    d = export_merged(st, tmp_path / "v000003", 3, {"optimizer_step": 3, "run": "test"})
    man = json.loads((d / "merged_manifest.json").read_text())
    assert man["format"] == "fn-lora-merged-v2" and man["weight_version"] == "3" and man["lora_rank"] == 4
    assert man["tensors"] == len(man["keys"]) and all("merged_sha256" in e for e in man["keys"].values())
    with pytest.raises(FileExistsError):
        export_merged(st, tmp_path / "v000003", 4)
    sha = wp.file_sha(pkg / "deploy_manifest.json")
    ov = wp.build_overlay(pkg, sha, d, tmp_path / "overlay")
    assert ov["schema"] == "arcforge.kaggle.model_overlay.v1" and ov["report"]["replaced"] == man["tensors"]
    assert (tmp_path / "overlay" / "DONE").exists() and ov["rl_merged"]["optimizer_step"] == 3
    patch = wp.build_patch(pkg, tmp_path / "overlay", tmp_path / "patch")
    pdir = tmp_path / "patch"
    assert patch["schema"] == "arcforge.kaggle.weight_patch.v1"
    assert all(f.startswith("patch-model-") for f in patch["files"]) and (pdir / "patch.json").exists()
    assert 0 < len(patch["tensors"]) <= man["tensors"]
    _, base = read_package(pkg)
    _, viapatch = read_package(pkg, weight_patch=pdir)
    _, viamerged = read_package(pkg, merged=d)
    for k in base:
        assert torch.equal(viapatch[k].view(torch.uint8), viamerged[k].view(torch.uint8)), k
    assert any(not torch.equal(viapatch[k].view(torch.uint8), base[k].view(torch.uint8)) for k in patch["tensors"])
    # a patch is bound to its base package
    with pytest.raises(ValueError, match="patches the package"):
        wp.WeightPatch(pdir, "0" * 64)
    with pytest.raises(FileExistsError):
        wp.build_patch(pkg, tmp_path / "overlay", tmp_path / "patch")
    # the overlay names the base manifest it was made from: a package with other shard bytes is refused
    other, _ = _package(tmp_path / "b", seed=1)
    with pytest.raises(RuntimeError, match="hashes to"):
        wp.build_patch(other, tmp_path / "overlay", tmp_path / "patch2")


def test_routing_replay_forces_recorded_experts():
    st = _student(2)
    c = st.cfg
    ids = torch.randint(0, c.vocab_size, (1, 16), generator=torch.Generator().manual_seed(1))
    rep = RoutingReplay("observe", len(st.layers), c.num_experts_per_tok)
    rep.install(st)
    rep.set_routing(torch.zeros(16, len(st.layers), c.num_experts_per_tok, dtype=torch.long) - 1)
    with torch.no_grad():
        h_nat = st.hidden(ids)
    # record the natural choices, then force them: identical output, full agreement
    nat = []
    for layer in st.layers:
        layer.moe.replay = None
    x = F.embedding(ids, st.embed)
    from arc_forge_2026_b200.models import reference as R
    for layer in st.layers:
        y = R.rms_norm(x, layer.in_norm, c.rms_norm_eps)
        x2 = x + (layer._attn(y, 1, 16) if layer.kind == "full_attention" else layer._gdn(y, 1, 16))
        y2 = R.rms_norm(x2, layer.post_norm, c.rms_norm_eps).reshape(16, -1)
        _, nid = R.route(y2.float() @ layer.moe.router.t(), c.num_experts_per_tok, c.norm_topk_prob)
        nat.append(nid)
        x = layer(x)
    recorded = torch.stack(nat, 1)
    force = RoutingReplay("force", len(st.layers), c.num_experts_per_tok)
    force.install(st)
    force.set_routing(recorded)
    with torch.no_grad():
        h_forced = st.hidden(ids)
    assert torch.allclose(h_forced, h_nat, atol=1e-6)
    assert sum(force.stats["equal"]) == sum(force.stats["rows"]) == 16 * len(st.layers)
    force.set_routing(torch.roll(recorded, 1, dims=0))  # other experts: the output changes
    with torch.no_grad():
        assert not torch.allclose(st.hidden(ids), h_nat, atol=1e-4)


def test_rl_service_steps_publish_save(tmp_path):
    pytest.importorskip("fastapi")
    from fastapi.testclient import TestClient
    from arc_forge_2026_b200.train.rl_service import RLTrainer, create_app
    st = _student(3)
    tr = RLTrainer(st, tmp_path, lr=1e-2, r=4, alpha=8.0)
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, st.cfg.vocab_size, (2, 12), generator=g)
    labels = torch.randint(0, st.cfg.vocab_size, (2, 12), generator=g)
    batch = {"ids": ids.tolist(), "labels": labels.tolist(), "mask": [[1] * 12] * 2, "advantages": [1.0, 1.0],
             "behavior_logp": [[-8.3] * 12] * 2}
    with TestClient(create_app(tr)) as c:
        assert c.get("/health").json()["step"] == 0
        reps = [c.post("/train", json={"batch": batch, "algo": "mis"}).json() for _ in range(6)]
        # positive advantages: the labels' log-probabilities (ratio to the fixed behaviour) rise
        assert reps[-1]["ratio_mean"] > reps[0]["ratio_mean"]
        r = c.post("/train", json={"batch": batch, "algo": "bpo"}).json()
        assert r["step"] == 7 and r["tokens"] == 24
        assert (tmp_path / "merged" / "v000001" / "DONE").exists() is False
        assert c.post("/publish", json={"weight_version": 1}).status_code == 200
        assert (tmp_path / "merged" / "v000001" / "DONE").exists()
        assert c.post("/publish", json={"weight_version": 1}).status_code == 500  # versions must increase
        assert c.post("/save").json()["path"].endswith("checkpoint-7")


def test_rl_step_accumulated_over_calls_equals_one_call(tmp_path):
    """begin + accumulate(half) + accumulate(other half) + step gives the adapters of one /train over both halves
    (token-weighted gradient accumulation)."""
    from arc_forge_2026_b200.train.lora import lora_state
    from arc_forge_2026_b200.train.rl_service import RLTrainer
    g = torch.Generator().manual_seed(3)
    c = preset("tiny_cpu")
    B, T = 2, 12
    batch = {"ids": torch.randint(0, c.vocab_size, (B, T), generator=g),
             "labels": torch.randint(0, c.vocab_size, (B, T), generator=g),
             "mask": torch.tensor([[1] * T, [1] * 7 + [0] * 5]),
             "advantages": torch.tensor([0.5, -1.0]), "behavior_logp": -torch.rand(B, T, generator=g) * 3}
    one, acc = RLTrainer(_student(4), tmp_path / "a", lr=1e-2), RLTrainer(_student(4), tmp_path / "b", lr=1e-2)
    r1 = one.train({"batch": batch})
    acc.begin()
    for i in range(B):
        acc.accumulate({"batch": {k: v[i:i + 1] for k, v in batch.items()}})
    r2 = acc.step_opt()
    assert r2["tokens"] == r1["tokens"] == 19 and r2["batches"] == 2
    assert abs(r1["loss"] - r2["loss"]) < 1e-5 and abs(r1["grad_norm"] - r2["grad_norm"]) < 1e-4 * (1 + r1["grad_norm"])
    s1, s2 = lora_state(one.student), lora_state(acc.student)
    assert all(torch.allclose(s1[k].float(), s2[k].float(), atol=1e-6) for k in s1)
    with pytest.raises(RuntimeError):
        acc.step_opt()


def test_full_weight_rl_trains_the_projections_publishes_and_resumes(tmp_path):
    """--trainable full: fp32 masters of the LoRA targets and the shared experts of layers >= F train, nothing else
    moves; /publish writes the merged version from the masters; a resumed trainer passes the resume gate and
    continues exactly like an uninterrupted one, and a checkpoint whose masters do not re-export the published
    version is refused."""
    from safetensors.torch import load_file
    from arc_forge_2026_b200.train.rl_service import RLTrainer
    g = torch.Generator().manual_seed(5)
    c = preset("tiny_cpu")
    B, T = 2, 10
    batch = {"ids": torch.randint(0, c.vocab_size, (B, T), generator=g),
             "labels": torch.randint(0, c.vocab_size, (B, T), generator=g), "mask": torch.ones(B, T),
             "advantages": torch.tensor([1.0, -0.5]), "behavior_logp": -torch.rand(B, T, generator=g) * 3}
    st = _student(6)
    before = {n: p.detach().clone() for n, p in st.named_parameters()}
    tr = RLTrainer(st, tmp_path / "run", lr=1e-3, trainable="full", freeze_first_layers=1)
    trainable = {id(p) for p in tr.params}
    names = {n for n, p in st.named_parameters() if id(p) in trainable}
    assert names and not any(n.startswith("layers.0.") for n in names)
    assert all(p.dtype == torch.float32 for p in tr.params)
    for _ in range(3):
        rep = tr.train({"batch": batch})
    assert rep["step"] == 3 and rep["grad_norm"] > 0
    changed = {n for n, p in st.named_parameters() if not torch.equal(p.detach(), before[n])}
    assert changed and changed <= names, sorted(changed - names)[:3]
    path = Path(tr.publish({"weight_version": 1})["path"])
    man = json.loads((path / "merged_manifest.json").read_text())
    assert man["trainer"] == "full" and man["trained_keys"] == len(tr.full.slots)
    tensors = load_file(str(path / "model.safetensors"))
    w = tr.full.weights()
    key = next(k for k in w if k.endswith("o_proj.weight"))
    assert torch.equal(tensors[key], w[key].to(torch.bfloat16))
    assert man["keys"][key]["changed_elements"] > 0
    ck = Path(tr.save({})["path"])
    tr.train({"batch": batch})
    # resume from the checkpoint: the gate passes and the next step matches the uninterrupted trainer's
    tr2 = RLTrainer(_student(6), tmp_path / "run", lr=1e-3, trainable="full", freeze_first_layers=1)
    tr2.load(ck)
    tr2.train({"batch": batch})
    a, b = tr.full.weights(), tr2.full.weights()
    assert all(torch.equal(a[k], b[k]) for k in a)
    # a checkpoint whose masters were altered does not re-export the published version
    state = torch.load(ck / "trainer_state.pt", weights_only=False)
    state["full"][key] = state["full"][key] + 1e-2
    bad = tmp_path / "bad"
    bad.mkdir()
    torch.save(state, bad / "trainer_state.pt")
    tr3 = RLTrainer(_student(6), tmp_path / "run", lr=1e-3, trainable="full", freeze_first_layers=1)
    with pytest.raises(RuntimeError, match="resume gate"):
        tr3.load(bad)
