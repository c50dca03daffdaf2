"""RL / LoRA pieces on CPU: adapters (identity at init, gradients, exact merge), fn-lora-merged-v2 export, the
delta-only weight patch, routing replay, and the HTTP trainer service taking optimizer steps."""
import json

import pytest
import torch
import torch.nn.functional as F

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.formats.weight_patch import apply_patch, write_patch
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
    key = "model.layers.0.in_proj_ba.weight"
    assert tensors[key].dtype == torch.bfloat16 and info[key]["changed"] > 0
    assert tensors["model.layers.0.in_proj_qkvz.weight"].dtype == torch.float8_e4m3fn
    assert "model.layers.0.in_proj_qkvz.weight_scale_inv" in tensors


def test_merged_export_and_weight_patch(tmp_path):
    st = _student(1)
    attach_lora(st, r=4, alpha=8.0)
    with torch.no_grad():
        for layer in st.layers:
            for ad in layer.lora.values():
                ad.B.normal_(0, 0.01)
    d = export_merged(st, tmp_path / "v000001", 1)
    assert (d / "DONE").exists()
    man = json.loads((d / "merged_manifest.json").read_text())
    assert man["format"] == "fn-lora-merged-v2" and man["weight_version"] == 1 and man["lora_rank"] == 4
    with pytest.raises(FileExistsError):
        export_merged(st, tmp_path / "v000001", 2)
    base = {"a": torch.randn(4, 4).bfloat16(), "b": torch.randn(3).bfloat16(), "c": torch.zeros(2)}
    new = dict(base, b=base["b"] + 1)
    p = write_patch(base, new, tmp_path / "patch")
    assert json.loads((p / "patch_manifest.json").read_text())["changed"] == 1
    out = apply_patch(base, p)
    assert torch.equal(out["b"], new["b"]) and out["a"] is base["a"]
    with pytest.raises(RuntimeError):
        apply_patch(dict(base, b=base["b"] * 2), p)


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
