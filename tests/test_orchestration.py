"""RL orchestration on CPU: the replica controller (fan-out, fail-closed partial update, reset), the node topology
planner, and the synchronous orchestrator driving a real trainer service over in-process HTTP with fake replicas
(rounds, state / rounds.jsonl, STOP, resume)."""
import json
import random

import pytest

from arc_forge_2026_b200.serve.replicas import ReplicaError, Replicas
from arc_forge_2026_b200.train.topology import plan

fastapi = pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402


class FakeReplica:
    def __init__(self, fail_updates=False):
        self.updates, self.fail = [], fail_updates

    def __call__(self, method, path, body):
        if path == "/health":
            return 200, {"status": "ok"}
        if path == "/update_weights_from_disk":
            if self.fail:
                return 400, {"success": False, "message": "boom"}
            self.updates.append(body["model_path"])
            return 200, {"success": True}
        if path == "/v1/completions":
            rng = random.Random(body["rid"])
            ids = [rng.randrange(1, 40) for _ in range(body["max_tokens"])]
            return 200, {"choices": [{"token_ids": ids}]}
        return 404, {}


def test_replicas_fan_out_and_fail_closed():
    a, b = FakeReplica(), FakeReplica()
    reps = Replicas(["a", "b"], transport=lambda root, m, p, body: {"a": a, "b": b}[root](m, p, body))
    assert reps.health()["ok"]
    assert reps.update_weights("/w1")["weight_version"] == 1 and a.updates == b.updates == ["/w1"]
    with pytest.raises(ReplicaError):
        reps.update_weights("/w0", weight_version=1)  # versions must increase
    b.fail = True
    with pytest.raises(ReplicaError, match="partial"):
        reps.update_weights("/w2")
    assert reps.closed and not reps.health()["ok"]
    with pytest.raises(ReplicaError, match="closed"):
        reps.update_weights("/w3")
    b.fail = False
    assert reps.reset()["reopened"]
    assert reps.update_weights("/w3")["weight_version"] == 2  # the failed update never became a version


def test_topology_plan():
    p = plan("tp1x4", gpus=8)
    assert [r["gpus"] for r in p["replicas"]] == [[0], [1], [2], [3]]
    assert p["trainer"]["gpus"] == [4, 5, 6, 7] and p["trainer"]["world"] == 4
    assert p["controller"]["launch"]["argv"][-3].count(",") == 3
    with pytest.raises(ValueError):
        plan("ep1x9", gpus=8)
    with pytest.raises(ValueError):
        plan("ep2x2")


def test_sync_orchestrator_rounds_stop_and_resume(tmp_path):
    from arc_forge_2026_b200.config import preset
    from arc_forge_2026_b200.serve.replicas import create_app as controller_app
    from arc_forge_2026_b200.train.orchestrator import Orchestrator
    from arc_forge_2026_b200.train.rl_service import RLTrainer, create_app as trainer_app
    from arc_forge_2026_b200.train.student import random_student
    fakes = {"r0": FakeReplica(), "r1": FakeReplica()}
    ctrl = TestClient(controller_app(Replicas(["r0", "r1"], transport=lambda root, m, p, b: fakes[root](m, p, b))))
    trainer = RLTrainer(random_student(preset("tiny_cpu"), "cpu", seed=0, checkpoint_layers=False), tmp_path / "out",
                        lr=1e-3, r=4, alpha=8.0)
    tr = TestClient(trainer_app(trainer))

    def transport(root, method, path, body):
        if root in fakes:
            return fakes[root](method, path, body)
        client = {"ctrl": ctrl, "trainer": tr}[root]
        r = client.request(method, path, json=body)
        return r.status_code, r.json()

    prompts = [[3, 5, 7], [2, 4], [9, 9, 9, 9]]

    def reward(prompt, out):  # prefers small tokens
        return -sum(out) / len(out)

    def make():
        return Orchestrator(tmp_path / "run", prompts, ["r0", "r1"], "trainer", reward, controller="ctrl",
                            prompts_per_round=2, group=3, max_tokens=5, transport=transport)
    orch = make()
    recs = orch.run_rounds(2)
    assert [r["round"] for r in recs] == [0, 1] and recs[-1]["weight_version"] == 2
    assert trainer.step == 2 and trainer.weight_version == 2
    assert len(fakes["r0"].updates) == 2 and fakes["r0"].updates == fakes["r1"].updates
    lines = (tmp_path / "run" / "rounds.jsonl").read_text().splitlines()
    assert len(lines) == 2 and json.loads(lines[1])["samples"] == 6
    (tmp_path / "run" / "STOP").write_text("")
    assert make().run_rounds(5) == []
    (tmp_path / "run" / "STOP").unlink()
    again = make()  # resumes from state.json
    assert again.state["round"] == 2
    assert [r["round"] for r in again.run_rounds(3)] == [2]
    assert trainer.step == 3


def _stream_rig(tmp_path, replica=None):
    from arc_forge_2026_b200.config import preset
    from arc_forge_2026_b200.serve.replicas import create_app as controller_app
    from arc_forge_2026_b200.train.rl_service import RLTrainer, create_app as trainer_app
    from arc_forge_2026_b200.train.student import random_student
    fakes = {"r0": replica or FakeReplica(), "r1": replica or FakeReplica()}
    ctrl = TestClient(controller_app(Replicas(["r0", "r1"], transport=lambda root, m, p, b: fakes[root](m, p, b))))
    trainer = RLTrainer(random_student(preset("tiny_cpu"), "cpu", seed=0, checkpoint_layers=False), tmp_path / "out",
                        lr=1e-3, r=4, alpha=8.0)
    tr = TestClient(trainer_app(trainer))
    lock = __import__("threading").Lock()

    def transport(root, method, path, body):
        if root in fakes:
            return fakes[root](method, path, body)
        client = {"ctrl": ctrl, "trainer": tr}[root]
        with lock:  # one in-process client at a time
            r = client.request(method, path, json=body)
        return r.status_code, r.json()
    return fakes, trainer, transport


def test_stream_orchestrator_trains_batches_with_back_pressure_and_resumes(tmp_path):
    from arc_forge_2026_b200.train.orchestrator import StreamConfig, StreamOrchestrator
    fakes, trainer, transport = _stream_rig(tmp_path)
    prompts = [[3, 5, 7], [2, 4], [9, 9, 9, 9], [1, 1]]
    cfg = StreamConfig(max_groups_in_flight=2, max_pooled_groups=3, batch_groups=2, max_staleness=1)

    def make():
        return StreamOrchestrator(tmp_path / "run", prompts, ["r0", "r1"], "trainer", lambda p, o: -sum(o) / len(o),
                                  controller="ctrl", group=3, max_tokens=4, transport=transport, cfg=cfg)
    recs = make().run_stream(3)
    assert [r["weight_version"] for r in recs] == [1, 2, 3] and trainer.step == 3
    assert all(len(r["groups"]) == 2 for r in recs)
    used = [g for r in recs for g in r["groups"] + r["dead"]]
    assert len(used) == len(set(used))  # no group trained twice
    assert all(r["weight_version"] - 1 - max(r["sampled_versions"]) <= 1 for r in recs)  # staleness bound
    groups = [json.loads(x) for x in (tmp_path / "run" / "groups.jsonl").read_text().splitlines()]
    # back-pressure: never more than max_pooled + in flight launched beyond what was consumed
    assert len(groups) <= len(used) + cfg.max_pooled_groups + cfg.max_groups_in_flight
    assert fakes["r0"].updates and fakes["r0"].updates == fakes["r1"].updates
    # resume: recorded, unconsumed groups are trained first and nothing is trained twice
    again = make()
    pooled = {r["group"] for r in again.pool}
    recs2 = again.run_stream(5)
    assert [r["weight_version"] for r in recs2] == [4, 5]
    used2 = [g for r in recs2 for g in r["groups"] + r["dead"]]
    assert not set(used2) & set(used) and pooled <= set(used2) | {r["group"] for r in again.pool}
    # STOP: no new launches, the run ends
    (tmp_path / "run" / "STOP").write_text("")
    assert len(make().run_stream(9)) <= 2


class FlakyReplica(FakeReplica):
    """Fails every completion of the prompts it is told to, with the same message."""

    def __init__(self, bad_prompts):
        super().__init__()
        self.bad = bad_prompts

    def __call__(self, method, path, body):
        if path == "/v1/completions" and body["prompt"] in self.bad:
            return 503, {"error": "replica overloaded"}
        return super().__call__(method, path, body)


def test_stream_quarantine_keeps_running_and_the_breaker_trips(tmp_path):
    from arc_forge_2026_b200.train.orchestrator import CircuitOpen, StreamConfig, StreamOrchestrator
    prompts = [[3, 5, 7], [2, 4], [9, 9, 9, 9], [1, 1]]
    fakes, trainer, transport = _stream_rig(tmp_path, FlakyReplica([[2, 4]]))
    cfg = StreamConfig(max_groups_in_flight=2, max_pooled_groups=4, batch_groups=2, breaker_repeats=50,
                       breaker_recent=50)
    orch = StreamOrchestrator(tmp_path / "run", prompts, ["r0", "r1"], "trainer", lambda p, o: float(len(o)),
                              controller="ctrl", group=2, max_tokens=3, transport=transport, cfg=cfg)
    recs = orch.run_stream(3)  # one prompt in four fails: its groups are quarantined, training goes on
    assert len(recs) == 3
    q = [json.loads(x) for x in (tmp_path / "run" / "quarantine.jsonl").read_text().splitlines()]
    assert q and all("503" in r["signature"] for r in q)
    trained = {g for r in recs for g in r["groups"]}
    assert not trained & {r["group"] for r in q}
    # the same signature three times within the window opens the breaker
    run2 = tmp_path / "run2"
    fakes2, _, transport2 = _stream_rig(tmp_path / "b", FlakyReplica([[3, 5, 7], [2, 4], [9, 9, 9, 9], [1, 1]]))
    orch2 = StreamOrchestrator(run2, prompts, ["r0", "r1"], "trainer", lambda p, o: 0.0, controller="ctrl", group=2,
                               max_tokens=3, transport=transport2,
                               cfg=StreamConfig(max_groups_in_flight=2, breaker_repeats=3, breaker_window=3600))
    with pytest.raises(CircuitOpen, match="3 times"):
        orch2.run_stream(2)
    # a high quarantined share among the recent groups opens it too
    orch3 = StreamOrchestrator(tmp_path / "run3", prompts, ["r0", "r1"], "trainer", lambda p, o: 0.0,
                               controller="ctrl", group=2, max_tokens=3, transport=transport2,
                               cfg=StreamConfig(max_groups_in_flight=1, breaker_repeats=100, breaker_recent=4,
                                                breaker_max_share=0.5))
    with pytest.raises(CircuitOpen, match="quarantined"):
        orch3.run_stream(2)
