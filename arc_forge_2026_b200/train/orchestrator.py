"""RL orchestrator: rollouts on the serving replicas, rewards, trainer steps, publish, weight update -- the sync
(rounds) and stream (continuous groups) pipelines of the reference's ``training/work/qwen38fn_rl/orchestrator.py:1-70``
(its task harnesses and audits are application layer).

One round:

1. P prompts (seeded draw from the prompt file), G completions each, spread round-robin over the replicas
   (``POST /v1/completions`` with ``token_ids`` back; ``logprobs`` are used as the behaviour log-probabilities when
   the replica returns them, else the step is on-policy);
2. rewards from a pluggable ``reward(prompt_ids, completion_ids) -> float`` (``module:function``), advantages
   normalised within each prompt's group of G (mean 0, unit std; a constant group gets 0);
3. the trainer takes one step over the round: ``/begin``, one ``/accumulate`` per group, ``/step``;
4. ``/publish`` with the next weight version, then the replica controller's ``/update_weights_from_disk`` with the
   published path (a partial update closes the controller and stops the run);
5. ``state.json`` (atomic) and one line of ``rounds.jsonl``.

A ``STOP`` file in the run directory ends the run at the next round boundary; a restart resumes after the last
completed round. Transports are injectable (``http_json`` by default) so tests run replicas and trainer in-process.

Stream mode (:class:`StreamOrchestrator`, ``--pipeline stream``): no rounds. A dispatcher keeps up to
``max_groups_in_flight`` groups (one prompt x G samples) running, launching the next as one finishes (prompts follow a
seeded per-epoch shuffle); finished groups are recorded in ``groups.jsonl`` with the weight version they were sampled
under and enter the pool, and nothing new launches while the pool holds ``max_pooled_groups`` unconsumed groups
(back-pressure). The learner takes ``batch_groups`` live groups in completion order, drops groups older than
``max_staleness`` versions as dead, trains one step, publishes V + 1, updates the replicas in place and appends one
line to ``batches.jsonl``. STOP: nothing new launches, groups in flight finish into the pool, and the run ends after
the current batch; a restart puts recorded, unconsumed groups back into the pool. Quarantine: a group whose rollout
fails (replica error, bad output, ``group_timeout``) is recorded in ``quarantine.jsonl`` and skipped while the run
continues; the circuit breaker stops the run when the same error signature repeats ``breaker_repeats`` times within
``breaker_window`` seconds, or when quarantined groups exceed ``breaker_max_share`` of the last ``breaker_recent``.

    python -m arc_forge_2026_b200.train.orchestrator --run run1 --prompts prompts.jsonl \\
        --replicas http://127.0.0.1:30571 --controller http://127.0.0.1:30570 --trainer http://127.0.0.1:31000 \\
        --reward mypkg.rewards:score --rounds 100
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import random
import threading
import time
from collections import deque
from dataclasses import dataclass
from pathlib import Path

from ..serve.replicas import http_json


class Orchestrator:
    def __init__(self, run_dir, prompts: list[list[int]], replicas: list[str], trainer: str, reward,
                 controller: str | None = None, prompts_per_round: int = 4, group: int = 4, max_tokens: int = 32,
                 algo: str = "bpo", seed: int = 0, transport=None):
        self.run = Path(run_dir)
        self.run.mkdir(parents=True, exist_ok=True)
        self.prompts = prompts
        self.replicas, self.trainer, self.controller = list(replicas), trainer, controller
        self.reward = reward
        self.P, self.G, self.max_tokens, self.algo, self.seed = prompts_per_round, group, max_tokens, algo, seed
        self.t = transport or http_json
        st = self.run / "state.json"
        self.state = json.loads(st.read_text()) if st.exists() else {"round": 0, "weight_version": 0}

    def _call(self, root, method, path, body=None):
        status, out = self.t(root, method, path, body)
        if status != 200:
            raise RuntimeError(f"{root}{path}: HTTP {status}: {out}")
        return out

    def _save_state(self):
        tmp = self.run / "state.json.tmp"
        tmp.write_text(json.dumps(self.state) + "\n")
        os.replace(tmp, self.run / "state.json")

    def rollout(self, rnd: int):
        rng = random.Random(self.seed * 1_000_003 + rnd)
        picks = [rng.randrange(len(self.prompts)) for _ in range(self.P)]
        groups, k = [], 0
        for pi in picks:
            prompt = self.prompts[pi]
            outs = []
            for g in range(self.G):
                rep = self.replicas[k % len(self.replicas)]
                k += 1
                r = self._call(rep, "POST", "/v1/completions",
                               {"prompt": prompt, "max_tokens": self.max_tokens, "logprobs": True,
                                "rid": f"rl-{rnd}-{pi}-{g}"})
                ch = r["choices"][0]
                lp = ch.get("logprobs")
                outs.append({"ids": ch["token_ids"], "logprobs": lp.get("token_logprobs") if isinstance(lp, dict)
                             else None})
            groups.append((prompt, outs))
        return groups

    @staticmethod
    def advantages(rewards: list[float]) -> list[float]:
        m = sum(rewards) / len(rewards)
        sd = math.sqrt(sum((r - m) ** 2 for r in rewards) / len(rewards))
        return [0.0 if sd < 1e-8 else (r - m) / sd for r in rewards]

    @staticmethod
    def batch(prompt, outs, advs):
        """ids / labels / mask over prompt + completion (completion tokens trained), right-padded with 0."""
        seqs = [list(prompt) + list(o["ids"]) for o in outs]
        T = max(len(s) for s in seqs) - 1
        ids, labels, mask, beh = [], [], [], []
        have_lp = all(o["logprobs"] is not None for o in outs)
        for s, o in zip(seqs, outs):
            x, y = s[:-1], s[1:]
            m = [0] * (len(prompt) - 1) + [1] * len(o["ids"])
            pad = T - len(x)
            ids.append(x + [0] * pad)
            labels.append(y + [0] * pad)
            mask.append(m + [0] * pad)
            if have_lp:
                beh.append([0.0] * (len(prompt) - 1) + list(o["logprobs"]) + [0.0] * pad)
        b = {"ids": ids, "labels": labels, "mask": mask, "advantages": advs}
        if have_lp:
            b["behavior_logp"] = beh
        return b

    def round(self) -> dict:
        rnd = self.state["round"]
        t0 = time.perf_counter()
        groups = self.rollout(rnd)
        rewards_all = []
        self._call(self.trainer, "POST", "/begin", {})
        for prompt, outs in groups:
            rewards = [float(self.reward(prompt, o["ids"])) for o in outs]
            rewards_all += rewards
            self._call(self.trainer, "POST", "/accumulate",
                       {"batch": self.batch(prompt, outs, self.advantages(rewards)), "algo": self.algo})
        report = self._call(self.trainer, "POST", "/step", {})
        v = self.state["weight_version"] + 1
        pub = self._call(self.trainer, "POST", "/publish", {"weight_version": v})
        if self.controller is not None:
            self._call(self.controller, "POST", "/update_weights_from_disk",
                       {"model_path": pub["path"], "weight_version": v})
        self.state = {"round": rnd + 1, "weight_version": v, "published": pub["path"]}
        rec = {"round": rnd, "weight_version": v, "reward_mean": sum(rewards_all) / len(rewards_all),
               "samples": len(rewards_all), "trainer": report, "seconds": round(time.perf_counter() - t0, 3)}
        with open(self.run / "rounds.jsonl", "a") as f:
            f.write(json.dumps(rec) + "\n")
        self._save_state()
        return rec

    def run_rounds(self, rounds: int) -> list[dict]:
        out = []
        while self.state["round"] < rounds:
            if (self.run / "STOP").exists():
                break
            out.append(self.round())
        return out


@dataclass
class StreamConfig:
    max_groups_in_flight: int = 4
    max_pooled_groups: int = 8
    batch_groups: int = 2
    max_staleness: int = 1
    group_timeout: float | None = None
    breaker_repeats: int = 3
    breaker_window: float = 3600.0
    breaker_recent: int = 20
    breaker_max_share: float = 0.5


class CircuitOpen(RuntimeError):
    """The stream's circuit breaker stopped the run (see the message for the error signature or share)."""


class StreamOrchestrator(Orchestrator):
    def __init__(self, run_dir, prompts, replicas, trainer, reward, controller=None, group: int = 4,
                 max_tokens: int = 32, algo: str = "bpo", seed: int = 0, transport=None, cfg: StreamConfig | None = None,
                 clock=time.monotonic):
        super().__init__(run_dir, prompts, replicas, trainer, reward, controller, 1, group, max_tokens, algo, seed,
                         transport)
        self.cfg = cfg or StreamConfig()
        self.clock = clock
        self.lock = threading.Condition()
        st = self.run / "stream.json"
        self.sstate = json.loads(st.read_text()) if st.exists() else {"weight_version": 0, "next_group": 0,
                                                                      "batches": 0}
        # resume: recorded groups not consumed by a batch go back to the pool, in completion order
        consumed = set()
        bpath = self.run / "batches.jsonl"
        if bpath.exists():
            for line in bpath.read_text().splitlines():
                rec = json.loads(line)
                consumed.update(rec["groups"] + rec["dead"])
        self.pool: list[dict] = []
        gpath = self.run / "groups.jsonl"
        recorded = set()
        if gpath.exists():
            for line in gpath.read_text().splitlines():
                rec = json.loads(line)
                recorded.add(rec["group"])
                if rec["status"] == "live" and rec["group"] not in consumed:
                    self.pool.append(rec)
        qpath = self.run / "quarantine.jsonl"
        if qpath.exists():
            recorded.update(json.loads(line)["group"] for line in qpath.read_text().splitlines())
        if any(g >= self.sstate["next_group"] for g in recorded):
            raise RuntimeError("groups.jsonl holds groups past stream.json's next_group: not a clean resume point")
        self.in_flight = 0
        self.stopping = False
        self.tripped: str | None = None
        self.sig_times: dict[str, deque] = {}
        self.recent: deque = deque(maxlen=self.cfg.breaker_recent)
        self.replica_turn = 0

    def _prompt_index(self, gi: int) -> int:
        n = len(self.prompts)
        order = list(range(n))
        random.Random(self.seed * 1_000_003 + gi // n).shuffle(order)
        return order[gi % n]

    def _append(self, name: str, rec: dict):
        with open(self.run / name, "a") as f:
            f.write(json.dumps(rec) + "\n")

    def _run_group(self, gi: int, version: int) -> dict:
        pi = self._prompt_index(gi)
        prompt, t0, outs = self.prompts[pi], self.clock(), []
        for g in range(self.G):
            with self.lock:
                rep = self.replicas[self.replica_turn % len(self.replicas)]
                self.replica_turn += 1
            r = self._call(rep, "POST", "/v1/completions", {"prompt": prompt, "max_tokens": self.max_tokens,
                                                            "logprobs": True, "rid": f"rl-g{gi}-{g}"})
            ch = r["choices"][0]
            ids = ch.get("token_ids")
            if not isinstance(ids, list) or not ids:
                raise ValueError("completion without token ids")
            lp = ch.get("logprobs")
            outs.append({"ids": ids, "logprobs": lp.get("token_logprobs") if isinstance(lp, dict) else None})
            if self.cfg.group_timeout is not None and self.clock() - t0 > self.cfg.group_timeout:
                raise TimeoutError("group timeout")
        rewards = [float(self.reward(prompt, o["ids"])) for o in outs]
        return {"group": gi, "prompt": pi, "weight_version": version, "status": "live", "outs": outs,
                "rewards": rewards}

    def _worker(self, gi: int, version: int):
        try:
            rec = self._run_group(gi, version)
        except Exception as e:  # noqa: BLE001 -- a group's failure is data for the quarantine, not a crash
            self._quarantine(gi, e)
            return
        with self.lock:
            self._append("groups.jsonl", rec)
            self.pool.append(rec)
            self.recent.append(False)
            self.in_flight -= 1
            self.lock.notify_all()

    def _quarantine(self, gi: int, e: Exception):
        sig = f"{type(e).__name__}: {(str(e).splitlines() or [''])[0][:200]}"
        now = self.clock()
        with self.lock:
            self._append("quarantine.jsonl", {"group": gi, "signature": sig, "time": now})
            times = self.sig_times.setdefault(sig, deque())
            times.append(now)
            while times and now - times[0] > self.cfg.breaker_window:
                times.popleft()
            self.recent.append(True)
            if len(times) >= self.cfg.breaker_repeats:
                self.tripped = f"{sig!r} {len(times)} times within {self.cfg.breaker_window:g} s"
            elif (len(self.recent) == self.recent.maxlen and
                  sum(self.recent) / len(self.recent) > self.cfg.breaker_max_share):
                self.tripped = f"{sum(self.recent)} of the last {len(self.recent)} groups quarantined"
            self.in_flight -= 1
            self.lock.notify_all()

    def _dispatch(self):
        c = self.cfg
        while True:
            with self.lock:
                while not (self.stopping or self.tripped) and (
                        self.in_flight >= c.max_groups_in_flight or len(self.pool) >= c.max_pooled_groups):
                    self.lock.wait(0.05)
                if self.stopping or self.tripped or (self.run / "STOP").exists():
                    return
                gi = self.sstate["next_group"]
                self.sstate["next_group"] = gi + 1
                self.in_flight += 1
                version = self.sstate["weight_version"]
            threading.Thread(target=self._worker, args=(gi, version), daemon=True).start()

    def _save_stream(self):
        tmp = self.run / "stream.json.tmp"
        tmp.write_text(json.dumps(self.sstate) + "\n")
        os.replace(tmp, self.run / "stream.json")

    def _train_batch(self, take: list[dict], dead: list[dict]) -> dict:
        t0 = time.perf_counter()
        self._call(self.trainer, "POST", "/begin", {})
        rewards = []
        for rec in take:
            rewards += rec["rewards"]
            self._call(self.trainer, "POST", "/accumulate",
                       {"batch": self.batch(self.prompts[rec["prompt"]], rec["outs"], self.advantages(rec["rewards"])),
                        "algo": self.algo})
        report = self._call(self.trainer, "POST", "/step", {})
        v = self.sstate["weight_version"] + 1
        pub = self._call(self.trainer, "POST", "/publish", {"weight_version": v})
        if self.controller is not None:
            self._call(self.controller, "POST", "/update_weights_from_disk",
                       {"model_path": pub["path"], "weight_version": v, "flush_cache": False})
        rec = {"batch": self.sstate["batches"], "weight_version": v, "groups": [r["group"] for r in take],
               "dead": [r["group"] for r in dead], "sampled_versions": [r["weight_version"] for r in take],
               "reward_mean": sum(rewards) / len(rewards), "samples": len(rewards), "trainer": report,
               "seconds": round(time.perf_counter() - t0, 3)}
        with self.lock:
            self._append("batches.jsonl", rec)
            self.sstate["weight_version"] = v
            self.sstate["batches"] += 1
            self._save_stream()
        return rec

    def run_stream(self, max_batches: int) -> list[dict]:
        """Train up to ``max_batches`` batches (fewer after STOP); raises :class:`CircuitOpen` when the breaker
        trips. Groups still in flight at the end finish into groups.jsonl for the next run."""
        out = []
        disp = threading.Thread(target=self._dispatch, daemon=True)
        disp.start()
        try:
            while self.sstate["batches"] < max_batches:
                with self.lock:
                    while True:
                        if self.tripped:
                            raise CircuitOpen(self.tripped)
                        live = [r for r in self.pool if r["weight_version"] >= self.sstate["weight_version"] -
                                self.cfg.max_staleness]
                        stopping = (self.run / "STOP").exists()
                        if len(live) >= self.cfg.batch_groups or (stopping and live and self.in_flight == 0):
                            break
                        if stopping and self.in_flight == 0:
                            return out
                        self.lock.wait(0.05)
                    v = self.sstate["weight_version"]
                    take, dead, rest = [], [], []
                    for r in self.pool:  # completion order
                        if r["weight_version"] < v - self.cfg.max_staleness:
                            dead.append(r)
                        elif len(take) < self.cfg.batch_groups:
                            take.append(r)
                        else:
                            rest.append(r)
                    self.pool = rest
                    self.lock.notify_all()
                out.append(self._train_batch(take, dead))
        finally:
            with self.lock:
                self.stopping = True
                self.lock.notify_all()
            disp.join()
            with self.lock:  # let the groups in flight land in groups.jsonl
                t_end = time.monotonic() + 60
                while self.in_flight and time.monotonic() < t_end:
                    self.lock.wait(0.05)
            self._save_stream()
        return out


def _load_reward(spec: str):
    mod, _, fn = spec.partition(":")
    return getattr(importlib.import_module(mod), fn)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--run", type=Path, required=True)
    ap.add_argument("--prompts", type=Path, required=True, help="jsonl with {'ids': [...]} per line")
    ap.add_argument("--replicas", required=True)
    ap.add_argument("--controller", default=None)
    ap.add_argument("--trainer", required=True)
    ap.add_argument("--reward", required=True, help="module:function(prompt_ids, completion_ids) -> float")
    ap.add_argument("--rounds", type=int, default=10)
    ap.add_argument("--prompts-per-round", dest="P", type=int, default=4)
    ap.add_argument("--group", type=int, default=4)
    ap.add_argument("--max-tokens", dest="max_tokens", type=int, default=64)
    ap.add_argument("--algo", default="bpo", choices=["bpo", "mis"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--pipeline", choices=["sync", "stream"], default="sync")
    ap.add_argument("--batches", type=int, default=10, help="stream: training batches")
    ap.add_argument("--max-groups-in-flight", dest="max_groups_in_flight", type=int, default=4)
    ap.add_argument("--max-pooled-groups", dest="max_pooled_groups", type=int, default=8)
    ap.add_argument("--batch-groups", dest="batch_groups", type=int, default=2)
    ap.add_argument("--max-staleness", dest="max_staleness", type=int, default=1)
    ap.add_argument("--group-timeout", dest="group_timeout", type=float, default=None)
    a = ap.parse_args(argv)
    prompts = [json.loads(line)["ids"] for line in a.prompts.read_text().splitlines() if line.strip()]
    if a.pipeline == "stream":
        cfg = StreamConfig(a.max_groups_in_flight, a.max_pooled_groups, a.batch_groups, a.max_staleness,
                           a.group_timeout)
        orch = StreamOrchestrator(a.run, prompts, a.replicas.split(","), a.trainer, _load_reward(a.reward),
                                  a.controller, a.group, a.max_tokens, a.algo, a.seed, cfg=cfg)
        for rec in orch.run_stream(a.batches):
            print(json.dumps(rec), flush=True)
        return
    orch = Orchestrator(a.run, prompts, a.replicas.split(","), a.trainer, _load_reward(a.reward), a.controller, a.P,
                        a.group, a.max_tokens, a.algo, a.seed)
    for rec in orch.run_rounds(a.rounds):
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
