"""Synchronous RL orchestrator: rollouts on the serving replicas, rewards, one trainer step, publish, weight update
(the sync mode of the reference's ``training/work/qwen38fn_rl/orchestrator.py:1-70``; its stream and async
pipelines, quarantine and task harnesses are application layer).

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
import time
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
    a = ap.parse_args(argv)
    prompts = [json.loads(line)["ids"] for line in a.prompts.read_text().splitlines() if line.strip()]
    orch = Orchestrator(a.run, prompts, a.replicas.split(","), a.trainer, _load_reward(a.reward), a.controller, a.P,
                        a.group, a.max_tokens, a.algo, a.seed)
    for rec in orch.run_rounds(a.rounds):
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
