"""Split one 8-GPU B200 node between rollout replicas and the trainer, and write the launch plan (the reference's
``training/work/qwen38fn_rl/configure_b200.py`` topologies: tp2x2, tp1x4, tp1x6, tp1x5, tp1x3, tp1x2).

A topology reads ``ep<E>x<R>``: R rollout replicas of E GPUs each, GPUs counted from 0, the trainer on the GPUs
after them (``torchrun`` with one rank per GPU). The HTTP server runs one engine per process, so replicas are
single-GPU (E = 1); the reference's TP1 names map directly (tp1x4 -> ep1x4). Multi-GPU replicas (E > 1, expert
parallelism across the replica's ranks) are an engine feature (``bench.py --gpus N``) the server does not front yet.

    python -m arc_forge_2026_b200.train.topology --topology ep1x4 --gpus 8 --out run/plan.json

plan.json: {topology, gpus, replicas: [{name, gpus, port, url, launch}], controller: {port, url, launch},
trainer: {gpus, world, launch}}; ``launch`` are the commands (environment + argv) a launcher runs.
"""
from __future__ import annotations

import argparse
import json
import re
from pathlib import Path

ALIASES = {"tp1x4": "ep1x4", "tp1x6": "ep1x6", "tp1x5": "ep1x5", "tp1x3": "ep1x3", "tp1x2": "ep1x2"}


def plan(topology: str, gpus: int = 8, base_port: int = 30571, preset: str = "qwen3next_80b",
         trainer_args: str = "", host: str = "127.0.0.1") -> dict:
    topo = ALIASES.get(topology, topology)
    m = re.fullmatch(r"ep(\d+)x(\d+)", topo)
    if not m:
        raise ValueError(f"topology {topology!r}: expected ep<E>x<R> (or one of {sorted(ALIASES)})")
    ep, reps = int(m.group(1)), int(m.group(2))
    if ep != 1 or reps < 1:
        raise ValueError("replicas are single-GPU server processes (ep1x<R>, R >= 1)")
    used = ep * reps
    if used > gpus:
        raise ValueError(f"{reps} replicas x {ep} GPUs exceed the node's {gpus}")
    replicas = []
    for r in range(reps):
        ids = list(range(r * ep, (r + 1) * ep))
        port = base_port + r
        env = {"CUDA_VISIBLE_DEVICES": ",".join(map(str, ids))}
        argv = ["python", "-m", "arc_forge_2026_b200.serve.server", "--preset", preset, "--gpu", "--host", host,
                "--port", str(port)]
        replicas.append({"name": f"r{r}", "gpus": ids, "port": port, "url": f"http://{host}:{port}",
                         "launch": {"env": env, "argv": argv}})
    ctrl_port = base_port - 1
    controller = {"port": ctrl_port, "url": f"http://{host}:{ctrl_port}",
                  "launch": {"env": {}, "argv": ["python", "-m", "arc_forge_2026_b200.serve.replicas", "--backends",
                                                 ",".join(r["url"] for r in replicas), "--port", str(ctrl_port)]}}
    tgpus = list(range(used, gpus))
    trainer = {"gpus": tgpus, "world": len(tgpus)}
    if tgpus:
        trainer["launch"] = {"env": {"CUDA_VISIBLE_DEVICES": ",".join(map(str, tgpus))},
                             "argv": ["python", "-m", "torch.distributed.run", "--nnodes=1",
                                      f"--nproc-per-node={len(tgpus)}", "--master-addr", host, "--master-port",
                                      "29500", "-m", "arc_forge_2026_b200.train.rl_service"] + trainer_args.split()}
    return {"topology": topo, "gpus": gpus, "replicas": replicas, "controller": controller, "trainer": trainer}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--topology", required=True)
    ap.add_argument("--gpus", type=int, default=8)
    ap.add_argument("--base-port", dest="base_port", type=int, default=30571)
    ap.add_argument("--preset", default="qwen3next_80b")
    ap.add_argument("--trainer-args", dest="trainer_args", default="")
    ap.add_argument("--out", type=Path, required=True)
    a = ap.parse_args(argv)
    p = plan(a.topology, a.gpus, a.base_port, a.preset, a.trainer_args)
    a.out.parent.mkdir(parents=True, exist_ok=True)
    tmp = a.out.with_name(a.out.name + ".tmp")
    tmp.write_text(json.dumps(p, indent=1) + "\n")
    tmp.replace(a.out)
    print(json.dumps({"plan": str(a.out), "replicas": len(p["replicas"]), "trainer_gpus": p["trainer"]["gpus"]}))
    return p


if __name__ == "__main__":
    main()
