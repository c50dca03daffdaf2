"""Distributed checkpoints of the trainers through ``torch.distributed.checkpoint`` (DCP), the format the reference
resumes QAD from (FSDP2 + DCP, ``training/work/qwen38fn_qad/train_qad.py:140-167``), loadable at another world size.

Layout of a checkpoint directory:

    .metadata, __<rank>_0.distcp     DCP storage
    trainer.json                     {format "afb-dcp-v1", step, plan, world, groups: [{n, chunk, step}]}

Keys: ``model.<parameter name>`` for every trainable master (replicated on every rank under ZeRO: DCP writes it
once), and the optimizer moments of group ``g`` as flat vectors over the group's parameters in order, cut into the
element ranges the ranks owned: ``optim.g<g>.m.<lo>-<hi>`` / ``.v.<lo>-<hi>``. A load reads, for its own range,
every saved range that overlaps it, so a run saved on N ranks resumes on M. ``AdamWBF16`` (one process, per-
parameter state), ``ShardedAdamW`` and ``FusedShardedAdamW`` all map to this flat form.
"""
from __future__ import annotations

import json
import os
from pathlib import Path

import torch
import torch.distributed as dist

FORMAT = "afb-dcp-v1"


def _rank_world(opt):
    if getattr(opt, "sharded", False):
        return opt.rank, opt.world
    return 0, 1


def _groups(opt):
    """Per parameter group: params, n, chunk, local range [lo, hi), flat local m / v views, step."""
    rank, world = _rank_world(opt)
    out = []
    if getattr(opt, "sharded", False):
        for g in opt.groups:
            params = g["params"]
            n = sum(p.numel() for p in params)
            chunk = g["chunk"]
            lo, hi = min(n, rank * chunk), min(n, (rank + 1) * chunk)
            out.append({"params": params, "n": n, "chunk": chunk, "lo": lo, "hi": hi,
                        "m": g["m"][: hi - lo], "v": g["v"][: hi - lo], "step": g["step"], "ref": g})
        return out
    for group in opt.param_groups:  # AdamWBF16: materialise the flat moments (zeros before the first step)
        params = list(group["params"])
        ms, vs, steps = [], [], [0]
        for p in params:
            st = opt.state.get(p, {})
            ms.append(st["m"].reshape(-1) if "m" in st else torch.zeros(p.numel(), dtype=torch.bfloat16, device=p.device))
            vs.append(st["v"].reshape(-1) if "v" in st else torch.zeros(p.numel(), dtype=torch.bfloat16, device=p.device))
            steps.append(st.get("step", 0))
        n = sum(p.numel() for p in params)
        out.append({"params": params, "n": n, "chunk": n, "lo": 0, "hi": n, "m": torch.cat(ms) if ms else None,
                    "v": torch.cat(vs) if vs else None, "step": max(steps), "ref": group})
    return out


def save_dcp(path, student, opt, step: int, plan: str, extra: dict | None = None) -> Path:
    import torch.distributed.checkpoint as dcp
    path = Path(path)
    rank, world = _rank_world(opt)
    groups = _groups(opt)
    sd = {f"model.{n}": p.detach() for n, p in student.named_parameters() if p.requires_grad}
    for gi, g in enumerate(groups):
        if g["hi"] > g["lo"]:
            sd[f"optim.g{gi}.m.{g['lo']}-{g['hi']}"] = g["m"]
            sd[f"optim.g{gi}.v.{g['lo']}-{g['hi']}"] = g["v"]
    if rank == 0:
        path.mkdir(parents=True, exist_ok=True)
    if dist.is_initialized() and world > 1:
        dist.barrier()
    dcp.save(sd, checkpoint_id=str(path))
    if rank == 0:
        meta = {"format": FORMAT, "step": step, "plan": plan, "world": world,
                "groups": [{"n": g["n"], "chunk": g["chunk"], "step": g["step"]} for g in groups], **(extra or {})}
        (path / "trainer.json.tmp").write_text(json.dumps(meta) + "\n")
        os.replace(path / "trainer.json.tmp", path / "trainer.json")
    if dist.is_initialized() and world > 1:
        dist.barrier()
    return path


def is_dcp(path) -> bool:
    p = Path(path) / "trainer.json"
    return p.exists() and json.loads(p.read_text()).get("format") == FORMAT


@torch.no_grad()
def load_dcp(path, student, opt, plan: str | None = None) -> int:
    """Restore masters and optimizer moments saved by :func:`save_dcp` (any world size); returns the step."""
    import torch.distributed.checkpoint as dcp
    path = Path(path)
    meta = json.loads((path / "trainer.json").read_text())
    if meta.get("format") != FORMAT:
        raise ValueError(f"{path} is not a {FORMAT} checkpoint")
    if plan is not None and meta["plan"] != plan:
        raise RuntimeError(f"checkpoint plan {meta['plan']} != this run's plan {plan}: refusing to resume")
    groups = _groups(opt)
    if len(groups) != len(meta["groups"]) or any(g["n"] != m["n"] for g, m in zip(groups, meta["groups"])):
        raise ValueError("parameter groups differ from the checkpoint's")
    sd = {f"model.{n}": p.detach() for n, p in student.named_parameters() if p.requires_grad}
    pieces = []  # (group, old lo, old hi, m buffer, v buffer)
    for gi, (g, m) in enumerate(zip(groups, meta["groups"])):
        old_chunk = m["chunk"]
        for r in range(meta["world"]):
            olo, ohi = min(m["n"], r * old_chunk), min(m["n"], (r + 1) * old_chunk)
            if ohi <= olo or ohi <= g["lo"] or olo >= g["hi"]:
                continue
            dev = g["params"][0].device
            mb = torch.empty(ohi - olo, dtype=torch.bfloat16, device=dev)
            vb = torch.empty_like(mb)
            sd[f"optim.g{gi}.m.{olo}-{ohi}"], sd[f"optim.g{gi}.v.{olo}-{ohi}"] = mb, vb
            pieces.append((gi, olo, ohi, mb, vb))
    dcp.load(sd, checkpoint_id=str(path))
    for gi, olo, ohi, mb, vb in pieces:
        g = groups[gi]
        lo, hi = max(olo, g["lo"]), min(ohi, g["hi"])
        g["m"][lo - g["lo"]:hi - g["lo"]].copy_(mb[lo - olo:hi - olo])
        g["v"][lo - g["lo"]:hi - g["lo"]].copy_(vb[lo - olo:hi - olo])
    for g, m in zip(groups, meta["groups"]):
        if getattr(opt, "sharded", False):
            g["ref"]["step"] = m["step"]
        else:  # scatter the flat moments back into AdamWBF16's per-parameter state
            o = 0
            for p in g["params"]:
                k = p.numel()
                opt.state[p] = {"step": m["step"], "m": g["m"][o:o + k].view_as(p).clone(),
                                "v": g["v"][o:o + k].view_as(p).clone()}
                o += k
    return int(meta["step"])
