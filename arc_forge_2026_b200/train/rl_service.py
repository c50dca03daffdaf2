"""RL trainer service: HTTP-driven optimizer steps on the student with LoRA adapters or, with
``--trainable full``, on the projection weights themselves (the reference's
``training/work/qwen38fn_lora/train_rl_service.py:1-61`` and ``dense_full_rl.py:1-37``).

Full-weight mode: the LoRA's target projections of every layer past ``--freeze-first-layers`` plus the shared
expert's gate / up / down projections are the trainable set, as fp32 masters (a bf16 master would drop most updates:
an RL step's lr times the update is below the bf16 spacing of |w|) with fp32 AdamW state; the forward multiplies the
bf16 cast (or the block-FP8 QAT weight) of the master, as deployed. Everything else stays frozen. ``/publish`` writes
the merged version from the masters (trainer "full"); ``/save`` checkpoints masters and optimizer; a resumed trainer
re-exports its restored masters at the checkpoint's weight version and refuses to continue unless that equals the
published version byte for byte (the resume gate).

Rank 0 serves HTTP; each request becomes one command that every rank executes (the command is broadcast over a
gloo group with ``broadcast_object_list``, so the GPU process group carries only gradients). Routes:

    GET  /health                       {ok, step, weight_version, busy}
    POST /train   {batch | batch_path, algo?, clip?, cap?}
                                       one optimizer step: forward, per-token log-probabilities under logits / T,
                                       BPO (clipped ratio) or MIS (truncated importance weight) loss, backward into
                                       the adapters, gradients averaged over ranks, global-norm clip, AdamW
    POST /begin                        start a step accumulated over several calls (zeroes the gradients)
    POST /accumulate {batch | batch_path, algo?, clip?, cap?}
                                       forward + backward of one micro-batch; gradients add up (token-weighted)
    POST /step                         apply the accumulated step: gradients / tokens of the step, averaged over
                                       ranks, clipped, AdamW
    POST /publish {weight_version}     merged adapters -> <out>/merged/v<version:06d> (``fn-lora-merged-v2``); versions
                                       must increase
    POST /save                         <out>/checkpoint-<step>/ (adapters + optimizer state + step), via .tmp rename
    POST /stop

Batch (``batch`` inline or a ``torch.save`` file at ``batch_path``): ``ids`` [B, T] int64 input tokens, ``labels``
[B, T] int64 next tokens, ``mask`` [B, T] (1 = trained), ``advantages`` [B, T] or [B], ``behavior_logp`` [B, T]
(the sampler's log-probabilities; absent: on-policy), optional ``temperature`` (default 1.0) and ``routing`` [B*T, layers, top_k]
(routing replay, forced).
"""
from __future__ import annotations

import argparse
import json
import os
import threading
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..parallel.shard_optim import average_gradients
from .lora import DEFAULT_TARGETS, PROJ_MODULE, attach_lora, export_merged, load_lora_state, lora_state
from .losses import bpo_loss, mis_loss, selective_logprob
from .optim import AdamWBF16, clip_grad_norm_
from .routing_replay import RoutingReplay


class FullWeights:
    """The full-weight trainable set of a student: {package key: fp32 master} of the LoRA targets of layers
    >= ``freeze_first_layers`` and of their shared expert (gate / up halves of the fused ``shared_w13`` and
    ``shared_down``), the base weights hashed at install (what the merged manifest compares against), and the
    trainable parameters in model order."""

    def __init__(self, student, targets=DEFAULT_TARGETS, shared: bool = True, freeze_first_layers: int = 0):
        n = len(student.layers)
        if not 0 <= freeze_first_layers < n:
            raise ValueError(f"--freeze-first-layers {freeze_first_layers} of {n} layers")
        for p in student.parameters():
            p.requires_grad_(False)
        self.params, self.slots = [], []  # slots: (key, parameter, row slice or None)
        for i, layer in enumerate(student.layers):
            if i < freeze_first_layers:
                continue
            for name in targets:
                w = getattr(layer, name, None)
                if w is None:
                    continue
                self._train(w)
                self.slots.append((f"model.layers.{i}.{PROJ_MODULE[name]}.{name}.weight", w, None))
            moe = getattr(layer, "moe", None)
            if shared and moe is not None and getattr(moe, "shared_w13", None) is not None:
                Is = moe.shared_w13.shape[0] // 2
                self._train(moe.shared_w13)
                self._train(moe.shared_down)
                p = f"model.layers.{i}.mlp.shared_expert"
                self.slots += [(f"{p}.gate_proj.weight", moe.shared_w13, slice(0, Is)),
                               (f"{p}.up_proj.weight", moe.shared_w13, slice(Is, 2 * Is)),
                               (f"{p}.down_proj.weight", moe.shared_down, None)]
        self.freeze_first_layers = freeze_first_layers
        self.base = self.weights()

    def _train(self, w):
        if w.dtype != torch.float32:
            raise RuntimeError("full-weight training needs fp32 master weights")
        w.requires_grad_(True)
        self.params.append(w)

    def weights(self) -> dict[str, torch.Tensor]:
        """{package key: fp32 CPU copy of the master}."""
        return {k: (p.detach() if sl is None else p.detach()[sl]).float().cpu().clone() for k, p, sl in self.slots}

    def load(self, state: dict[str, torch.Tensor]):
        with torch.no_grad():
            for k, p, sl in self.slots:
                (p if sl is None else p[sl]).copy_(state[k].to(p.device))


#: manifest fields a re-export must reproduce (the rest are timings and provenance)
RESUME_EXPORT_FIELDS = ("format", "weight_version", "base_model", "tensors", "bytes", "trainer", "trained_keys")


def export_differences(published: dict, again: dict) -> list[str]:
    """What differs between a published merged manifest and a re-export of the same version: the
    RESUME_EXPORT_FIELDS and every key's entry. [] = the same bytes."""
    diff = [f"{f}: {published.get(f)!r} != {again.get(f)!r}" for f in RESUME_EXPORT_FIELDS
            if published.get(f) != again.get(f)]
    a, b = published.get("keys", {}), again.get("keys", {})
    if set(a) != set(b):
        diff.append(f"keys: {sorted(set(a) ^ set(b))[:3]} on one side only")
    changed = sorted(k for k in set(a) & set(b) if a[k] != b[k])
    if changed:
        diff.append(f"{len(changed)} tensors differ, e.g. {changed[0]}")
    return diff


class RLTrainer:
    def __init__(self, student, out_dir, lr: float = 2e-5, r: int = 16, alpha: float = 32.0, max_norm: float = 1.0,
                 group=None, trainable: str = "lora", freeze_first_layers: int = 0):
        self.student = student
        self.out = Path(out_dir)
        self.trainable = trainable
        if trainable == "lora":
            self.full = None
            self.params = attach_lora(student, r, alpha)
            self.opt = AdamWBF16([{"params": self.params, "lr": lr}])
        elif trainable == "full":
            self.full = FullWeights(student, freeze_first_layers=freeze_first_layers)
            self.params = self.full.params
            self.opt = torch.optim.AdamW(self.params, lr=lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0)
        else:
            raise ValueError(f"--trainable {trainable!r}: lora | full")
        self.max_norm = max_norm
        self.group = group
        self.step = 0
        self.weight_version = 0
        self.replay = None
        self.busy = False

    def _batch(self, cmd):
        if "batch_path" in cmd:
            return torch.load(cmd["batch_path"], map_location="cpu", weights_only=False)
        return {k: torch.tensor(v) if isinstance(v, list) else v for k, v in cmd["batch"].items()}

    def begin(self, cmd: dict | None = None) -> dict:
        self.opt.zero_grad(set_to_none=True)
        self.acc = {"tokens": 0, "loss_sum": 0.0, "batches": 0, "ratio_sum": 0.0, "ent_sum": 0.0, "t0": time.perf_counter()}
        return {"step": self.step, "begun": True}

    def accumulate(self, cmd: dict) -> dict:
        """Forward + backward of one micro-batch; the loss enters as a token sum (divided by the step's tokens at
        ``step``), so a step over several calls equals one call over their concatenation."""
        if getattr(self, "acc", None) is None:
            raise RuntimeError("accumulate before begin")
        b = self._batch(cmd)
        dev = self.student.embed.device
        ids, labels = b["ids"].long().to(dev), b["labels"].long().to(dev)
        mask = b["mask"].float().to(dev).reshape(-1)
        adv = b["advantages"].float().to(dev)
        if adv.dim() == 1:
            adv = adv[:, None].expand_as(ids)
        adv = adv.reshape(-1)
        T = float(b.get("temperature", 1.0))
        if "routing" in b:
            if self.replay is None:
                c = self.student.cfg
                self.replay = RoutingReplay("force", len(self.student.layers), c.num_experts_per_tok)
                self.replay.install(self.student)
            self.replay.set_routing(b["routing"].long())
        h = self.student.hidden(ids).reshape(ids.numel(), -1)
        logp, ent = selective_logprob(h, self.student.lm_head, labels.reshape(-1), T)
        # the sampler's log-probabilities; without them the batch is treated as on-policy (ratio 1)
        beh = (b["behavior_logp"].float().to(dev).reshape(-1) if b.get("behavior_logp") is not None
               else logp.detach())
        algo = cmd.get("algo", "bpo")
        if algo == "bpo":
            loss = bpo_loss(logp, beh, adv, mask, clip=tuple(cmd.get("clip", (0.2, 0.28))))
        elif algo == "mis":
            loss = mis_loss(logp, beh, adv, mask, cap=float(cmd.get("cap", 2.0)))
        else:
            raise ValueError(f"unknown RL loss {algo!r}")
        m = mask > 0
        n = int(m.sum())
        (loss * n).backward()
        with torch.no_grad():
            ratio = torch.exp(logp.detach() - beh)
            self.acc["tokens"] += n
            self.acc["loss_sum"] += float(loss.detach()) * n
            self.acc["ratio_sum"] += float(ratio[m].sum()) if n else 0.0
            self.acc["ent_sum"] += float(ent.detach()[m].sum()) if n else 0.0
            self.acc["batches"] += 1
        return {"step": self.step, "batches": self.acc["batches"], "tokens": self.acc["tokens"],
                "loss": float(loss.detach())}

    def step_opt(self, cmd: dict | None = None) -> dict:
        acc = getattr(self, "acc", None)
        if acc is None or acc["batches"] == 0:
            raise RuntimeError("step without accumulated batches")
        tokens = max(1, acc["tokens"])
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            average_gradients(self.params, self.group)
        with torch.no_grad():
            for p in self.params:
                if p.grad is not None:
                    p.grad.div_(tokens)
        norm = clip_grad_norm_(self.params, self.max_norm)
        self.opt.step()
        self.step += 1
        report = {"step": self.step, "loss": acc["loss_sum"] / tokens, "grad_norm": float(norm), "tokens": acc["tokens"],
                  "batches": acc["batches"], "ratio_mean": acc["ratio_sum"] / tokens if acc["tokens"] else None,
                  "entropy": acc["ent_sum"] / tokens if acc["tokens"] else None,
                  "seconds": round(time.perf_counter() - acc["t0"], 4)}
        if self.replay is not None:
            st = self.replay.stats
            report["routing_equal_frac"] = sum(st["equal"]) / max(1, sum(st["rows"]))
        self.acc = None
        return report

    def train(self, cmd: dict) -> dict:
        """One optimizer step on one batch (begin + accumulate + step)."""
        self.begin()
        self.accumulate(cmd)
        return self.step_opt()

    def publish(self, cmd: dict) -> dict:
        v = int(cmd["weight_version"])
        if v <= self.weight_version:
            raise ValueError(f"weight_version {v} must exceed the last published {self.weight_version}")
        path = self._export(self.out / "merged" / f"v{v:06d}", v)
        self.weight_version = v
        return {"path": str(path), "weight_version": v}

    def _export(self, path, v: int):
        if self.full is None:
            return export_merged(self.student, path, v, {"optimizer_step": self.step})
        return export_merged(self.student, path, v, {"optimizer_step": self.step}, weights=self.full.weights(),
                             base=self.full.base)

    def save(self, cmd: dict) -> dict:
        target = self.out / f"checkpoint-{self.step}"
        tmp = target.with_name(target.name + ".tmp")
        tmp.mkdir(parents=True, exist_ok=False)
        weights = {"lora": lora_state(self.student)} if self.full is None else {"full": self.full.weights(),
                                                                                "base": self.full.base}
        torch.save({**weights, "trainable": self.trainable, "opt": self.opt.state_dict(), "step": self.step,
                    "weight_version": self.weight_version}, tmp / "trainer_state.pt")
        os.replace(tmp, target)
        return {"path": str(target)}

    def load(self, path):
        st = torch.load(Path(path) / "trainer_state.pt", map_location="cpu", weights_only=False)
        if st.get("trainable", "lora") != self.trainable:
            raise ValueError(f"checkpoint trains {st.get('trainable', 'lora')!r}, this trainer {self.trainable!r}")
        if self.full is None:
            load_lora_state(self.student, st["lora"])
        else:
            self.full.load(st["full"])
            self.full.base = st["base"]
        self.opt.load_state_dict(st["opt"])
        self.step, self.weight_version = st["step"], st["weight_version"]
        if self.full is not None and self.weight_version > 0:
            self.check_resumed_export()

    def check_resumed_export(self):
        """Resume gate (full mode): the restored masters exported again at the checkpoint's weight version must be the
        published ``merged/v<version>`` byte for byte; raises otherwise."""
        import shutil
        import tempfile
        v = self.weight_version
        published = self.out / "merged" / f"v{v:06d}"
        if not (published / "DONE").is_file():
            raise RuntimeError(f"resume gate: {published} has no DONE, nothing to compare the restored weights with")
        scratch = Path(tempfile.mkdtemp(prefix=f"resume-check-v{v:06d}-"))
        try:
            again = self._export(scratch / published.name, v)
            a = json.loads((published / "merged_manifest.json").read_text())
            b = json.loads((again / "merged_manifest.json").read_text())
            a.pop("optimizer_step", None)
            b.pop("optimizer_step", None)
            diff = export_differences(a, b)
        finally:
            shutil.rmtree(scratch)
        if diff:
            raise RuntimeError(f"resume gate: restored weights differ from {published}: " + "; ".join(diff))

    def execute(self, cmd: dict) -> dict:
        """Run one command on this rank (every rank runs the same commands in the same order)."""
        op = cmd["op"]
        if op == "train":
            return self.train(cmd)
        if op == "begin":
            return self.begin(cmd)
        if op == "accumulate":
            return self.accumulate(cmd)
        if op == "step":
            return self.step_opt(cmd)
        if op == "publish":
            return self.publish(cmd) if not dist.is_initialized() or dist.get_rank() == 0 else {}
        if op == "save":
            return self.save(cmd) if not dist.is_initialized() or dist.get_rank() == 0 else {}
        raise ValueError(f"unknown command {op!r}")


def create_app(trainer: RLTrainer, control_group=None):
    """Rank 0's HTTP front; with ``control_group`` (gloo) every command is broadcast to the other ranks first."""
    from fastapi import FastAPI, HTTPException

    app = FastAPI(title="arc_forge_2026_b200 RL trainer")
    lock = threading.Lock()

    def run(cmd):
        with lock:
            trainer.busy = True
            try:
                if control_group is not None:
                    dist.broadcast_object_list([cmd], src=0, group=control_group)
                return trainer.execute(cmd)
            except Exception as e:  # noqa: BLE001
                raise HTTPException(500, f"{type(e).__name__}: {e}") from e
            finally:
                trainer.busy = False

    @app.get("/health")
    def health():
        return {"ok": True, "step": trainer.step, "weight_version": trainer.weight_version, "busy": trainer.busy}

    @app.post("/train")
    def train(body: dict):
        return run({"op": "train", **body})

    @app.post("/begin")
    def begin(body: dict | None = None):
        return run({"op": "begin"})

    @app.post("/accumulate")
    def accumulate(body: dict):
        return run({"op": "accumulate", **body})

    @app.post("/step")
    def step(body: dict | None = None):
        return run({"op": "step"})

    @app.post("/publish")
    def publish(body: dict):
        return run({"op": "publish", **body})

    @app.post("/save")
    def save(body: dict | None = None):
        return run({"op": "save"})

    return app


def follower_loop(trainer: RLTrainer, control_group):
    """Ranks > 0: execute the commands rank 0 broadcasts until a stop command."""
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=0, group=control_group)
        cmd = box[0]
        if cmd is None or cmd.get("op") == "stop":
            return
        trainer.execute(cmd)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="tiny_cpu")
    ap.add_argument("--out", type=Path, required=True)
    ap.add_argument("--lr", type=float, default=2e-5)
    ap.add_argument("--lora-rank", dest="lora_rank", type=int, default=16)
    ap.add_argument("--lora-alpha", dest="lora_alpha", type=float, default=32.0)
    ap.add_argument("--port", type=int, default=8100)
    ap.add_argument("--resume", type=Path)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--trainable", choices=["lora", "full"], default="lora",
                    help="lora: adapters on the projections; full: the projections (+ shared experts) themselves")
    ap.add_argument("--freeze-first-layers", dest="freeze_first_layers", type=int, default=0,
                    help="full: decoder layers 0..F-1 stay frozen")
    args = ap.parse_args(argv)
    from ..config import preset
    from .student import random_student
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))) if torch.cuda.is_available() else "cpu"
    control = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=600))
        control = dist.new_group(backend="gloo")
    student = random_student(preset(args.preset), dev, seed=args.seed)
    trainer = RLTrainer(student, args.out, args.lr, args.lora_rank, args.lora_alpha, trainable=args.trainable,
                        freeze_first_layers=args.freeze_first_layers)
    if args.resume:
        trainer.load(args.resume)
    if rank != 0:
        follower_loop(trainer, control)
        return
    import uvicorn
    args.out.mkdir(parents=True, exist_ok=True)
    (args.out / "trainer_endpoint.json").write_text(json.dumps({"host": "127.0.0.1", "port": args.port}) + "\n")
    uvicorn.run(create_app(trainer, control), host="127.0.0.1", port=args.port, log_level="info")
    if control is not None:
        dist.broadcast_object_list([{"op": "stop"}], src=0, group=control)


if __name__ == "__main__":
    main()
