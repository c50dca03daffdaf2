"""Quantisation-aware distillation (QAD) of the INT3 student against teacher top-k targets.

Modes (the reference's ``training/work/qwen38fn_qad/train_qad.py:1-21``):

* ``teacher`` -- run the teacher over the data and write ``qad-topk-v1`` targets (top-k ids, log-probs, tail) for
  every supervised position;
* ``train``   -- student forward (INT3 scale STE, FP8 QAT, fp32 router), fused LM-head + top-k tail KL (forward or
  reverse), backward with per-layer recompute, global-norm clipping, bf16-state AdamW with one learning rate per
  parameter group, and the scale invariants (a zero scale stays zero; no scale changes sign);
* ``score``   -- the loss of the current student without updates.

Distributed: one process per GPU (torchrun). Every rank trains on its own sequences; the trainable masters live in
a ZeRO-style sharded optimizer (``parallel/shard_optim.py``): gradients are reduce-scattered, each rank updates its
shard, masters are all-gathered. Checkpoints hold the trainable masters and optimizer state per rank plus a
``trainer.json`` with the step and the plan hash (DCP storage: ``train/checkpoint.py``, resumable at another world
size); resume refuses a different plan. ``--export`` writes the trained
tensors as a ``gean320-qad-v2-delta``.

    python -m arc_forge_2026_b200.train.qad --mode train --preset qwen3next_80b --synthetic --steps 10
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..config import QADConfig, preset
from ..formats.topk_targets import TopKReader, TopKWriter, synthetic_targets
from ..parallel.shard_optim import ShardedAdamW
from .kl import teacher_topk
from .losses import fused_topk_tail_kl
from .optim import AdamWBF16, clip_grad_norm_
from .student import QADStudent, random_student


def lr_for(group: str, qc: QADConfig) -> float:
    return {"scale": qc.lr_scale, "router": qc.lr_router}.get(group, qc.lr_dense)


def build_optimizer(student: QADStudent, qc: QADConfig, sharded: bool = False, group=None, fused: bool | None = None):
    """``sharded``: ZeRO-style over the ranks of ``group``; ``fused`` (default: on CUDA with several ranks) runs its
    reduce-scatter, clip, update and all-gather in the peer-memory kernels of ``parallel/zero.py`` instead of NCCL."""
    groups = student.param_groups()
    spec = [{"params": groups[g], "lr": lr_for(g, qc), "name": g} for g in groups if groups[g]]
    if sharded:
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        on_gpu = spec[0]["params"][0].is_cuda
        if fused is None:
            fused = on_gpu and world > 1
        if fused:
            from ..parallel.zero import FusedShardedAdamW
            return FusedShardedAdamW(spec, betas=qc.betas, weight_decay=qc.weight_decay, group=group)
        return ShardedAdamW(spec, betas=qc.betas, weight_decay=qc.weight_decay, group=group)
    return AdamWBF16(spec, betas=qc.betas, weight_decay=qc.weight_decay)


def _scales(student: QADStudent):
    return [p for L in student.layers for p in (L.moe.w13_scales, L.moe.w2_scales)]


@torch.no_grad()
def enforce_scale_invariants(student: QADStudent, signs: list[torch.Tensor] | None):
    """Zero scales stay zero and no scale crosses zero (a group's sign belongs to its INT3 codes)."""
    if signs is None:
        return [torch.sign(p).to(torch.int8) for p in _scales(student)]
    for p, s in zip(_scales(student), signs):
        sf = s.float()
        p.copy_(torch.where(sf == 0, torch.zeros_like(p), torch.where(torch.sign(p) != sf, sf * 1e-12, p)))
    return signs


def mask_zero_scale_grads(student: QADStudent, signs):
    for p, s in zip(_scales(student), signs):
        if p.grad is not None:
            p.grad.masked_fill_(s == 0, 0.0)


def train_step(student: QADStudent, opt, ids: torch.Tensor, targets: dict, qc: QADConfig, signs,
               accumulate: bool = False, sync: bool = True, micro_batches: int = 1, first: bool | None = None):
    """One micro-batch over ``ids`` [B, T] (every position supervised) and, unless ``accumulate``, the optimizer step.

    Gradient accumulation: call with ``accumulate=True`` for all but the last of ``micro_batches`` micro-batches
    (gradients are zeroed at the first one, ``first`` defaults to "the optimizer has no pending gradients"); the
    loss is divided by ``micro_batches`` so the step sees the mean over the whole global batch.
    Returns (mean loss, grad norm) as floats when ``sync``, else the loss as a device tensor (no host sync)."""
    sharded = getattr(opt, "sharded", False)
    if first is None:
        first = not getattr(opt, "_afb_pending", False)
    if first:
        opt.zero_grad(set_to_none=not sharded)
    opt._afb_pending = True
    n = ids.numel()
    h = student.hidden(ids).reshape(n, -1)
    loss = fused_topk_tail_kl(h, student.lm_head, student.lm_head_t, targets["ids"], targets["lp"], targets["tail"],
                              qc.direction) / n
    (loss / micro_batches).backward()
    norm = None
    if not accumulate:
        mask_zero_scale_grads(student, signs)
        if sharded and not sync and getattr(opt, "async_step", False):
            opt.step(qc.grad_clip, sync=False)
        elif sharded:
            norm = opt.step(qc.grad_clip)
        else:
            norm = clip_grad_norm_([p for g in opt.param_groups for p in g["params"]], qc.grad_clip)
            opt.step()
        enforce_scale_invariants(student, signs)
        opt._afb_pending = False
    if not sync:
        return loss.detach()
    return float(loss.detach()), norm


def plan_hash(args) -> str:
    keys = ("preset", "seq_len", "batch", "steps", "topk", "direction", "seed", "layers")
    return hashlib.sha256(json.dumps({k: getattr(args, k) for k in keys}, sort_keys=True).encode()).hexdigest()[:16]


def _start_profile(dev):
    from torch.profiler import ProfilerActivity, profile
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if dev.type == "cuda" else [])
    prof = profile(activities=acts, record_shapes=True)
    prof.__enter__()
    return prof


def _finish_profile(prof, out: Path, step: int, rank: int):
    """Stop the profiler and write, for this rank, the op table sorted by device time (self and total), the same
    grouped by input shape, and a Chrome trace. Profiled steps run slower: their tok/s is not a result."""
    prof.__exit__(None, None, None)
    out.mkdir(parents=True, exist_ok=True)
    base = out / f"profile_step{step}_rank{rank}"
    ka = prof.key_averages()
    dev_key = "self_device_time_total" if torch.cuda.is_available() else "self_cpu_time_total"
    tot_key = "device_time_total" if torch.cuda.is_available() else "cpu_time_total"
    with open(f"{base}.txt", "w") as f:
        f.write(ka.table(sort_by=dev_key, row_limit=60) + "\n")
        f.write(ka.table(sort_by=tot_key, row_limit=60) + "\n")
        f.write(prof.key_averages(group_by_input_shape=True).table(sort_by=dev_key, row_limit=60) + "\n")
    prof.export_chrome_trace(f"{base}.trace.json")


def save_checkpoint(path: Path, student: QADStudent, opt, step: int, phash: str, rank: int):
    """DCP checkpoint (``train/checkpoint.py``): masters once, optimizer moments by owned range, loadable at another
    world size."""
    from .checkpoint import save_dcp
    save_dcp(path, student, opt, step, phash)


def load_checkpoint(path: Path, student: QADStudent, opt, phash: str, rank: int) -> int:
    from .checkpoint import is_dcp, load_dcp
    if is_dcp(path):
        return load_dcp(path, student, opt, phash)
    # per-rank torch.save files of earlier checkpoints (same world size only)
    meta = json.loads((Path(path) / "trainer.json").read_text())
    if meta["plan"] != phash:
        raise RuntimeError(f"checkpoint plan {meta['plan']} != this run's plan {phash}: refusing to resume")
    st = torch.load(Path(path) / f"rank{rank:03d}.pt", map_location="cpu", weights_only=False)
    with torch.no_grad():
        for n, p in student.named_parameters():
            p.copy_(st["params"][n])
    opt.load_state_dict(st["opt"])
    return int(meta["step"])


def export(student: QADStudent, out: Path, meta: dict):
    from ..formats.qad_delta import delta_tensors, export_delta
    named = dict(student.named_parameters())
    fp8 = {n for n in named if n.rsplit(".", 1)[-1] in ("q_proj", "k_proj", "v_proj", "in_proj_qkvz", "out_proj")}
    scales = {n: n.replace("moe.w13_scales", "mlp.experts.w13_scales").replace("moe.w2_scales", "mlp.experts.w2_scales")
              for n in named if n.endswith("_scales")}
    return export_delta(delta_tensors(named, fp8, scales), out, meta)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["train", "teacher", "score"], default="train")
    ap.add_argument("--preset", default="qwen3next_80b")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (0 = preset)")
    ap.add_argument("--seq-len", dest="seq_len", type=int, default=16384)
    ap.add_argument("--batch", type=int, default=1, help="sequences per rank per step")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--topk", type=int, default=64)
    ap.add_argument("--direction", default="reverse", choices=["forward", "reverse"])
    ap.add_argument("--synthetic", action="store_true", help="random tokens and random valid teacher targets")
    ap.add_argument("--targets", type=Path, help="qad-topk-v1 root (train/score)")
    ap.add_argument("--out", type=Path, help="teacher: targets root; train: checkpoint directory")
    ap.add_argument("--resume", action="store_true")
    ap.add_argument("--save-every", dest="save_every", type=int, default=0,
                    help="train: write a checkpoint every N steps (0: only after the last step)")
    ap.add_argument("--profile-step", dest="profile_step", type=int, default=-1,
                    help="profile this step with torch.profiler: device-time tables by op and by input shape and a "
                         "Chrome trace, written under --out (or the working directory) as profile_step<N>.*")
    ap.add_argument("--fast-kernels", dest="fast_kernels", default="all",
                    help="native training kernels to use: all, none, or a comma list (train/kernels.py NAMES); on a "
                         "GPU the first step then fails if an enabled kernel fell back to PyTorch")
    ap.add_argument("--export", type=Path)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--teacher-preset", dest="teacher_preset", default="",
                    help="teacher mode on a GPU: run this (block-FP8) preset on the serving kernels, e.g. "
                         "qwen3next_80b_teacher; empty: score with the student itself")
    args = ap.parse_args(argv)
    from . import kernels
    kernels.enable(args.fast_kernels)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        dist.init_process_group("nccl" if dev.type == "cuda" else "gloo", timeout=datetime.timedelta(seconds=600))
    kw = {"num_layers": args.layers} if args.layers else {}
    cfg = preset(args.preset, **kw)
    qc = QADConfig(seq_len=args.seq_len, topk=args.topk, direction=args.direction)
    student = random_student(cfg, dev, seed=args.seed)
    gen = torch.Generator().manual_seed(args.seed * 7919 + rank)

    def batch(step):
        ids = torch.randint(0, cfg.vocab_size, (args.batch, args.seq_len), generator=gen).to(dev)
        n = ids.numel()
        if args.synthetic or args.targets is None:
            t = synthetic_targets(n, args.topk, cfg.vocab_size, gen, dev)
        else:
            r = TopKReader(args.targets, "train")
            start = ((step * world + rank) * n) % max(1, r.rows - n)
            t = r.rows_slice(start, start + n, dev)
        return ids, t

    if args.mode == "teacher":
        if args.out is None:
            raise SystemExit("--out is required in teacher mode")
        w = TopKWriter(args.out, "train", args.topk)
        native = None
        if dev.type == "cuda" and args.teacher_preset:  # the block-FP8 teacher on the serving kernels
            from ..models.hybrid import HybridModel
            from .teacher import NativeTeacher
            tkw = {"num_layers": args.layers} if args.layers else {}
            native = NativeTeacher(HybridModel.random(preset(args.teacher_preset, **tkw), dev, seed=args.seed + 101),
                                   args.seq_len)
        with torch.no_grad():
            for step in range(args.steps):
                ids, _ = batch(step)
                if native is not None:
                    for row in ids:
                        t_ids, t_lp, t_tail = native.targets(row, args.topk)
                        w.append(t_ids, t_lp, t_tail, row)
                    continue
                h = student.hidden(ids).reshape(ids.numel(), -1)
                z = (h @ student.lm_head.t()).float()
                t_ids, t_lp, t_tail = teacher_topk(z, args.topk)
                w.append(t_ids, t_lp, t_tail, ids.reshape(-1))
        w.close({"source": "trainer-prefill", "teacher": args.teacher_preset if native is not None else args.preset})
        return

    opt = build_optimizer(student, qc, sharded=True, group=dist.group.WORLD if world > 1 else None)
    signs = enforce_scale_invariants(student, None)
    phash = plan_hash(args)
    start = 0
    if args.resume and args.out and (args.out / "trainer.json").exists():
        start = load_checkpoint(args.out, student, opt, phash, rank)
    for step in range(start, args.steps):
        ids, t = batch(step)
        prof = _start_profile(dev) if step == args.profile_step else None
        t0 = time.perf_counter()
        if args.mode == "score":
            with torch.no_grad():
                h = student.hidden(ids).reshape(ids.numel(), -1)
                loss = float(fused_topk_tail_kl(h, student.lm_head, student.lm_head_t, t["ids"], t["lp"], t["tail"],
                                                qc.direction) / ids.numel())
            norm = 0.0
        else:
            kernels.reset()
            loss, norm = train_step(student, opt, ids, t, qc, signs)
            if step == start and dev.type == "cuda":
                kernels.assert_step_calls(no_fallback=True)  # an enabled native kernel must not fall back
        if dev.type == "cuda":
            torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if prof is not None:
            _finish_profile(prof, args.out or Path("."), step, rank)
        if rank == 0:
            print(json.dumps({"step": step, "loss": round(loss, 6), "grad_norm": round(norm, 4),
                              "tok_s": round(ids.numel() * world / dt, 1),
                              "peak_gib": round(torch.cuda.max_memory_allocated() / 2**30, 2)
                              if dev.type == "cuda" else None}), flush=True)
        last = step == args.steps - 1
        if args.out and args.mode == "train" and (last or (args.save_every > 0 and (step + 1) % args.save_every == 0)):
            save_checkpoint(args.out, student, opt, step + 1, phash, rank)
    if args.export and rank == 0:
        export(student, args.export, {"preset": args.preset, "plan": phash})
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
