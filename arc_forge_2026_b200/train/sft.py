"""Supervised fine-tuning of the student with LoRA adapters over packed bins (the reference's
``training/work/qwen38fn_lora/train_tito_mm.py:1-30``: LoRA on the projections, packed <=120k-token bins, dense QAT,
merged export).

    python -m arc_forge_2026_b200.train.sft --data sft.jsonl --preset tiny_gpu --max-len 16384 \\
        --bins-per-step 4 --steps 100 --out run/sft [--offload-checkpoints] [--init qad_ckpt/]

Data: jsonl, one example per line: ``{"ids": [...], "loss_mask": [...]}`` (mask optional, 1 = trained) or
``{"prompt_ids": [...], "completion_ids": [...]}`` (loss on the completion only). An example with images adds
``"images": [{"pixels": "<.npy of the processor's flattened patches [P, 3 * 2 * 16 * 16], merge-block order>",
"grid_thw": [t, h, w]}, ...]``; its ``--image-token-id`` tokens (t h w / 4 per image, in order) take the frozen vision
tower's merged features (``models/vision.py``; ``--vision-weights`` a torch state dict of ``model.visual.*`` names, or
``--vision-random``), its deepstack features are added after the first decoder layers, and its attention rotates by
the three-row multimodal positions (the preset needs ``mrope_section``). Such an example trains as a bin of its own,
as the reference's image rows do (``training/work/qwen38fn_lora/multimodal.py:108-126``). Examples are packed into bins
(``train/packing.py``: best-fit decreasing, 64-aligned, sequences isolated from each other); rank r of a data-
parallel run takes bins r, r + world, ... Each optimizer step runs ``--bins-per-step`` bins per rank; the loss is the
token mean of -log p(label) over the step's trained tokens on all ranks; adapter gradients are averaged over ranks
(replicated LoRA, one fp32 all-reduce), clipped by global norm, AdamW with bf16 moments. ``--offload-checkpoints``
keeps the layer checkpoints in pinned host memory (``train/offload.py``). At the end (and with ``--save-every``)
the adapters and optimizer state are saved, and ``--export`` writes the merged model (``fn-lora-merged-v2``).
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import json
import os
import random
import time
from pathlib import Path

import torch
import torch.distributed as dist


def load_examples(path, media: list | None = None) -> tuple[list[list[int]], list[list[int]]]:
    """(ids, loss masks) of every example; when ``media`` is a list, it receives each example's image list (or None),
    with ``pixels`` paths resolved against the data file's folder."""
    seqs, masks = [], []
    root = Path(path).parent
    for line in Path(path).read_text().splitlines():
        if not line.strip():
            continue
        ex = json.loads(line)
        if ex.get("images") and media is None:
            raise ValueError("an example has images: pass a list for them (and a vision tower to the trainer)")
        if "ids" in ex:
            ids = list(ex["ids"])
            m = list(ex.get("loss_mask", [1] * len(ids)))
        else:
            p, c = list(ex["prompt_ids"]), list(ex["completion_ids"])
            ids, m = p + c, [0] * len(p) + [1] * len(c)
        if len(ids) != len(m):
            raise ValueError("loss_mask length differs from ids")
        if len(ids) >= 2:
            seqs.append(ids)
            masks.append(m)
            if media is not None:
                imgs = ex.get("images") or None
                if imgs:
                    imgs = [{"pixels": root / im["pixels"] if isinstance(im["pixels"], str) else im["pixels"],
                             "grid_thw": [int(x) for x in im["grid_thw"]]} for im in imgs]
                media.append(imgs)
    return seqs, masks


def media_inputs(tower, images, ids: torch.Tensor, image_token_id: int, merge: int):
    """Vision features and three-row positions of one bin holding one multimodal sequence: (merged features [n, H],
    deepstack features, pos3 [3, L]); rows past the sequence (bin padding) continue the count on all three rows."""
    import numpy as np

    from ..models.vision import mrope_positions
    pix, grids = [], []
    for im in images:
        p = im["pixels"]
        pix.append(torch.from_numpy(np.load(p)) if isinstance(p, (str, Path)) else torch.as_tensor(p))
        grids.append(im["grid_thw"])
    dev = ids.device
    with torch.no_grad():
        merged, ds = tower(torch.cat(pix).float().to(dev), torch.tensor(grids))
    types = (ids == image_token_id).long().cpu()  # padding rows are text rows: they continue the count
    return merged, ds, mrope_positions(types, torch.tensor(grids), merge).to(dev)


def step_loss(student, bins, total_tokens: int, temperature: float = 1.0, offload: bool = False, media=None,
              tower=None, image_token_id: int = -1):
    """Backward of sum(-log p) / total_tokens over ``bins``; returns the summed loss (float). ``media[i]``: the image
    list of bin i's one sequence (None for text bins)."""
    from .losses import selective_logprob
    tot = 0.0
    for i, b in enumerate(bins):
        ctx = contextlib.nullcontext()
        if offload and b.ids.is_cuda:
            from .offload import CheckpointOffload
            ctx = CheckpointOffload()
        args, extra = b.forward_args(), {}
        if media is not None and media[i]:
            if tower is None:
                raise ValueError("an image example needs a vision tower")
            merged, ds, args["pos3"] = media_inputs(tower, media[i], b.ids, image_token_id,
                                                    tower.cfg.spatial_merge_size)
            extra = dict(image_features=merged, deepstack=ds, image_token_id=image_token_id)
        with ctx:
            h = student.hidden(b.ids[None], pack=args, **extra).reshape(b.ids.numel(), -1)
            labels = b.labels.clamp_min(0)
            logp, _ = selective_logprob(h, student.lm_head, labels, temperature)
            m = (b.labels >= 0).float()
            loss = -(logp * m).sum() / max(1, total_tokens)
        loss.backward()
        tot += float(loss.detach()) * max(1, total_tokens)
    return tot


def main(argv=None):
    from ..config import preset
    from .lora import attach_lora, export_merged, load_lora_state, lora_state
    from .optim import AdamWBF16, clip_grad_norm_
    from .packing import pack
    from .student import random_student
    ap = argparse.ArgumentParser()
    ap.add_argument("--data", type=Path, required=True)
    ap.add_argument("--preset", default="tiny_gpu")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--max-len", dest="max_len", type=int, default=16384)
    ap.add_argument("--bins-per-step", dest="bins_per_step", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--lr", type=float, default=1e-4)
    ap.add_argument("--lora-r", dest="lora_r", type=int, default=16)
    ap.add_argument("--lora-alpha", dest="lora_alpha", type=float, default=32.0)
    ap.add_argument("--max-norm", dest="max_norm", type=float, default=1.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--offload-checkpoints", dest="offload", action="store_true")
    ap.add_argument("--init", type=Path, default=None, help="DCP checkpoint of the student (e.g. a QAD run)")
    ap.add_argument("--out", type=Path, required=True)
    ap.add_argument("--save-every", dest="save_every", type=int, default=0)
    ap.add_argument("--resume", action="store_true")
    ap.add_argument("--export", action="store_true", help="write the merged model to <out>/merged at the end")
    ap.add_argument("--image-token-id", dest="image_token_id", type=int, default=-1)
    ap.add_argument("--vision-weights", dest="vision_weights", type=Path, default=None,
                    help="torch state dict of the vision tower (model.visual.* names, prefix stripped)")
    ap.add_argument("--vision-random", dest="vision_random", action="store_true",
                    help="a random vision tower of the default shape, out width = the preset's hidden (synthetic)")
    ap.add_argument("--vision-depth", dest="vision_depth", type=int, default=0)
    ap.add_argument("--mrope-section", dest="mrope_section", default=None,
                    help="t,h,w split of the rotary frequencies for image examples (overrides the preset's)")
    args = ap.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(seconds=600))
    over = {"num_layers": args.layers} if args.layers else {}
    if args.mrope_section:
        over["mrope_section"] = tuple(int(x) for x in args.mrope_section.split(","))
    cfg = preset(args.preset, **over)
    student = random_student(cfg, dev, seed=args.seed)
    if args.init is not None:
        from .checkpoint import load_dcp
        from .optim import AdamWBF16 as _Opt
        groups = [{"params": [p for p in student.parameters() if p.requires_grad], "lr": 0.0}]
        load_dcp(args.init, student, _Opt(groups))  # masters only matter here
    params = attach_lora(student, args.lora_r, args.lora_alpha, seed=args.seed)
    opt = AdamWBF16([{"params": params, "lr": args.lr}])
    media_ex: list = []
    seqs, masks = load_examples(args.data, media_ex)
    text = [i for i, m in enumerate(media_ex) if not m]
    bins = pack([seqs[i] for i in text], args.max_len, loss_masks=[masks[i] for i in text]) if text else []
    media = [None] * len(bins)
    tower = None
    if any(media_ex):  # each image example is a bin of its own
        from dataclasses import replace

        from ..models.vision import VisionConfig, VisionTower
        vcfg = replace(VisionConfig(out_hidden_size=cfg.hidden_size),
                       **({"depth": args.vision_depth,
                           "deepstack_visual_indexes": tuple(i for i in (8, 16, 24) if i < args.vision_depth)}
                          if args.vision_depth else {}))
        if args.vision_weights is not None:
            tower = VisionTower(vcfg)
            tower.load_state_dict(torch.load(args.vision_weights, map_location="cpu"), strict=True)
        elif args.vision_random:
            tower = VisionTower.random(vcfg, seed=args.seed)
        else:
            raise SystemExit("image examples need --vision-weights or --vision-random")
        tower = tower.to(dev).eval()
        for i, m in enumerate(media_ex):
            if m:
                bins += pack([seqs[i]], args.max_len, loss_masks=[masks[i]])
                media.append(m)
    rng = random.Random(args.seed)
    order = list(range(len(bins)))
    start = 0
    state_path = args.out / "trainer_state.pt"
    if args.resume and state_path.exists():
        st = torch.load(state_path, map_location="cpu", weights_only=False)
        load_lora_state(student, st["lora"])
        opt.load_state_dict(st["opt"])
        start = st["step"]
    if rank == 0:
        args.out.mkdir(parents=True, exist_ok=True)
        print(json.dumps({"examples": len(seqs), "bins": len(bins), "max_len": args.max_len,
                          "fill": round(sum(len(s) for s in seqs) / (len(bins) * args.max_len), 3)}), flush=True)

    def save(step):
        if rank == 0:
            tmp = args.out / "trainer_state.pt.tmp"
            torch.save({"lora": lora_state(student), "opt": opt.state_dict(), "step": step}, tmp)
            os.replace(tmp, state_path)

    for step in range(start, args.steps):
        rng.seed(args.seed * 1_000_003 + step)
        pick = [order[rng.randrange(len(order))] for _ in range(args.bins_per_step * world)]
        mine = [bins[i].to(dev) for i in pick[rank::world]]
        mine_media = [media[i] for i in pick[rank::world]]
        total = torch.tensor([float(sum(bins[i].tokens for i in pick))], device=dev)  # identical on every rank
        t0 = time.perf_counter()
        opt.zero_grad(set_to_none=True)
        loss_sum = step_loss(student, mine, int(total.item()), offload=args.offload, media=mine_media, tower=tower,
                             image_token_id=args.image_token_id)
        ls = torch.tensor([loss_sum], device=dev, dtype=torch.float64)
        if world > 1:
            from ..parallel.shard_optim import average_gradients
            average_gradients(params)  # the mean of per-rank gradients ...
            for p in params:           # ... times world = the gradient of the global token mean
                if p.grad is not None:
                    p.grad.mul_(world)
            dist.all_reduce(ls)
        norm = clip_grad_norm_(params, args.max_norm)
        opt.step()
        if cuda:
            torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if rank == 0:
            toks = sum(int(bins[i].ids.numel()) for i in pick)
            print(json.dumps({"step": step, "loss": round(float(ls) / max(1.0, float(total)), 6),
                              "grad_norm": round(norm, 4), "trained_tokens": int(total.item()),
                              "tok_s": round(toks / dt, 1)}), flush=True)
        if args.save_every and (step + 1) % args.save_every == 0:
            save(step + 1)
    save(args.steps)
    if args.export and rank == 0:
        export_merged(student, args.out / "merged", 1, {"sft_steps": args.steps})
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
