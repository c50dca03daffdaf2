"""Data-parallel gradient synchronisation and the ZeRO-style sharded optimizer of QAD training.

* :func:`average_gradients` -- one flat fp32 bucket, averaged with a single all-reduce; every rank rejects a step
  together when any rank has non-finite gradients (the reference's ``sync_gradients`` /
  ``_assert_on_every_rank``, ``training/work/qwen38fn_lora/distributed_utils.py:100-160``).
* :class:`ShardedAdamW` -- one flat fp32 master buffer per parameter group, whose views are the model's parameters
  and gradients; each rank owns ``1/world`` of every group: gradients are reduce-scattered (mean) into the owned
  shard, AdamW with bf16 moments (native kernel) updates the shard, and the new masters are all-gathered back.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


@torch.no_grad()
def average_gradients(params, group=None):
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1).float() for g in grads])
    bad = torch.zeros(1, device=flat.device) if bool(torch.isfinite(flat).all()) else torch.ones(1, device=flat.device)
    dist.all_reduce(bad, group=group)
    if float(bad) > 0:
        raise FloatingPointError("non-finite gradients on at least one rank")
    dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=group)
    o = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[o:o + n].view_as(g))
        o += n


class ShardedAdamW:
    """ZeRO-style AdamW over parameter groups ``[{"params": [...], "lr": x}, ...]`` of fp32 masters."""

    sharded = True

    def __init__(self, groups, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, group=None):
        self.pg = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.betas, self.eps, self.wd = betas, eps, weight_decay
        self.groups = []
        for g in groups:
            params = list(g["params"])
            n = sum(p.numel() for p in params)
            chunk = math.ceil(n / self.world)
            dev = params[0].device
            flat = torch.zeros(chunk * self.world, dtype=torch.float32, device=dev)
            grad = torch.zeros_like(flat)
            o = 0
            for p in params:
                k = p.numel()
                flat[o:o + k].copy_(p.detach().reshape(-1))
                p.data = flat[o:o + k].view_as(p)
                p.grad = grad[o:o + k].view_as(p)  # autograd accumulates into these views
                o += k
            self.groups.append(dict(params=params, lr=g["lr"], flat=flat, grad=grad, chunk=chunk,
                                    m=torch.zeros(chunk, dtype=torch.bfloat16, device=dev),
                                    v=torch.zeros(chunk, dtype=torch.bfloat16, device=dev), step=0))

    @property
    def param_groups(self):
        return [{"params": g["params"], "lr": g["lr"]} for g in self.groups]

    def zero_grad(self, set_to_none: bool = False):
        for g in self.groups:
            g["grad"].zero_()

    @torch.no_grad()
    def step(self, max_norm: float = 0.0) -> float:
        """Reduce-scatter the gradients, clip by the global norm (summed over ranks), update the owned shards and
        all-gather the masters. Returns the global gradient norm."""
        b1, b2 = self.betas
        shards = []
        sq = None
        for g in self.groups:
            c = g["chunk"]
            shard_g = torch.empty(c, dtype=torch.float32, device=g["flat"].device)
            if self.world > 1:
                dist.reduce_scatter_tensor(shard_g, g["grad"], op=dist.ReduceOp.AVG, group=self.pg)
            else:
                shard_g.copy_(g["grad"])
            shards.append(shard_g)
            part = shard_g.pow(2).sum()
            sq = part if sq is None else sq + part
        if self.world > 1:
            dist.all_reduce(sq, group=self.pg)
        norm = float(sq.sqrt())
        if not math.isfinite(norm):
            raise FloatingPointError(f"non-finite gradient norm {norm}")
        scale = max_norm / (norm + 1e-6) if 0 < max_norm < norm else 1.0
        for g, shard_g in zip(self.groups, shards):
            c = g["chunk"]
            if scale != 1.0:
                shard_g.mul_(scale)
            shard_p = g["flat"][self.rank * c:(self.rank + 1) * c]
            g["step"] += 1
            if shard_p.is_cuda:
                from ..ops import C
                C().adamw(shard_p, shard_g, g["m"], g["v"], None, g["lr"], b1, b2, self.eps, self.wd, g["step"])
            else:
                m = b1 * g["m"].float() + (1 - b1) * shard_g
                v = b2 * g["v"].float() + (1 - b2) * shard_g * shard_g
                g["m"].copy_(m)
                g["v"].copy_(v)
                bc1, bc2 = 1 - b1 ** g["step"], 1 - b2 ** g["step"]
                shard_p.sub_(g["lr"] * (self.wd * shard_p + (m / bc1) / ((v / bc2).sqrt() + self.eps)))
            if self.world > 1:
                dist.all_gather_into_tensor(g["flat"], shard_p.clone(), group=self.pg)
        return norm

    def state_dict(self):
        return {"groups": [{"m": g["m"], "v": g["v"], "step": g["step"]} for g in self.groups]}

    def load_state_dict(self, sd):
        for g, s in zip(self.groups, sd["groups"]):
            g["m"].copy_(s["m"])
            g["v"].copy_(s["v"])
            g["step"] = s["step"]
