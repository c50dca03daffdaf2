"""ZeRO-style AdamW whose gradient reduce-scatter, scale, global-norm clip, shard update and parameter all-gather run
in native peer-memory kernels (``csrc/zero_comm.cu``) instead of NCCL collectives around a separate update.

Drop-in for :class:`parallel.shard_optim.ShardedAdamW` on GPUs (same constructor and ``step(max_norm)``): every
group's fp32 masters and gradients are one flat buffer inside a symmetric heap (the model's parameters and their
``.grad`` become views of it), so each rank's kernels read the peers' gradients and shards directly over NVLink.
The reduction order is fixed (rank 0 first), so the update is bitwise identical from run to run.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops._ext import C, check_status
from .ep import MAX_RANKS, _align

ZERO_GRADS, ZERO_NORM, ZERO_PARAMS = 0, 1, 2
RS_BLOCKS = 148 * 8  # blocks of the reduce-scatter and update grids: a full SM of 256-thread blocks each


class FusedShardedAdamW:
    sharded = True
    async_step = True  # step(sync=False) issues no host synchronisation

    def __init__(self, groups, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, group=None):
        self.pg = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        self.betas, self.eps, self.wd = betas, eps, weight_decay
        specs = []
        off = 0
        for g in groups:
            params = list(g["params"])
            n = sum(p.numel() for p in params)
            chunk = (math.ceil(n / self.world) + 3) // 4 * 4  # 16-byte vectors in the exchange kernels
            size = chunk * self.world * 4
            specs.append((params, g["lr"], n, chunk, off, off + _align(size)))
            off += 2 * _align(size)
        off_flags = off
        off_norm = _align(off_flags + 3 * MAX_RANKS * 8)
        total = _align(off_norm + MAX_RANKS * 4)
        dev = specs[0][0][0].device
        ext = C()
        self.heap = ext.SymmHeap(total, self.rank, self.world, dev.index or 0)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, self.heap.handle(), group=group)
            self.heap.open(handles)
        buf = self.heap.tensor()
        self.groups = []
        for params, lr, n, chunk, g_off, p_off in specs:
            flat = buf[p_off:p_off + chunk * self.world * 4].view(torch.float32)
            grad = buf[g_off:g_off + chunk * self.world * 4].view(torch.float32)
            o = 0
            with torch.no_grad():
                for p in params:
                    k = p.numel()
                    flat[o:o + k].copy_(p.detach().reshape(-1))
                    p.data = flat[o:o + k].view_as(p)
                    p.grad = grad[o:o + k].view_as(p)
                    o += k
            self.groups.append(dict(params=params, lr=lr, n=n, chunk=chunk, g_off=g_off, p_off=p_off, flat=flat,
                                    grad=grad, shard=torch.zeros(chunk, dtype=torch.float32, device=dev),
                                    m=torch.zeros(chunk, dtype=torch.bfloat16, device=dev),
                                    v=torch.zeros(chunk, dtype=torch.bfloat16, device=dev), step=0))
        self.partials = torch.zeros(len(self.groups), RS_BLOCKS, dtype=torch.float32, device=dev)
        self.sent = torch.zeros(3, dtype=torch.int64, device=dev)
        self.expected = torch.zeros(3, dtype=torch.int64, device=dev)
        self.norm = torch.zeros(1, dtype=torch.float32, device=dev)
        self.ctx = ext.ZeroCtx(self.world, self.rank, list(self.heap.peers()), off_flags, off_norm, self.sent,
                               self.expected, self.norm)
        if self.world > 1:
            torch.cuda.synchronize()
            dist.barrier(group=group)  # every heap zeroed and mapped before the first flag

    @property
    def param_groups(self):
        return [{"params": g["params"], "lr": g["lr"]} for g in self.groups]

    def zero_grad(self, set_to_none: bool = False):
        for g in self.groups:
            g["grad"].zero_()

    @torch.no_grad()
    def step(self, max_norm: float = 0.0, sync: bool = True):
        """One fused update; returns the global gradient norm (a float when ``sync``, else the device scalar).

        A non-finite norm leaves masters and moments unchanged on every rank (the kernels skip the update) and
        raises ``FloatingPointError`` when ``sync``; a peer that does not arrive within the wait limit raises
        ``RuntimeError`` from the device status word."""
        b1, b2 = self.betas
        c = self.ctx
        c.signal(ZERO_GRADS)
        c.wait(ZERO_GRADS)
        for gi, g in enumerate(self.groups):
            c.rs(g["g_off"], g["chunk"], 1.0 / self.world, g["shard"], self.partials[gi])
        c.norm_publish(self.partials.view(-1))
        c.wait(ZERO_NORM)
        for g in self.groups:
            g["step"] += 1
            c.adamw(g["p_off"], g["chunk"], g["shard"], g["m"], g["v"], g["n"], g["lr"], b1, b2, self.eps, self.wd,
                    g["step"], max_norm, RS_BLOCKS)
        c.signal(ZERO_PARAMS)  # the update stored every rank's new shard into every heap
        c.wait(ZERO_PARAMS)
        if not sync:
            return self.norm
        norm = float(self.norm.item())
        check_status()
        if not math.isfinite(norm):
            for g in self.groups:
                g["step"] -= 1
            raise FloatingPointError(f"non-finite gradient norm {norm} (update skipped on every rank)")
        return norm

    def state_dict(self):
        return {"groups": [{"m": g["m"], "v": g["v"], "step": g["step"]} for g in self.groups]}

    def load_state_dict(self, sd):
        for g, s in zip(self.groups, sd["groups"]):
            g["m"].copy_(s["m"])
            g["v"].copy_(s["v"])
            g["step"] = s["step"]

    def close(self):
        if self.heap is not None:
            torch.cuda.synchronize()
            self.heap.close()
            self.heap = None
