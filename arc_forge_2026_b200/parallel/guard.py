"""Cross-rank agreement checks of small integer packets (the reference's ``pair_check_i64`` and replication checks,
``agi2/work/qwen38fn_l4/probes/hostcomm/hostcomm.cu:1429-1441``, ``hostcomm.py:496-532``): every rank must hold the
same values (step counters, exchange capacities, accepted lengths of a replicated decision).

:class:`ReplicaGuard` runs the check on the device over peer memory (``csrc/guard.cu``): no host synchronisation; a
difference raises the status bit "cross-rank mismatch", which ``ops.check_status()`` turns into an exception at the
next host check. :func:`host_check` is the same check through the process group (CPU / gloo).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import C
from .ep import MAX_RANKS, _align


class ReplicaGuard:
    def __init__(self, world: int, rank: int, device, n_max: int = 64, group=None):
        if not 1 <= world <= MAX_RANKS:
            raise ValueError(f"1..{MAX_RANKS} ranks")
        self.world, self.rank, self.n_max = world, rank, n_max
        dev = torch.device(device)
        off_slots = 0
        off_flags = _align(2 * MAX_RANKS * n_max * 8)
        total = _align(off_flags + MAX_RANKS * 8)
        ext = C()
        self.heap = ext.SymmHeap(total, rank, world, dev.index if dev.index is not None else 0)
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, self.heap.handle(), group=group)
            self.heap.open(handles)
            torch.cuda.synchronize(dev)
            dist.barrier(group=group)
        self.calls = torch.zeros(1, dtype=torch.int64, device=dev)
        self.mismatches = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ctx = ext.GuardCtx(world, rank, list(self.heap.peers()), off_slots, off_flags, n_max, self.calls,
                                self.mismatches)

    def check(self, packet) -> None:
        """Enqueue the comparison of ``packet`` (int64, at most n_max values) across the ranks."""
        t = torch.as_tensor(packet, dtype=torch.int64, device=self.calls.device).reshape(-1).contiguous()
        if t.numel() > self.n_max:
            raise ValueError(f"packet of {t.numel()} > {self.n_max}")
        self.ctx.check(t)

    def close(self):
        if self.heap is not None:
            torch.cuda.synchronize(self.calls.device)
            self.heap.close()
            self.heap = None


def host_check(values, group=None) -> None:
    """Raise on every rank if any rank's ``values`` differ (through the process group)."""
    vals = [int(v) for v in values]
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    got = [None] * dist.get_world_size(group)
    dist.all_gather_object(got, vals, group=group)
    if any(g != got[0] for g in got):
        raise RuntimeError(f"cross-rank mismatch: {got}")
