"""Failure detection across ranks, on the host: heartbeats through the rendezvous store, a peer check that names
the ranks that went silent, and decisions every rank takes together (a step is rejected on all ranks when any rank
saw a non-finite value -- the reference's ``_assert_on_every_rank``, ``distributed_utils.py:112-160``).

A rank learns that a peer died before its next launch (``Heartbeat.check``) or from a short process-group timeout;
nothing here waits on the GPU, so a lost peer never leaves a kernel spinning (device waits are bounded separately
and report through the kernel status word).
"""
from __future__ import annotations

import threading
import time

import torch
import torch.distributed as dist


class PeerLost(RuntimeError):
    def __init__(self, ranks: list[int], age_s: dict[int, float]):
        super().__init__(f"no heartbeat from rank(s) {ranks} for " +
                         ", ".join(f"{r}: {age_s[r]:.1f} s" for r in ranks))
        self.ranks = ranks


class Heartbeat:
    """Each rank stamps ``hb/<rank>`` in the store every ``period_s``; ``check`` raises ``PeerLost`` for peers whose
    stamp is older than ``timeout_s``. ``stop`` (clean exit) writes a tombstone so peers can tell exit from death."""

    def __init__(self, store, rank: int, world: int, period_s: float = 0.5, timeout_s: float = 5.0, prefix="hb"):
        self.store, self.rank, self.world = store, rank, world
        self.period_s, self.timeout_s, self.prefix = period_s, timeout_s, prefix
        self._stop = threading.Event()
        self._beat()
        self._t = threading.Thread(target=self._run, name="afb-heartbeat", daemon=True)
        self._t.start()

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def _beat(self):
        self.store.set(self._key(self.rank), repr(time.time()))

    def _run(self):
        while not self._stop.wait(self.period_s):
            try:
                self._beat()
            except Exception:  # noqa: BLE001 - the store went away: the job is ending
                return

    def ages(self) -> dict[int, float]:
        now, out = time.time(), {}
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                v = self.store.get(self._key(r)).decode()
            except Exception:  # noqa: BLE001
                out[r] = float("inf")
                continue
            out[r] = float("inf") if v == "exited" else now - float(v)
        return out

    def check(self):
        ages = self.ages()
        lost = sorted(r for r, a in ages.items() if a > self.timeout_s)
        if lost:
            raise PeerLost(lost, ages)

    def stop(self, clean: bool = True):
        self._stop.set()
        self._t.join(timeout=5)
        if clean:
            try:
                self.store.set(self._key(self.rank), "exited")
            except Exception:  # noqa: BLE001
                pass


def all_ranks_ok(ok: bool, group=None) -> bool:
    """True only if every rank passed ``ok`` True (one tiny all-reduce; every rank must call it)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return ok
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([0 if ok else 1], dtype=torch.int32, device=dev)
    dist.all_reduce(t, group=group)
    return int(t.item()) == 0


def finite_or_raise(values: list[torch.Tensor], group=None, what: str = "gradients"):
    """Every rank raises together when any rank holds a non-finite value in ``values``."""
    ok = all(bool(torch.isfinite(v).all()) for v in values)
    if not all_ranks_ok(ok, group):
        raise FloatingPointError(f"non-finite {what} on at least one rank (this rank: {'ok' if ok else 'bad'})")
