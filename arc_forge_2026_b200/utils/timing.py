"""Named timing sections: CUDA events recorded on the current stream (no host sync until ``report``), or wall
clock without a GPU -- the role of the reference's ``qad_timing.section`` and per-module forward timers
(``qad_timing.py:1-32``, ``distributed_utils.py:10-42``)."""
from __future__ import annotations

import collections
import time
from contextlib import contextmanager

import torch


class Sections:
    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self.cuda = torch.cuda.is_available()
        self._pending: list[tuple[str, object, object]] = []
        self.totals_ms: dict[str, float] = collections.defaultdict(float)
        self.counts: dict[str, int] = collections.defaultdict(int)

    @contextmanager
    def section(self, name: str):
        if not self.enabled:
            yield
            return
        if self.cuda:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            try:
                yield
            finally:
                b.record()
                self._pending.append((name, a, b))
        else:
            t0 = time.perf_counter()
            try:
                yield
            finally:
                self._pending.append((name, t0, time.perf_counter()))

    def report(self) -> dict[str, dict[str, float]]:
        """Resolve pending sections (one synchronize) and return {name: {ms, calls}} accumulated so far."""
        if self.cuda and self._pending:
            torch.cuda.synchronize()
        for name, a, b in self._pending:
            ms = a.elapsed_time(b) if self.cuda else (b - a) * 1000.0
            self.totals_ms[name] += ms
            self.counts[name] += 1
        self._pending.clear()
        return {k: {"ms": round(v, 3), "calls": self.counts[k]} for k, v in self.totals_ms.items()}
