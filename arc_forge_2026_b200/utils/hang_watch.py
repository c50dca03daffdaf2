"""Hang evidence: a watchdog that, when a named phase runs longer than its limit, writes every thread's Python
stack, the CUDA allocator state and the device status word to a file (and stderr) -- once per phase entry -- so a
stuck collective or kernel leaves a trace without a debugger (the role of the reference's ``hang_watch.py:1-24``).

    watch = HangWatch("/tmp/hangs", limit_s=120)
    with watch.phase("train_step", step=i):
        ...

The watchdog only observes: it never kills the process or touches the GPU beyond reading counters.
"""
from __future__ import annotations

import os
import sys
import threading
import time
import traceback
from contextlib import contextmanager


class HangWatch:
    def __init__(self, out_dir: str, limit_s: float = 300.0, poll_s: float = 1.0, rank: int | None = None):
        self.out_dir = out_dir
        self.limit_s = limit_s
        self.poll_s = poll_s
        self.rank = int(os.environ.get("RANK", "0")) if rank is None else rank
        self._lock = threading.Lock()
        self._phase = None  # (name, info, t0, dumped)
        self._stop = threading.Event()
        self.dumps: list[str] = []
        self._thread = threading.Thread(target=self._run, name="afb-hang-watch", daemon=True)
        self._thread.start()

    @contextmanager
    def phase(self, name: str, **info):
        with self._lock:
            self._phase = [name, info, time.monotonic(), False]
        try:
            yield
        finally:
            with self._lock:
                self._phase = None

    def close(self):
        self._stop.set()
        self._thread.join(timeout=5)

    def _run(self):
        while not self._stop.wait(self.poll_s):
            with self._lock:
                ph = self._phase
                if ph is None or ph[3] or time.monotonic() - ph[2] < self.limit_s:
                    continue
                ph[3] = True
                name, info, t0 = ph[0], dict(ph[1]), ph[2]
            self._dump(name, info, time.monotonic() - t0)

    def _dump(self, name: str, info: dict, elapsed: float):
        os.makedirs(self.out_dir, exist_ok=True)
        path = os.path.join(self.out_dir, f"hang-rank{self.rank}-{name}-{int(time.time())}.txt")
        lines = [f"phase {name!r} on rank {self.rank} running for {elapsed:.1f} s (limit {self.limit_s} s)",
                 f"info: {info}", ""]
        me = threading.get_ident()
        names = {t.ident: t.name for t in threading.enumerate()}
        for tid, frame in sys._current_frames().items():
            if tid == me:
                continue
            lines.append(f"--- thread {names.get(tid, tid)}")
            lines.extend(s.rstrip() for s in traceback.format_stack(frame))
        lines.append("")
        lines.extend(self._cuda_state())
        text = "\n".join(lines) + "\n"
        with open(path + ".tmp", "w") as f:
            f.write(text)
        os.replace(path + ".tmp", path)
        self.dumps.append(path)
        print(f"[hang-watch] {lines[0]} -> {path}", file=sys.stderr, flush=True)

    @staticmethod
    def _cuda_state() -> list[str]:
        try:
            import torch
            if not torch.cuda.is_available():
                return ["cuda: not available"]
            out = [f"cuda device {torch.cuda.current_device()}: allocated {torch.cuda.memory_allocated() / 2**30:.2f}"
                   f" GiB, reserved {torch.cuda.memory_reserved() / 2**30:.2f} GiB"]
            try:  # the status word of the bounded waits (reading it needs no sync of the stuck stream)
                from ..ops import C
                st = C().status_tensor(torch.cuda.current_device())
                out.append(f"kernel status word: {int(st[0].item())}")
            except Exception as e:  # noqa: BLE001
                out.append(f"kernel status word: unavailable ({e})")
            return out
        except Exception as e:  # noqa: BLE001
            return [f"cuda state unavailable: {e}"]
