"""Registry of the trainer's native kernels: which fused paths are enabled, and how often each ran per step (the
reference's trainer fast-kernel registry with ``--fast-kernels`` and ``assert_step_calls``,
``training/work/qwen38fn_lora/trainer_kernels.py:1-47,317,428``).

Every fused training op (``train/fused.py``, ``train/gdn_chunk.py``, ``train/fakequant.py``) asks :func:`use` whether
its native kernel may run and records the outcome with :func:`hit`. After a step the trainer calls
:func:`assert_step_calls` so a silent fallback to the PyTorch path (a missing extension, an unexpected shape) fails
the run instead of slowing it down.

    from arc_forge_2026_b200.train import kernels
    kernels.enable("all")                    # or a comma list, or "none" (the --fast-kernels flag)
    kernels.reset()
    loss.backward()
    kernels.assert_step_calls({"gdn_chunk": 36, "conv_silu": 36}, no_fallback=True)
"""
from __future__ import annotations

import collections
import os
import threading

NAMES = ("gdn_chunk", "conv_silu", "rms_norm", "gated_rms_norm", "swiglu", "moe_combine", "moe_dispatch",
         "int3_weight", "fp8_weight", "topk_tail_kl", "hc", "ple", "lora_grad",
         "grouped_gemm", "attention")

# opt-in kernels: correct and tested, but slower than the path they replace at the QAD shapes (measured), so "all"
# leaves them off; name them explicitly to run them
OPT_IN = {"grouped_gemm"}

_lock = threading.Lock()
_enabled: set[str] = set(NAMES) - OPT_IN
_calls: collections.Counter = collections.Counter()
_fallbacks: collections.Counter = collections.Counter()


def enable(spec: str | list[str] | None) -> set[str]:
    """``"all"`` / ``None``: every native path except the opt-in ones; ``"none"``: PyTorch everywhere; else a comma
    list of NAMES."""
    global _enabled
    if spec is None or spec == "all":
        names = set(NAMES) - OPT_IN
    elif spec == "none" or spec == "":
        names = set()
    else:
        names = {s.strip() for s in (spec.split(",") if isinstance(spec, str) else spec) if s.strip()}
        bad = names - set(NAMES)
        if bad:
            raise ValueError(f"unknown fast kernels {sorted(bad)}; known: {', '.join(NAMES)}")
    with _lock:
        _enabled = names
    return set(names)


def enabled(name: str) -> bool:
    return name in _enabled


def use(name: str) -> bool:
    """Whether the native kernel ``name`` may run (checked before the op picks its path)."""
    return name in _enabled


def hit(name: str, native: bool):
    with _lock:
        (_calls if native else _fallbacks)[name] += 1


def reset():
    with _lock:
        _calls.clear()
        _fallbacks.clear()


def counts() -> dict:
    with _lock:
        return {"native": dict(_calls), "fallback": dict(_fallbacks)}


def assert_step_calls(expected: dict[str, int] | None = None, no_fallback: bool = True):
    """Raise if a native op ran a different number of times than ``expected`` or (``no_fallback``) any enabled op
    took its PyTorch path since the last :func:`reset`."""
    c = counts()
    errors = []
    for name, n in (expected or {}).items():
        if c["native"].get(name, 0) != n:
            errors.append(f"{name}: {c['native'].get(name, 0)} native calls, expected {n}")
    if no_fallback:
        for name, n in c["fallback"].items():
            if name in _enabled:
                errors.append(f"{name}: {n} calls fell back to PyTorch")
    if errors:
        raise RuntimeError("trainer kernel check failed: " + "; ".join(errors))
    return c


if os.environ.get("AFB_FAST_KERNELS") is not None:  # strict: unknown names raise at import
    enable(os.environ["AFB_FAST_KERNELS"])
