"""Loader of the native extension ``arc_forge_2026_b200/_C.so``.

On a machine with a CUDA device the extension is mandatory: a missing or stale build raises at import
instead of silently falling back to PyTorch. Without a device (CPU-only hosts) the ops package still imports
and the oracle paths run; calling a native op then raises.
"""
from __future__ import annotations

import importlib

import torch

_C = None
_ERR: Exception | None = None


def _load():
    global _C, _ERR
    if _C is not None or _ERR is not None:
        return _C
    try:
        _C = importlib.import_module("arc_forge_2026_b200._C")
    except ImportError as e:  # pragma: no cover - depends on the build
        _ERR = e
        if torch.cuda.is_available():
            raise ImportError(
                "arc_forge_2026_b200._C is not built; run `python -m arc_forge_2026_b200.build` "
                f"(a CUDA device is present, so there is no fallback): {e}") from e
    return _C


def C():
    mod = _load()
    if mod is None:
        raise RuntimeError(f"native extension unavailable: {_ERR}")
    return mod


def available() -> bool:
    return _load() is not None


def check_status(device: int | None = None, clear: bool = True) -> int:
    """Read (and clear) the device status word that bounded waits / bounds checks write. Raises on error bits."""
    dev = torch.cuda.current_device() if device is None else device
    st = C().status_tensor(dev)
    word = int(st[0].item())
    if clear and word:
        st.zero_()
    if word:
        names = {1: "mbarrier wait timed out", 2: "peer wait timed out", 4: "index out of bounds", 8: "TMEM",
                 16: "cross-rank mismatch"}
        raise RuntimeError("kernel status: " + ", ".join(v for k, v in names.items() if word & k))
    return word
