"""Delta-only weight patch: the tensors of a trained model that differ from its base, so a server swaps only those
(the reference's ``arcforge.kaggle.weight_patch.v1``, ``training/work/qwen38fn_rl/rl_weight_patch.py:1-26``).

    <dir>/patch.safetensors    changed tensors, base keys and dtypes
    <dir>/patch_manifest.json  format, base / patched sha256 per changed tensor, counts
    <dir>/DONE
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import torch

FORMAT = "arcforge.weight_patch.v1"


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def write_patch(base: dict[str, torch.Tensor], new: dict[str, torch.Tensor], out_dir, meta: dict | None = None) -> Path:
    from safetensors.torch import save_file
    changed = {}
    for k, t in new.items():
        if k not in base:
            raise KeyError(f"{k} is not in the base")
        b = base[k]
        if t.dtype != b.dtype or t.shape != b.shape:
            raise ValueError(f"{k}: {t.dtype}{tuple(t.shape)} vs base {b.dtype}{tuple(b.shape)}")
        if not torch.equal(t.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8)):
            changed[k] = t.contiguous().cpu()
    target = Path(out_dir)
    tmp = target.with_name(target.name + ".tmp")
    tmp.mkdir(parents=True)
    save_file(changed, str(tmp / "patch.safetensors"))
    manifest = {"format": FORMAT, "changed": len(changed), "total": len(new),
                "tensors": {k: {"sha256_base": _sha(base[k].cpu()), "sha256_patched": _sha(v)}
                            for k, v in changed.items()}, **(meta or {})}
    (tmp / "patch_manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    os.replace(tmp, target)
    (target / "DONE").write_text("")
    return target


def apply_patch(base: dict[str, torch.Tensor], patch_dir, verify: bool = True) -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file
    d = Path(patch_dir)
    if not (d / "DONE").exists():
        raise RuntimeError(f"{d} is not published (no DONE)")
    manifest = json.loads((d / "patch_manifest.json").read_text())
    if manifest["format"] != FORMAT:
        raise ValueError(manifest["format"])
    patch = load_file(str(d / "patch.safetensors"))
    out = dict(base)
    for k, t in patch.items():
        if verify:
            ent = manifest["tensors"][k]
            if _sha(base[k].cpu()) != ent["sha256_base"]:
                raise RuntimeError(f"{k}: the base differs from the one the patch was made against")
            if _sha(t) != ent["sha256_patched"]:
                raise RuntimeError(f"{k}: patch bytes corrupted")
        out[k] = t
    return out
