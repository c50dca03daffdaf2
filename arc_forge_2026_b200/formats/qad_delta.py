"""``gean320-qad-v2-delta``: the trained tensors of a QAD run in the deployed package's format, and materialisation
of a servable package from delta + source.

Delta directory (``training/work/qwen38fn_qad/train_qad.py:247-302``)::

    delta-00000.safetensors ...   shards of <= 4 GiB
    delta_manifest.json           {"format", meta..., "files": [{file, keys}], "tensors": {key: {dtype, shape, sha256}}}
    DONE

Trained expert scales go out as the package's ``w13_scales`` / ``w2_scales`` (bf16), the FP8-QAT projections as
e4m3 ``weight`` + fp32 ``weight_scale_inv`` (the 128x128 block quantisation of the bf16 cast, i.e. exactly what the
forward used), everything else as bf16. Publication is atomic: ``<dir>.partial`` -> rename, with DONE inside.
"""
from __future__ import annotations

import hashlib
import json
import shutil
from pathlib import Path

import torch
from safetensors.torch import load_file, save_file

from ..quant.fp8 import quantize_weight_block

FORMAT = "gean320-qad-v2-delta"
SHARD_BYTES = 4 << 30


def _sha_tensor(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def delta_tensors(named: dict[str, torch.Tensor], fp8_names: set[str], scale_names: dict[str, str]):
    """Map trained fp32 masters to package tensors. ``scale_names``: parameter name -> package key."""
    out = {}
    for name, t in named.items():
        t = t.detach().float().cpu()
        if name in scale_names:
            out[scale_names[name]] = t.to(torch.bfloat16)
        elif name in fp8_names:
            q, s = quantize_weight_block(t.to(torch.bfloat16).float())
            base = name[: -len(".weight")] if name.endswith(".weight") else name
            out[base + ".weight"] = q
            out[base + ".weight_scale_inv"] = s
        else:
            out[name] = t.to(torch.bfloat16)
    return out


def export_delta(tensors: dict[str, torch.Tensor], out_dir: Path, meta: dict | None = None) -> Path:
    target = Path(out_dir)
    partial = target.with_name(target.name + ".partial")
    if target.exists() or partial.exists():
        raise FileExistsError(target)
    partial.mkdir(parents=True)
    files, manifest, shard, size = [], {}, {}, 0

    def flush():
        nonlocal shard, size
        if shard:
            fn = f"delta-{len(files):05d}.safetensors"
            save_file(shard, str(partial / fn))
            files.append({"file": fn, "keys": sorted(shard)})
        shard, size = {}, 0

    for k in sorted(tensors):
        v = tensors[k].contiguous()
        manifest[k] = {"dtype": str(v.dtype), "shape": list(v.shape), "sha256": _sha_tensor(v)}
        shard[k] = v
        size += v.numel() * v.element_size()
        if size >= SHARD_BYTES:
            flush()
    flush()
    (partial / "delta_manifest.json").write_text(json.dumps({"format": FORMAT, **(meta or {}), "files": files,
                                                             "tensors": manifest}, indent=1) + "\n")
    (partial / "DONE").write_text("ok\n")
    partial.rename(target)
    return target


def load_delta(delta_dir: Path, verify: bool = True) -> dict[str, torch.Tensor]:
    d = Path(delta_dir)
    if not (d / "DONE").exists():
        raise FileNotFoundError(f"{d}: delta not published")
    man = json.loads((d / "delta_manifest.json").read_text())
    if man.get("format") != FORMAT:
        raise ValueError(f"{d}: format {man.get('format')!r}")
    out = {}
    for f in man["files"]:
        out.update(load_file(str(d / f["file"])))
    if verify:
        for k, info in man["tensors"].items():
            if _sha_tensor(out[k]) != info["sha256"]:
                raise ValueError(f"{d}: sha256 mismatch for {k}")
    return out


def materialize(source_dir: Path, delta_dir: Path, out_dir: Path) -> Path:
    """Copy a package and overwrite the tensors the delta names (shard by shard), atomically."""
    src, out = Path(source_dir), Path(out_dir)
    partial = out.with_name(out.name + ".partial")
    if out.exists() or partial.exists():
        raise FileExistsError(out)
    delta = load_delta(delta_dir)
    shutil.copytree(src, partial)
    remaining = set(delta)
    for f in sorted(partial.glob("*.safetensors")):
        t = load_file(str(f))
        hit = [k for k in t if k in delta]
        if hit:
            for k in hit:
                if t[k].shape != delta[k].shape or t[k].dtype != delta[k].dtype:
                    raise ValueError(f"{k}: delta {tuple(delta[k].shape)}/{delta[k].dtype} vs package "
                                     f"{tuple(t[k].shape)}/{t[k].dtype}")
                t[k] = delta[k]
                remaining.discard(k)
            save_file(t, str(f))
    if remaining:
        raise KeyError(f"delta tensors not in the package: {sorted(remaining)[:5]}")
    (partial / "DONE").write_text("ok\n")
    partial.rename(out)
    return out
