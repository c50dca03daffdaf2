"""LoRA adapters for RL / SFT on the QAD student, and the merged export serving loads.

Adapters sit on the dense projections (attention q/k/v/o, GDN in_proj_qkvz / in_proj_ba / out_proj): the frozen
base output (block-FP8 QAT weight where the deployed model runs FP8) plus ``scale * (x A^T) B^T`` computed in fp32,
``scale = alpha / r`` (the reference's LoRABF16, ``training/work/qwen38fn_lora/trainer_kernels.py:167-213``).

Merged export, ``fn-lora-merged-v2`` (the reference's ``merged_export.py:1-40``)::

    <dir>/model.safetensors      merged adapted projections only, under the model's keys:
                                 FP8-served ones as e4m3 ``<key>`` + fp32 ``<key minus .weight>.weight_scale_inv``
                                 [N/128, K/128], the rest bf16
    <dir>/merged_manifest.json   the reference's fields: format, weight_version, step, optimizer_step, base_model,
                                 lora rank / alpha / scale, tensors, bytes, dense_qat, and ``keys`` {key: shape,
                                 format (fp8_e4m3_block128 / fp32_scale_inv / bf16), scale_key, base / merged
                                 sha256, changed_elements}
    <dir>/DONE                   written last; <dir>.tmp -> <dir> rename before it

Merge: ``(W + scale * B @ A)`` in fp32 from the original base, rounded once (so rounding never compounds across
publishes).
"""
from __future__ import annotations

import hashlib
import json
import math
import os
from pathlib import Path

import torch
from torch import nn

from ..quant.fp8 import quantize_weight_block

FORMAT = "fn-lora-merged-v2"
FP8_PROJ = ("q_proj", "k_proj", "v_proj", "in_proj_qkvz", "out_proj")
# the module each adapted projection sits in, in the package's key names (formats/int3_package.py)
PROJ_MODULE = {"q_proj": "self_attn", "k_proj": "self_attn", "v_proj": "self_attn", "o_proj": "self_attn",
               "in_proj_qkvz": "linear_attn", "in_proj_ba": "linear_attn", "out_proj": "linear_attn"}
DEFAULT_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "in_proj_qkvz", "in_proj_ba", "out_proj")


def _tgrad_splits(T: int, M: int) -> int:
    """T splits of the native tgrad: about 4 CTAs per SM, no split longer than 2,048 rows (long fp32 sums drift)."""
    tiles = max(1, (M + 127) // 128)
    return max(1, min((T + 63) // 64, max(-(-148 * 4 // tiles), -(-T // 2048))))


class _LoRANative(torch.autograd.Function):
    """``scale * (x A^T) B^T`` with the native LoRA kernels (``csrc/lora.cu``): the bf16 activations and output
    gradients are read once in bf16, never copied to fp32; the rank-r expansions (s B^T, ds A) stay fp32 GEMMs."""

    @staticmethod
    def forward(ctx, x, A, B, scale):
        from ..ops import C
        lead = x.shape[:-1]
        xb = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
        s = C().lora_rows_times(xb, A.detach().float().contiguous())            # [T, r]
        ctx.save_for_backward(xb, s, A, B)
        ctx.scale, ctx.lead, ctx.xdtype = scale, lead, x.dtype
        return ((s @ B.float().t()) * scale).view(*lead, B.shape[0])

    @staticmethod
    def backward(ctx, dy):
        from . import kernels
        from ..ops import C
        xb, s, A, B = ctx.saved_tensors
        c = C()
        dyb = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16).contiguous()
        T = dyb.shape[0]
        dB = c.lora_tgrad(dyb, s, _tgrad_splits(T, dyb.shape[1])) * ctx.scale              # [N, r]
        ds = c.lora_rows_times(dyb, B.detach().float().t().contiguous()) * ctx.scale      # [T, r]
        dA = c.lora_tgrad(xb, ds.contiguous(), _tgrad_splits(T, xb.shape[1])).t()         # [r, K]
        dx = (ds @ A.float()).to(ctx.xdtype).view(*ctx.lead, A.shape[1])
        kernels.hit("lora_grad", True)
        return dx, dA, dB, None


class LoRAAdapter(nn.Module):
    def __init__(self, in_features: int, out_features: int, r: int, alpha: float, device, generator=None):
        super().__init__()
        self.r, self.alpha, self.scale = r, alpha, alpha / r
        self.A = nn.Parameter(torch.randn(r, in_features, generator=generator, device=device) / math.sqrt(in_features))
        self.B = nn.Parameter(torch.zeros(out_features, r, device=device))

    def forward(self, x):
        from . import kernels
        if (x.is_cuda and kernels.use("lora_grad") and self.r in (8, 16, 32, 64) and x.shape[-1] % 8 == 0
                and self.B.shape[0] % 8 == 0):
            return _LoRANative.apply(x, self.A, self.B, self.scale)
        if x.is_cuda:
            kernels.hit("lora_grad", False)
        return ((x.float() @ self.A.t()) @ self.B.t()) * self.scale

    def delta(self) -> torch.Tensor:
        return (self.B.float() @ self.A.float()) * self.scale


def attach_lora(student, r: int = 16, alpha: float = 32.0, targets=DEFAULT_TARGETS, seed: int = 0):
    """Freeze every student parameter and attach adapters to the ``targets`` projections of every layer.
    Returns the adapter parameters (the only trainable ones)."""
    for p in student.parameters():
        p.requires_grad_(False)
    g = torch.Generator(device=next(student.parameters()).device).manual_seed(seed)
    params = []
    for layer in student.layers:
        for name in targets:
            w = getattr(layer, name, None)
            if w is None:
                continue
            ad = LoRAAdapter(w.shape[1], w.shape[0], r, alpha, w.device, g)
            layer.lora[name] = ad
            params += [ad.A, ad.B]
    return params


def lora_state(student) -> dict[str, torch.Tensor]:
    return {f"layers.{i}.{n}.{k}": getattr(ad, k).detach().cpu()
            for i, layer in enumerate(student.layers) for n, ad in layer.lora.items() for k in ("A", "B")}


def load_lora_state(student, state: dict[str, torch.Tensor]):
    with torch.no_grad():
        for i, layer in enumerate(student.layers):
            for n, ad in layer.lora.items():
                ad.A.copy_(state[f"layers.{i}.{n}.A"])
                ad.B.copy_(state[f"layers.{i}.{n}.B"])


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _entry(key: str, stored: torch.Tensor, base_stored: torch.Tensor | None, fmt: str) -> dict:
    """One ``keys`` entry of the merged manifest (the v2 fields: shape, format, base / merged sha256, changed
    elements counted in the stored form)."""
    ent = {"shape": list(stored.shape), "format": fmt}
    if fmt == "fp8_e4m3_block128":
        ent["scale_key"] = key[: -len(".weight")] + ".weight_scale_inv"
    if base_stored is not None:
        ent["base_sha256"] = _sha(base_stored)
    ent["merged_sha256"] = _sha(stored)
    if base_stored is None:
        ent["changed_elements"] = int(stored.numel())
    else:
        ent["changed_elements"] = int((stored.contiguous().view(torch.uint8).view(stored.numel(), -1) !=
                                       base_stored.contiguous().view(torch.uint8).view(stored.numel(), -1))
                                      .any(-1).sum())
    return ent


def deployed_form(key: str, w: torch.Tensor, fp8: bool) -> dict[str, torch.Tensor]:
    """The tensors a served model loads for weight ``w`` (fp32 math): block-FP8 e4m3 + fp32 ``weight_scale_inv``
    for the projections the deployed model runs in FP8, bf16 otherwise."""
    if fp8:
        q, sc = quantize_weight_block(w.float())
        return {key: q, key[: -len(".weight")] + ".weight_scale_inv": sc.float()}
    return {key: w.to(torch.bfloat16)}


def merged_tensors(student, key_prefix: str = "model.layers", weights: dict | None = None,
                   base: dict | None = None) -> tuple[dict, dict]:
    """{package key: tensor} of the merged adapted projections and their manifest ``keys`` entries.

    LoRA mode (``weights`` None): each adapted projection is ``W + scale * B @ A`` in fp32 from the frozen base,
    rounded once. Full mode: ``weights`` {key: trained weight} replace the projections directly and ``base``
    {key: original weight} gives the base the manifest hashes against."""
    out, keys = {}, {}

    def put(key, merged, base_w, fp8):
        dep = deployed_form(key, merged, fp8)
        dep_base = deployed_form(key, base_w, fp8) if base_w is not None else {}
        for k, t in dep.items():
            fmt = ("fp8_e4m3_block128" if t.dtype == torch.float8_e4m3fn else
                   "fp32_scale_inv" if k.endswith("weight_scale_inv") else "bf16")
            keys[k] = _entry(k, t, dep_base.get(k) if fmt != "fp32_scale_inv" else None, fmt)
            if fmt == "fp32_scale_inv" and k in dep_base:
                keys[k]["changed_elements"] = int((t != dep_base[k]).sum())
            out[k] = t.contiguous()

    if weights is not None:
        for key, w in sorted(weights.items()):
            name = key.split(".")[-2]
            put(key, w.detach().float().cpu(), None if base is None else base[key].detach().float().cpu(),
                name in FP8_PROJ)
        return out, keys
    for i, layer in enumerate(student.layers):
        for name, ad in layer.lora.items():
            base_w = getattr(layer, name).detach().float().cpu()
            merged = (base_w + ad.delta().detach().float().cpu()).to(torch.bfloat16).float()
            put(f"{key_prefix}.{i}.{PROJ_MODULE[name]}.{name}.weight", merged, base_w.to(torch.bfloat16).float(),
                name in FP8_PROJ)
    return out, keys


def export_merged(student, out_dir, weight_version: int, meta: dict | None = None, weights: dict | None = None,
                  base: dict | None = None, base_model: str | None = None) -> Path:
    """Publish one merged version (``fn-lora-merged-v2``, the reference's manifest fields) at ``out_dir``.
    ``weights`` / ``base``: full-weight trainer (see :func:`merged_tensors`)."""
    from safetensors.torch import load_file, save_file
    target = Path(out_dir)
    tmp = target.with_name(target.name + ".tmp")
    if target.exists() or tmp.exists():
        raise FileExistsError(target)
    tmp.mkdir(parents=True)
    tensors, keys = merged_tensors(student, weights=weights, base=base)
    path = tmp / "model.safetensors"
    save_file(tensors, str(path), metadata={"format": "pt", "fn_lora_merged": FORMAT,
                                            "weight_version": str(weight_version)})
    back = load_file(str(path))  # read back bitwise before publishing
    if set(back) != set(tensors):
        raise RuntimeError("read-back tensor set differs")
    for k, t in tensors.items():
        if not torch.equal(back[k].view(torch.uint8), t.contiguous().view(torch.uint8)):
            raise RuntimeError(f"read-back mismatch for {k}")
    full = weights is not None
    ads = [] if full else [ad for layer in student.layers for ad in layer.lora.values()]
    n_fp8 = sum(1 for e in keys.values() if e["format"] == "fp8_e4m3_block128")
    manifest = {"format": FORMAT, "weight_version": str(weight_version), "step": weight_version,
                "base_model": base_model, "lora_rank": ads[0].r if ads else None,
                "lora_alpha": ads[0].alpha if ads else None, "scale": ads[0].scale if ads else None,
                "tensors": len(tensors), "bytes": path.stat().st_size,
                **({"trainer": "full", "trained_keys": len(weights)} if full else {}), **(meta or {}),
                "dense_qat": {"scheme": "block_fp8_e4m3_128x128", "scale_suffix": "weight_scale_inv",
                              "modules": n_fp8, "forward_checked": None},
                "keys": keys}
    (tmp / "merged_manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    os.replace(tmp, target)
    (target / "DONE").write_text("")
    return target
