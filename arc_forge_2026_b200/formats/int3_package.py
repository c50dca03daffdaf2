"""INT3 deploy package: the servable checkpoint of a compressed model (the reference's
``training/work/qwen38fn_eval/build_int3_deploy.py:149-226``, ``export_int3_sidecar.py:1-15``).

Directory::

    config.json                          the model config + ``quantization_config.arc_int3``
                                         {schema_version 1, bits 3, group_size 128, num_experts,
                                          scale_dtype bfloat16, layout humming_uint3_g128_nozp,
                                          w13_rows gate_then_up, dense_fp8_modules, dense_bf16_modules}
    model-0000i-of-0000N.safetensors     shards of <= shard_bytes
    model.safetensors.index.json         {"weight_map": {key: shard}}
    deploy_manifest.json                 files with size + sha256, payload bytes, expert count
    DONE

Keys follow the Hugging Face Qwen3-Next naming: ``model.layers.N.mlp.experts.{w13,w2}_{qweight,scales}`` (the
Humming uint3 pack: 32 codes per 3 int32 words, LSB first, code c means (c - 4) * scale, w13 rows gate then up),
``model.layers.N.mlp.gate.weight`` (router), ``...mlp.shared_expert.{gate,up,down}_proj.weight``,
``...mlp.shared_expert_gate.weight``, ``...self_attn.{q,k,v,o}_proj.weight`` / ``q_norm`` / ``k_norm``,
``...linear_attn.{in_proj_qkvz,in_proj_ba,out_proj}.weight`` / ``conv1d.weight`` / ``A_log`` / ``dt_bias`` /
``norm.weight``, layer norms, ``model.embed_tokens.weight``, ``model.norm.weight``, ``lm_head.weight``. Dense FP8
modules store e4m3 ``weight`` + fp32 ``weight_scale_inv`` [ceil(N/128), ceil(K/128)]. The writer and reader are
this repository's own; the layout is kept so packages interchange.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
from pathlib import Path

import torch

from ..config import FULL, ModelConfig
from ..quant.fp8 import dequant_weight_block, quantize_weight_block
from ..quant.uint3 import pack_uint3, unpack_uint3

DENSE_FP8 = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "linear_attn.in_proj_qkvz",
             "linear_attn.out_proj")


def _file_sha(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def package_tensors(ref, codes_scales, dense_fp8: bool = True) -> dict[str, torch.Tensor]:
    """Keys of the package from the fp32 oracle model (``models.reference.HybridMoE``) and its INT3 experts
    ``codes_scales[layer] = (w13_codes, w13_scales, w2_codes, w2_scales)``."""
    out = {}

    def put(key, w, fp8=False):
        w = w.detach().float().cpu()
        if fp8:
            q, s = quantize_weight_block(w.to(torch.bfloat16).float())
            out[key + ".weight"], out[key + ".weight_scale_inv"] = q, s
        else:
            out[key + (".weight" if not key.endswith(("A_log", "dt_bias")) else "")] = w.to(torch.bfloat16)
    out["model.embed_tokens.weight"] = ref.embed_tokens.weight.detach().cpu().to(torch.bfloat16)
    out["model.norm.weight"] = ref.norm.weight.detach().cpu().to(torch.bfloat16)
    out["lm_head.weight"] = ref.lm_head.weight.detach().cpu().to(torch.bfloat16)
    for i, L in enumerate(ref.layers):
        p = f"model.layers.{i}"
        put(f"{p}.input_layernorm", L.input_layernorm.weight)
        put(f"{p}.post_attention_layernorm", L.post_attention_layernorm.weight)
        m = L.mixer
        if L.kind == FULL:
            for n in ("q_proj", "k_proj", "v_proj"):
                put(f"{p}.self_attn.{n}", getattr(m, n).weight, dense_fp8)
            put(f"{p}.self_attn.o_proj", m.o_proj.weight)
            put(f"{p}.self_attn.q_norm", m.q_norm.weight)
            put(f"{p}.self_attn.k_norm", m.k_norm.weight)
        else:
            put(f"{p}.linear_attn.in_proj_qkvz", m.in_proj_qkvz.weight, dense_fp8)
            put(f"{p}.linear_attn.in_proj_ba", m.in_proj_ba.weight)
            put(f"{p}.linear_attn.out_proj", m.out_proj.weight, dense_fp8)
            out[f"{p}.linear_attn.conv1d.weight"] = m.conv1d.detach().float().cpu()
            out[f"{p}.linear_attn.A_log"] = m.A_log.detach().float().cpu()
            out[f"{p}.linear_attn.dt_bias"] = m.dt_bias.detach().float().cpu()
            out[f"{p}.linear_attn.norm.weight"] = m.norm.detach().cpu().to(torch.bfloat16)
        moe = L.mlp
        put(f"{p}.mlp.gate", moe.gate.weight)
        put(f"{p}.mlp.shared_expert.gate_proj", moe.shared_gate_proj.weight)
        put(f"{p}.mlp.shared_expert.up_proj", moe.shared_up_proj.weight)
        put(f"{p}.mlp.shared_expert.down_proj", moe.shared_down_proj.weight)
        put(f"{p}.mlp.shared_expert_gate", moe.shared_expert_gate.weight)
        c13, s13, c2, s2 = codes_scales[i]
        out[f"{p}.mlp.experts.w13_qweight"] = pack_uint3(c13)
        out[f"{p}.mlp.experts.w13_scales"] = s13.to(torch.bfloat16).contiguous()
        out[f"{p}.mlp.experts.w2_qweight"] = pack_uint3(c2)
        out[f"{p}.mlp.experts.w2_scales"] = s2.to(torch.bfloat16).contiguous()
        if getattr(L, "hc", False):
            for n in ("hc_attn", "hc_mlp"):
                _put_hc(out, f"{p}.{n}", getattr(L, n))
        if getattr(L, "ple", None) is not None:  # n-gram table in block FP8; projections bf16; norms, conv fp32
            ple = L.ple
            q, s = quantize_weight_block(ple.table.detach().float().cpu())
            out[f"{p}.ple.table.weight"], out[f"{p}.ple.table.weight_scale_inv"] = q, s
            for n in ("key_proj", "value_proj"):
                out[f"{p}.ple.{n}"] = getattr(ple, n).detach().cpu().to(torch.bfloat16).contiguous()
            for n in ("norm_key", "norm_query", "norm_conv", "conv"):
                out[f"{p}.ple.{n}"] = getattr(ple, n).detach().float().cpu().contiguous()
    if getattr(ref, "hc_final", None) is not None:
        _put_hc(out, "model.hc_final", ref.hc_final)
    return out


def _put_hc(out: dict, prefix: str, mod):
    """Hyper-connection weights: the norm weight in fp32, the projections in bf16 (never FP8: the gate and the mix
    feed every branch of the residual stream)."""
    out[f"{prefix}.hc_norm.weight"] = mod.hc_norm.weight.detach().float().cpu()
    for n in ("w_down", "w_up", "w_inject"):
        w = getattr(mod, n, None)
        if w is not None:
            out[f"{prefix}.{n}"] = w.detach().cpu().to(torch.bfloat16).contiguous()


def write_package(tensors: dict[str, torch.Tensor], cfg: ModelConfig, out_dir, shard_bytes: int = 5 << 30,
                  dense_fp8: bool = True, meta: dict | None = None) -> Path:
    from safetensors.torch import save_file
    target = Path(out_dir)
    partial = target.with_name(target.name + ".partial")
    if target.exists() or partial.exists():
        raise FileExistsError(target)
    partial.mkdir(parents=True)
    shards, cur, size = [], {}, 0
    for k in sorted(tensors):
        t = tensors[k].contiguous()
        n = t.numel() * t.element_size()
        if cur and size + n > shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = t
        size += n
    if cur:
        shards.append(cur)
    weight_map, files = {}, []
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, str(partial / name))
        weight_map.update({k: name for k in sh})
        files.append(name)
    (partial / "model.safetensors.index.json").write_text(
        json.dumps({"metadata": {"total_size": sum(t.numel() * t.element_size() for t in tensors.values())},
                    "weight_map": weight_map}, indent=1, sort_keys=True) + "\n")
    config = dataclasses.asdict(cfg)
    config["quantization_config"] = {"arc_int3": {
        "schema_version": 1, "bits": 3, "group_size": 128, "num_experts": cfg.num_experts,
        "scale_dtype": "bfloat16", "layout": "humming_uint3_g128_nozp", "w13_rows": "gate_then_up",
        "dense_fp8_modules": list(DENSE_FP8) if dense_fp8 else [],
        "dense_bf16_modules": ["self_attn.o_proj", "linear_attn.in_proj_ba"]}}
    (partial / "config.json").write_text(json.dumps(config, indent=1, sort_keys=True) + "\n")
    manifest = {"format": "arc-int3-deploy-v1", "num_experts": cfg.num_experts,
                "payload_bytes": sum(t.numel() * t.element_size() for t in tensors.values()),
                "files": {f: {"bytes": (partial / f).stat().st_size, "sha256": _file_sha(partial / f)}
                          for f in files + ["config.json", "model.safetensors.index.json"]}, **(meta or {})}
    # the reference's byte form (json indent 2 + newline): RL overlays rebuild this file and hash it
    (partial / "deploy_manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    (partial / "DONE").write_text("")
    os.replace(partial, target)
    return target


def read_package(pkg_dir, verify: bool = True, weight_patch=None,
                 merged=None) -> tuple[ModelConfig, dict[str, torch.Tensor]]:
    """(config, tensors) of a package. ``weight_patch``: a ``arcforge.kaggle.weight_patch.v1`` directory made against
    this package, whose tensors replace the package's; ``merged``: a ``fn-lora-merged-v2`` directory whose tensors
    replace the package's under the same names (what a server's update from disk loads)."""
    from safetensors.torch import load_file
    d = Path(pkg_dir)
    if not (d / "DONE").exists():
        raise RuntimeError(f"{d} is not a published package (no DONE)")
    manifest = json.loads((d / "deploy_manifest.json").read_text())
    if verify:
        for f, ent in manifest["files"].items():
            if _file_sha(d / f) != ent["sha256"]:
                raise RuntimeError(f"{f}: sha256 mismatch")
    config = json.loads((d / "config.json").read_text())
    q = config.pop("quantization_config")["arc_int3"]
    if q["layout"] != "humming_uint3_g128_nozp" or q["bits"] != 3 or q["group_size"] != 128:
        raise ValueError(f"unsupported expert layout {q}")
    fields = {f.name for f in dataclasses.fields(ModelConfig)}
    cfg = ModelConfig(**{k: v for k, v in config.items() if k in fields})
    index = json.loads((d / "model.safetensors.index.json").read_text())
    tensors = {}
    for f in sorted(set(index["weight_map"].values())):
        tensors.update(load_file(str(d / f)))
    if weight_patch is not None:
        from .weight_patch import WeightPatch
        tensors = WeightPatch(weight_patch, _file_sha(d / "deploy_manifest.json")).apply(tensors)
    if merged is not None:
        tensors = apply_merged(tensors, merged)
    return cfg, tensors


def apply_merged(tensors: dict[str, torch.Tensor], merged_dir) -> dict[str, torch.Tensor]:
    """``tensors`` with a published merged version's tensors substituted (same names, dtypes and shapes; every
    merged tensor checked against the manifest's sha256)."""
    from safetensors.torch import load_file
    from .weight_patch import MERGED_FORMAT, tensor_sha
    m = Path(merged_dir)
    if not (m / "DONE").exists():
        raise RuntimeError(f"{m} is not published (no DONE)")
    man = json.loads((m / "merged_manifest.json").read_text())
    if man.get("format") != MERGED_FORMAT:
        raise ValueError(f"{m}: format {man.get('format')!r}")
    new = load_file(str(m / "model.safetensors"))
    out = dict(tensors)
    for k, t in new.items():
        if k not in out:
            raise KeyError(f"{k} of {m} is not in the package")
        if t.dtype != out[k].dtype or t.shape != out[k].shape:
            raise ValueError(f"{k}: merged {t.dtype}{tuple(t.shape)}, package {out[k].dtype}{tuple(out[k].shape)}")
        if tensor_sha(t) != man["keys"][k]["merged_sha256"]:
            raise RuntimeError(f"{k}: bytes differ from {m}/merged_manifest.json")
        out[k] = t
    return out


def dense_weight(tensors: dict[str, torch.Tensor], key: str, dtype=torch.bfloat16) -> torch.Tensor:
    """``key`` (without ``.weight``) as a plain matrix: block-FP8 modules are dequantised, bf16 ones returned."""
    w = tensors[key + ".weight"]
    if w.dtype == torch.float8_e4m3fn:
        return dequant_weight_block(w, tensors[key + ".weight_scale_inv"]).to(dtype)
    return w.to(dtype)


def expert_codes(tensors: dict[str, torch.Tensor], layer: int, cfg: ModelConfig):
    """(w13_codes, w13_scales, w2_codes, w2_scales) of one layer from its uint3 packs."""
    p = f"model.layers.{layer}.mlp.experts"
    H, I = cfg.hidden_size, cfg.moe_intermediate_size
    return (unpack_uint3(tensors[f"{p}.w13_qweight"], H), tensors[f"{p}.w13_scales"],
            unpack_uint3(tensors[f"{p}.w2_qweight"], I), tensors[f"{p}.w2_scales"])
