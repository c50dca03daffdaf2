"""gEAN / REAP expert saliency, keep-masks and expert pruning.

Saliency of expert ``j`` over a token set: ``S_j = sum(g * ||f||) / count`` -- the conditional mean over the
tokens routed to ``j`` of the routing weight times the norm of the expert's output, 0 for an expert no token
chose (``training/work/qwen38fn_eval/reap_mm_select.py:1-30,64-69``). A mask keeps the ``keep`` highest-scoring
experts in every layer (one count for all layers); ``retained_mass`` reports the kept share of the total score.

Pruning (``training/work/qwen38fn_eval/prune_experts.py``) drops the masked experts' weights, renumbers the
survivors in their original order and drops the matching router rows.
"""
from __future__ import annotations

import dataclasses
import json
from pathlib import Path

import torch

from ..models.reference import HybridMoE, SaliencyAccumulator

COUNTS, SUM_GF = 0, 4


def reap_scores(acc: torch.Tensor) -> torch.Tensor:
    """acc [L, 5, E] -> scores [L, E]."""
    counts, gf = acc[:, COUNTS], acc[:, SUM_GF]
    return torch.where(counts > 0, gf / counts.clamp_min(1e-30), torch.zeros_like(gf))


def keep_mask(scores: torch.Tensor, keep: int) -> torch.Tensor:
    """Boolean ``drop`` [L, E] that keeps the ``keep`` best experts of every layer (ties: lower index first)."""
    L, E = scores.shape
    if not 1 <= keep <= E:
        raise ValueError(f"keep {keep} of {E} experts")
    order = torch.sort(scores, dim=1, descending=True, stable=True).indices
    drop = torch.ones(L, E, dtype=torch.bool)
    for layer in range(L):
        drop[layer, order[layer, :keep]] = False
    return drop


def retained_mass(scores: torch.Tensor, drop: torch.Tensor) -> dict[str, float]:
    total = scores.sum(1).clamp_min(1e-30)
    kept = (scores * (~drop)).sum(1) / total
    return {"mean": float(kept.mean()), "min": float(kept.min())}


@torch.no_grad()
def collect_saliency(model: HybridMoE, batches) -> SaliencyAccumulator:
    """Run calibration batches (iterable of id tensors [B, T]) through ``model`` with saliency capture armed."""
    moes = model.moe_layers()
    acc = SaliencyAccumulator(len(moes), model.cfg.num_experts)
    for m in moes:
        m.saliency = acc
    try:
        for ids in batches:
            model(ids)
    finally:
        for m in moes:
            m.saliency = None
    return acc


@torch.no_grad()
def prune_experts(model: HybridMoE, drop: torch.Tensor) -> HybridMoE:
    """In-place prune to the kept experts of each layer; returns the model with ``cfg.num_experts`` updated."""
    keep_counts = (~drop).sum(1)
    if len(set(keep_counts.tolist())) != 1:
        raise ValueError("every layer must keep the same number of experts")
    keep = int(keep_counts[0])
    for layer, moe in enumerate(model.moe_layers()):
        idx = (~drop[layer]).nonzero().flatten()
        moe.w13 = torch.nn.Parameter(moe.w13.data[idx].clone())
        moe.w2 = torch.nn.Parameter(moe.w2.data[idx].clone())
        gate = torch.nn.Linear(moe.gate.in_features, keep, bias=False, dtype=moe.gate.weight.dtype)
        gate.weight.copy_(moe.gate.weight.data[idx])
        moe.gate = gate
    model.cfg = dataclasses.replace(model.cfg, num_experts=keep)
    for layer in model.layers:
        layer.mlp.cfg = model.cfg
        layer.mixer.cfg = model.cfg
    return model


def write_manifest(path: Path, drop: torch.Tensor, scores: torch.Tensor, meta: dict | None = None):
    """``prune_manifest.json``: keep lists per layer (original expert ids, ascending) + retained mass."""
    keep = [(~drop[layer]).nonzero().flatten().tolist() for layer in range(drop.shape[0])]
    doc = {"format": "prune-manifest-v1", "keep": keep, "retained_mass": retained_mass(scores, drop), **(meta or {})}
    path = Path(path)
    tmp = path.with_suffix(".tmp")
    tmp.write_text(json.dumps(doc, indent=1) + "\n")
    tmp.rename(path)
    return doc


@torch.no_grad()
def verify_pruned(pruned: HybridMoE, source: HybridMoE, manifest: dict) -> dict:
    """Byte-identity provenance of a pruned model (the reference's
    ``training/work/qwen38fn_eval/probes/verify_pruned_vs_incumbent.py``): every kept expert's w13 / w2 and router
    row equal the source's at its original id (manifest ``keep`` lists), every other tensor is unchanged. Raises
    on the first difference; returns counts of what was checked."""
    keep = manifest["keep"]
    src_moe, dst_moe = list(source.moe_layers()), list(pruned.moe_layers())
    if len(keep) != len(src_moe) or len(dst_moe) != len(src_moe):
        raise ValueError("manifest layers differ from the models'")
    experts = 0
    for layer, (a, b, ids) in enumerate(zip(src_moe, dst_moe, keep)):
        if b.w13.shape[0] != len(ids) or ids != sorted(ids):
            raise ValueError(f"layer {layer}: {b.w13.shape[0]} experts for {len(ids)} keep ids (ascending)")
        for j, e in enumerate(ids):
            for name in ("w13", "w2"):
                if not torch.equal(getattr(b, name)[j], getattr(a, name)[e]):
                    raise ValueError(f"layer {layer}: pruned expert {j} {name} differs from source expert {e}")
            if not torch.equal(b.gate.weight[j], a.gate.weight[e]):
                raise ValueError(f"layer {layer}: router row {j} differs from source row {e}")
            experts += 1
    moe_keys = (".mlp.w13", ".mlp.w2", ".mlp.gate.weight")
    sd_a, sd_b = source.state_dict(), pruned.state_dict()
    others = [k for k in sd_a if not k.endswith(moe_keys)]
    for k in others:
        if k not in sd_b or not torch.equal(sd_a[k], sd_b[k]):
            raise ValueError(f"{k}: changed by pruning")
    return {"experts": experts, "other_tensors": len(others)}

