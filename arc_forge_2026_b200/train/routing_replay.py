"""Routing replay (R3): every MoE layer takes the experts the rollout chose for each token, with gate weights from
the current router softmax at those experts, renormalised like the model's own top-k -- so the router logits stay
differentiable (the reference's ``training/work/qwen38fn_lora/routing_replay.py:1-40``). A recorded row of -1
takes the natural top-k. ``observe`` routes naturally and only counts agreement.

    rep = RoutingReplay("force", layers=48, top_k=10)
    rep.install(student)
    rep.set_routing(recorded)            # int64 [tokens, layers, top_k] for the next forward
"""
from __future__ import annotations

import torch


class RoutingReplay:
    def __init__(self, mode: str, layers: int, top_k: int):
        if mode not in ("observe", "force"):
            raise ValueError(f"routing replay mode {mode!r}")
        self.mode, self.layers, self.top_k = mode, layers, top_k
        self.routing = None
        self.stats = {"rows": [0] * layers, "equal": [0] * layers, "overlap": [0] * layers}

    def install(self, student):
        if len(student.layers) != self.layers:
            raise RuntimeError(f"{len(student.layers)} layers, routing has {self.layers}")
        for i, layer in enumerate(student.layers):
            layer.moe.replay = (self, i)

    def set_routing(self, recorded: torch.Tensor):
        if recorded.dim() != 3 or recorded.shape[1] != self.layers or recorded.shape[2] != self.top_k:
            raise ValueError(f"routing must be [tokens, {self.layers}, {self.top_k}], got {tuple(recorded.shape)}")
        self.routing = recorded

    def route(self, layer: int, logits: torch.Tensor, top_k: int, renorm: bool):
        probs = torch.softmax(logits.float(), dim=-1)
        nat_w, nat_ids = torch.topk(probs, top_k, dim=-1)
        if self.routing is None:
            raise RuntimeError("routing replay installed but no routing set for this forward")
        rec = self.routing[:, layer].to(logits.device)
        if rec.shape[0] != logits.shape[0]:
            raise ValueError(f"routing rows {rec.shape[0]} != tokens {logits.shape[0]}")
        valid = rec[:, 0] >= 0
        with torch.no_grad():  # agreement counters (recorded vs natural sets)
            a = torch.sort(nat_ids[valid], -1).values
            b = torch.sort(rec[valid], -1).values
            self.stats["rows"][layer] += int(valid.sum())
            self.stats["equal"][layer] += int((a == b).all(-1).sum())
            self.stats["overlap"][layer] += int((nat_ids[valid][:, :, None] == rec[valid][:, None, :]).any(-1).sum())
        if self.mode == "observe":
            w, ids = nat_w, nat_ids
        else:
            ids = torch.where(valid[:, None], rec, nat_ids)
            w = probs.gather(1, ids)
        if renorm:
            w = w / w.sum(-1, keepdim=True)
        return w, ids
