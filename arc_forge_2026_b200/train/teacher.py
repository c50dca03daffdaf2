"""QAD teacher on the serving kernels: the block-FP8 teacher (512 experts, e4m3 weights with 128x128 block scales,
bf16 elsewhere) runs each training sequence as a prefill through the native model, and the
top-k + tail targets of every position come from its LM head chunk by chunk (the reference's QAD ``--mode teacher``,
``training/work/qwen38fn_qad/train_qad.py:1-21``, which writes ``qad-topk-v1`` targets).
"""
from __future__ import annotations

import torch

from ..config import ServeConfig
from ..serve.engine import SpecEngine
from .kl import teacher_topk


class NativeTeacher:
    def __init__(self, model, max_len: int):
        self.model = model
        self.engine = SpecEngine(model, None, ServeConfig(spec_k=0, accept_mode="greedy"), 1, max_len + 64)

    @torch.no_grad()
    def targets(self, ids: torch.Tensor, k: int):
        """ids [T] -> (ids [T, k] int64, log-probs [T, k], tail log-mass [T]) of the teacher at every position."""
        out = []

        def on_chunk(hidden, start):
            z = self.model.logits(hidden, fp32=True)
            out.append(teacher_topk(z.float(), k))
        self.engine.score(ids.tolist(), on_chunk)
        return tuple(torch.cat([o[i] for o in out]) for i in range(3))
