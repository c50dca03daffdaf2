"""A CPU engine over the fp32 reference model with the serving engine's interface (``add_session``, ``extend_session``,
``step``, ``release``, ``sessions``). It serves the tiny CPU configuration and lets the HTTP
server, the scheduler and session handling be tested without a GPU. Decoding is greedy, one token per session per
step, with each session's incremental cache (attention K/V, GDN conv/ssm state) kept between calls. With a vision
tower (``models/vision.py``) a session's prompt may carry images: their merged features replace the image tokens'
embeddings, deepstack features join after the first layers, the prompt rotates by three-row multimodal positions, and
decoding continues at token index + the session's position delta."""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ..models.reference import HybridMoE


@dataclass
class CPUSession:
    sid: int
    prompt: list[int]
    max_new_tokens: int
    cache: list = field(default_factory=list)
    pos: int = 0
    logits: torch.Tensor | None = None
    generated: list[int] = field(default_factory=list)
    done: bool = False
    delta: int = 0  # multimodal RoPE: rotary position = token index + delta after an image prompt


class CPUEngine:
    def __init__(self, model: HybridMoE, max_sessions: int = 8, max_context: int = 4096, vision=None,
                 image_token_id: int = -1):
        self.model = model.eval()
        self.S = max_sessions
        self.max_context = max_context
        self.sessions: dict[int, CPUSession] = {}
        self.vision = vision.eval() if vision is not None else None
        self.image_token_id = image_token_id

    @property
    def free_slots(self) -> int:
        return self.S - len(self.sessions)

    @torch.no_grad()
    def update_weights(self, path) -> dict:
        """Load a state dict of the reference model (``.pt`` or ``.safetensors``) in place."""
        path = str(path)
        if path.endswith(".safetensors"):
            from safetensors.torch import load_file
            sd = load_file(path)
        else:
            sd = torch.load(path, map_location="cpu", weights_only=True)
        self.model.load_state_dict(sd, strict=True)
        return {"tensors": len(sd)}

    @torch.no_grad()
    def _feed(self, s: CPUSession, toks: list[int]):
        ids = torch.tensor([toks], dtype=torch.long)
        s.logits = self.model(ids, s.cache, s.pos + s.delta)[0, -1]
        s.pos += len(toks)

    @torch.no_grad()
    def _feed_images(self, s: CPUSession, toks: list[int], images):
        """Prefill a prompt with images: ``images`` = [(pixels [P, patch_dim], (t, h, w)), ...] in prompt order."""
        from ..models.vision import mrope_positions
        if self.vision is None or self.model.cfg.mrope_section is None:
            raise ValueError("image prompts need a vision tower and a model with mrope_section")
        pixels = torch.cat([torch.as_tensor(p).float() for p, _ in images])
        grid = torch.tensor([list(g) for _, g in images])
        merged, ds = self.vision.forward_reference(pixels, grid)
        ids = torch.tensor([toks], dtype=torch.long)
        pos3 = mrope_positions((ids[0] == self.image_token_id).long(), grid, self.vision.cfg.spatial_merge_size)
        h = self.model.hidden(ids, s.cache, positions=pos3, image_features=merged, deepstack=ds,
                              image_token_id=self.image_token_id)
        s.logits = self.model.lm_head(h)[0, -1]
        s.pos += len(toks)
        s.delta = int(pos3.max()) + 1 - len(toks)

    def _take(self, s: CPUSession):
        tok = int(s.logits.argmax())
        s.generated.append(tok)
        if len(s.generated) >= s.max_new_tokens:
            s.done = True
        return tok

    def add_session(self, sid: int, prompt: list[int], max_new_tokens: int, images=None) -> CPUSession:
        if sid in self.sessions:
            raise ValueError(f"session {sid} exists")
        if not self.free_slots:
            raise RuntimeError("no free session slot")
        if len(prompt) + max_new_tokens > self.max_context:
            raise ValueError("prompt + max_new_tokens exceed max_context")
        s = CPUSession(sid, list(prompt), max_new_tokens, cache=self.model.new_cache())
        self.sessions[sid] = s
        if images:
            self._feed_images(s, s.prompt, images)
        else:
            self._feed(s, s.prompt)
        self._take(s)
        return s

    def extend_session(self, sid: int, tokens: list[int], max_new_tokens: int) -> CPUSession:
        """Continue a finished session with more input (its cache is kept, only the new tokens are prefilled)."""
        s = self.sessions[sid]
        if s.pos + 1 + len(tokens) + max_new_tokens > self.max_context:
            raise ValueError("session would exceed max_context")
        last = s.generated[-1:] if s.generated else []
        s.prompt = s.prompt + s.generated + list(tokens)
        s.generated, s.done, s.max_new_tokens = [], False, max_new_tokens
        self._feed(s, last + list(tokens))
        self._take(s)
        return s

    def step(self) -> dict[int, list[int]]:
        out = {}
        for s in self.sessions.values():
            if s.done:
                continue
            self._feed(s, [s.generated[-1]])
            out[s.sid] = [self._take(s)]
        return out

    def release(self, sid: int):
        self.sessions.pop(sid)
