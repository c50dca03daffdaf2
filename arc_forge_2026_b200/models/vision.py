"""Vision tower of the multimodal model: a Qwen3-VL-style ViT (the reference's "FN" checkpoint carries one under
``model.visual.*``: 27 blocks, hidden 1152, 16 heads of 72, patch 16 x 16 over 2 frames, 2 x 2 spatial merge into the
2560-wide text hidden, deepstack features after blocks 8, 16 and 24). The reference loads that tower bit for bit from
the checkpoint and runs it frozen (``training/work/qwen38fn_lora/multimodal.py:46-70``), resamples the learned 48 x 48
position table exactly as its deployed server does (``training/work/qwen38fn_lora/vision_interp.py:20-46``) and
places image features with multimodal RoPE positions (``multimodal.py:108-126`` through ``get_rope_index``).

Here:

* :class:`VisionTower` holds the weights under the checkpoint's names (``patch_embed.proj``, ``pos_embed``,
  ``blocks.{i}.{norm1,attn.qkv,attn.proj,norm2,mlp.linear_fc1,mlp.linear_fc2}``, ``merger``,
  ``deepstack_merger_list.{j}``), so a checkpoint's ``model.visual.*`` tensors load with ``load_state_dict``;
* :meth:`VisionTower.forward_reference` is an fp32 PyTorch statement of the tower (the oracle of the tests);
* :meth:`VisionTower.forward` is the B200 path: every projection on the tcgen05 GEMM with its bias, GELU and residual
  add in the epilogue (one bf16 rounding per projection), attention on the tcgen05 training-attention
  forward in its bidirectional mode with the 72-wide heads zero-padded to 128 (the output projection's weight is
  padded to match once), and the elementwise work in ``csrc/vision.cu``;
* :func:`vit_interp` is the deployed position-table resampling (align-corners bilinear taps, weights rounded to the
  table's dtype, bf16 products and running sums), :func:`vision_rope_angles` the 2-D rotary angles and
  :func:`mrope_positions` the text model's three-row positions around image runs and
  :func:`mrope_angles` the interleaved multimodal rotary angles they give;
* :func:`merge_image_features` writes the merged image features over the image-token rows of a text embedding.

The tower is frozen everywhere in the reference, so only the forward is provided (no vision LoRA).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class VisionConfig:
    depth: int = 27
    hidden_size: int = 1152
    num_heads: int = 16
    intermediate_size: int = 4304
    in_channels: int = 3
    patch_size: int = 16
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    out_hidden_size: int = 2560
    num_position_embeddings: int = 2304
    deepstack_visual_indexes: tuple[int, ...] = (8, 16, 24)
    rope_theta: float = 10000.0
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def grid_side(self) -> int:
        return int(round(math.sqrt(self.num_position_embeddings)))

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.temporal_patch_size * self.patch_size ** 2

    @property
    def merged_dim(self) -> int:
        return self.hidden_size * self.spatial_merge_size ** 2


def _grids(grid_thw) -> list[tuple[int, int, int]]:
    rows = grid_thw.tolist() if isinstance(grid_thw, torch.Tensor) else list(grid_thw)
    return [(int(t), int(h), int(w)) for t, h, w in rows]


def merge_order(h: int, w: int, merge: int, device=None) -> torch.Tensor:
    """Row-major patch index of each position in merge-block order (the order the processor emits patches in: the
    merge x merge patches of one merged token are consecutive)."""
    idx = torch.arange(h * w, device=device).view(h // merge, merge, w // merge, merge)
    return idx.permute(0, 2, 1, 3).reshape(-1)


def vit_interp(grid_thw, side: int, merge: int, dtype=torch.bfloat16, device=None):
    """Four-tap bilinear resampling of the ``side x side`` position table to each image's ``h x w`` patch grid:
    (indices [P, 4] int64, weights [P, 4] in ``dtype``) for the patches of every image in order (P = sum t h w,
    merge-block order, the h x w pattern repeated for each of the t frames).

    Geometry: sample points ``linspace(0, side - 1, n)`` along each axis (corners aligned), taps at the floor and at
    floor + 1 clamped to the table; weights ``(1 - dh)(1 - dw), (1 - dh) dw, dh (1 - dw), dh dw`` formed in fp32 and
    then rounded to ``dtype`` -- the table dtype of the deployed server, which then multiplies and sums the four taps
    in that dtype."""
    all_i, all_w = [], []
    for t, h, w in _grids(grid_thw):
        if h % merge or w % merge:
            raise ValueError(f"grid {(t, h, w)} is not a multiple of the spatial merge {merge}")
        ys = torch.linspace(0, side - 1, h, dtype=torch.float32, device=device)
        xs = torch.linspace(0, side - 1, w, dtype=torch.float32, device=device)
        y0, x0 = ys.long(), xs.long()
        y1, x1 = (y0 + 1).clamp(max=side - 1), (x0 + 1).clamp(max=side - 1)
        fy, fx = (ys - y0)[:, None], (xs - x0)[None, :]
        wts = torch.stack([(1 - fy) * (1 - fx), (1 - fy) * fx, fy * (1 - fx), fy * fx], -1).reshape(-1, 4)
        idx = torch.stack([y0[:, None] * side + x0[None, :], y0[:, None] * side + x1[None, :],
                           y1[:, None] * side + x0[None, :], y1[:, None] * side + x1[None, :]], -1).reshape(-1, 4)
        order = merge_order(h, w, merge, device)
        all_i.append(idx[order].repeat(t, 1))
        all_w.append(wts[order].to(dtype).repeat(t, 1))
    return torch.cat(all_i), torch.cat(all_w)


def vision_rope_angles(grid_thw, head_dim: int, merge: int, theta: float = 10000.0, device=None) -> torch.Tensor:
    """2-D rotary angles [P, head_dim / 2] (fp32): the first head_dim / 4 entries rotate with the patch's row, the rest
    with its column, both over the frequencies ``theta^(-2j / (head_dim / 2))``; a head's dims j and j + head_dim / 2
    form a rotation pair."""
    nf = head_dim // 4
    inv = 1.0 / (theta ** (torch.arange(0, 2 * nf, 2, dtype=torch.float32, device=device) / (head_dim // 2)))
    out = []
    for t, h, w in _grids(grid_thw):
        order = merge_order(h, w, merge, device)
        rows, cols = (order // w).float(), (order % w).float()
        ang = torch.cat([rows[:, None] * inv[None, :], cols[:, None] * inv[None, :]], -1)
        out.append(ang.repeat(t, 1))
    return torch.cat(out)


def mrope_positions(token_types: torch.Tensor, image_grid_thw, merge: int) -> torch.Tensor:
    """Three-row (temporal, height, width) positions [3, T] of one sequence for multimodal RoPE. ``token_types``
    [T]: 0 text, 1 image. Text tokens advance all three rows together; a run of image tokens (one image: t h w /
    merge^2 tokens) sits at the current position in the temporal row and at current + (merged row / column) in the
    other two (with t > 1 frames the row index advances every t * w / merge tokens, as the reference's position rule
    has it; images have t = 1), and the next token continues at current + max(h, w) / merge."""
    types = token_types.tolist()
    grids = iter(_grids(image_grid_thw) if image_grid_thw is not None else [])
    pos = torch.zeros(3, len(types), dtype=torch.long)
    cur, i = 0, 0
    while i < len(types):
        j = i
        while j < len(types) and types[j] == types[i]:
            j += 1
        if types[i] == 0:
            pos[:, i:j] = torch.arange(cur, cur + j - i)
            cur += j - i
            i = j
            continue
        t, h, w = next(grids)
        gh, gw = h // merge, w // merge
        n = t * gh * gw
        if j - i < n:
            raise ValueError(f"image run of {j - i} tokens, grid {(t, h, w)} needs {n}")
        k = torch.arange(n)
        pos[0, i:i + n] = cur
        pos[1, i:i + n] = cur + k // (gw * t)
        pos[2, i:i + n] = cur + k % gw
        cur += max(h, w) // merge
        i += n
    return pos


def mrope_angles(pos3: torch.Tensor, rot: int, theta: float, sections: tuple[int, int, int]) -> torch.Tensor:
    """Rotary angles [T, rot / 2] (fp32) of the text attention from three-row positions [3, T], interleaved:
    frequency f takes its position from the height row when f = 1 (mod 3) and f < 3 sections[1], from the width row
    when f = 2 (mod 3) and f < 3 sections[2], else from the temporal row. For text tokens the three rows are equal,
    so this is ordinary RoPE at that position (decode after an image continues at token index + a per-sequence
    delta)."""
    nf = rot // 2
    if sum(sections) != nf:
        raise ValueError(f"sections {sections} do not cover {nf} frequencies")
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float32, device=pos3.device) / rot))
    f = torch.arange(nf, device=pos3.device)
    row = torch.zeros(nf, dtype=torch.long, device=pos3.device)
    row[(f % 3 == 1) & (f < 3 * sections[1])] = 1
    row[(f % 3 == 2) & (f < 3 * sections[2])] = 2
    return pos3.float()[row].t() * inv[None, :]


def merge_image_features(embeds: torch.Tensor, ids: torch.Tensor, image_token_id: int,
                         features: torch.Tensor) -> torch.Tensor:
    """Text embeddings [T, H] with the rows of ``image_token_id`` replaced, in order, by the tower's merged features
    [n_image_tokens, H] (a new tensor)."""
    mask = ids == image_token_id
    if int(mask.sum()) != features.shape[0]:
        raise ValueError(f"{int(mask.sum())} image tokens for {features.shape[0]} image features")
    out = embeds.clone()
    out[mask] = features.to(out.dtype)
    return out


class _Merger(nn.Module):
    def __init__(self, cfg: VisionConfig, postshuffle: bool):
        super().__init__()
        self.postshuffle = postshuffle
        self.norm = nn.LayerNorm(cfg.merged_dim if postshuffle else cfg.hidden_size, eps=cfg.eps)
        self.linear_fc1 = nn.Linear(cfg.merged_dim, cfg.merged_dim)
        self.linear_fc2 = nn.Linear(cfg.merged_dim, cfg.out_hidden_size)


class _Attn(nn.Module):
    def __init__(self, cfg: VisionConfig):
        super().__init__()
        self.qkv = nn.Linear(cfg.hidden_size, 3 * cfg.hidden_size)
        self.proj = nn.Linear(cfg.hidden_size, cfg.hidden_size)


class _Mlp(nn.Module):
    def __init__(self, cfg: VisionConfig):
        super().__init__()
        self.linear_fc1 = nn.Linear(cfg.hidden_size, cfg.intermediate_size)
        self.linear_fc2 = nn.Linear(cfg.intermediate_size, cfg.hidden_size)


class _Block(nn.Module):
    def __init__(self, cfg: VisionConfig):
        super().__init__()
        self.norm1 = nn.LayerNorm(cfg.hidden_size, eps=cfg.eps)
        self.norm2 = nn.LayerNorm(cfg.hidden_size, eps=cfg.eps)
        self.attn = _Attn(cfg)
        self.mlp = _Mlp(cfg)


class _PatchEmbed(nn.Module):
    def __init__(self, cfg: VisionConfig):
        super().__init__()
        k = (cfg.temporal_patch_size, cfg.patch_size, cfg.patch_size)
        self.proj = nn.Conv3d(cfg.in_channels, cfg.hidden_size, kernel_size=k, stride=k, bias=True)


class VisionTower(nn.Module):
    """The ViT under the checkpoint's parameter names; inputs are the processor's flattened patches
    ``pixels [P, in_channels * temporal_patch * patch^2]`` (merge-block order) and ``grid_thw [images, 3]``; outputs
    (merged features [P / merge^2, out_hidden], deepstack features: one such tensor per deepstack block)."""

    def __init__(self, cfg: VisionConfig = VisionConfig()):
        super().__init__()
        self.cfg = cfg
        self.patch_embed = _PatchEmbed(cfg)
        self.pos_embed = nn.Embedding(cfg.num_position_embeddings, cfg.hidden_size)
        self.blocks = nn.ModuleList(_Block(cfg) for _ in range(cfg.depth))
        self.merger = _Merger(cfg, postshuffle=False)
        self.deepstack_merger_list = nn.ModuleList(_Merger(cfg, postshuffle=True)
                                                   for _ in cfg.deepstack_visual_indexes)
        self._native = None

    @classmethod
    def random(cls, cfg: VisionConfig = VisionConfig(), seed: int = 0, std: float = 0.02) -> "VisionTower":
        g = torch.Generator().manual_seed(seed)
        m = cls(cfg)
        with torch.no_grad():
            for name, p in m.named_parameters():
                if "norm" in name:
                    p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g) if name.endswith("weight")
                            else 0.1 * torch.randn(p.shape, generator=g))
                else:
                    p.copy_(std * torch.randn(p.shape, generator=g))
        return m

    # ------------------------------------------------------------------ fp32 statement (oracle)
    @staticmethod
    def _ln(x, mod):
        return F.layer_norm(x, x.shape[-1:], mod.weight.float(), mod.bias.float(), mod.eps)

    @staticmethod
    def _lin(x, mod):
        return x @ mod.weight.float().t() + mod.bias.float()

    def _merge(self, x, m: _Merger):
        c = self.cfg
        x = self._ln(x.reshape(-1, c.merged_dim), m.norm) if m.postshuffle else \
            self._ln(x, m.norm).reshape(-1, c.merged_dim)
        return self._lin(F.gelu(self._lin(x, m.linear_fc1)), m.linear_fc2)

    @torch.no_grad()
    def forward_reference(self, pixels: torch.Tensor, grid_thw):
        c = self.cfg
        grids = _grids(grid_thw)
        dev = pixels.device
        x = pixels.float() @ self.patch_embed.proj.weight.float().reshape(c.hidden_size, -1).t() \
            + self.patch_embed.proj.bias.float()
        idx, wts = vit_interp(grids, c.grid_side, c.spatial_merge_size, torch.float32, dev)
        table = self.pos_embed.weight.float()
        x = x + (table[idx] * wts[..., None]).sum(1)
        ang = vision_rope_angles(grids, c.head_dim, c.spatial_merge_size, c.rope_theta, dev)
        cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
        seg = [h * w for t, h, w in grids for _ in range(t)]  # attention runs within each frame
        if sum(seg) != x.shape[0]:
            raise ValueError("pixels rows do not match grid_thw")
        H, Dh, half = c.num_heads, c.head_dim, c.head_dim // 2
        ds = []
        for li, blk in enumerate(self.blocks):
            y = self._ln(x, blk.norm1)
            q, k, v = self._lin(y, blk.attn.qkv).view(-1, 3, H, Dh).unbind(1)

            def rot(t):
                a, b = t[..., :half], t[..., half:]
                return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)
            q, k = rot(q), rot(k)
            o = torch.empty_like(q)
            p0 = 0
            for n in seg:  # attention within each frame of each image
                s = torch.einsum("qhd,khd->hqk", q[p0:p0 + n], k[p0:p0 + n]) / math.sqrt(Dh)
                o[p0:p0 + n] = torch.einsum("hqk,khd->qhd", s.softmax(-1), v[p0:p0 + n])
                p0 += n
            x = x + self._lin(o.reshape(-1, H * Dh), blk.attn.proj)
            y = self._ln(x, blk.norm2)
            x = x + self._lin(F.gelu(self._lin(y, blk.mlp.linear_fc1), approximate="tanh"), blk.mlp.linear_fc2)
            if li in c.deepstack_visual_indexes:
                ds.append(self._merge(x, self.deepstack_merger_list[c.deepstack_visual_indexes.index(li)]))
        return self._merge(x, self.merger), ds

    # ------------------------------------------------------------------ B200 path
    def refresh_native(self):
        """(Re)build the bf16 device copies the native forward reads; call after changing the weights."""
        c = self.cfg
        H, Dh, Dp = c.num_heads, c.head_dim, 128
        if Dh > Dp:
            raise ValueError(f"head dim {Dh} > {Dp}")
        b16 = lambda t: t.detach().to(torch.bfloat16).contiguous()  # noqa: E731
        blocks = []
        for blk in self.blocks:
            wp = torch.zeros(c.hidden_size, H, Dp, dtype=torch.bfloat16, device=blk.attn.proj.weight.device)
            wp[:, :, :Dh] = blk.attn.proj.weight.detach().view(c.hidden_size, H, Dh).to(torch.bfloat16)
            blocks.append(dict(n1w=b16(blk.norm1.weight), n1b=b16(blk.norm1.bias), n2w=b16(blk.norm2.weight),
                               n2b=b16(blk.norm2.bias), wqkv=b16(blk.attn.qkv.weight), bqkv=b16(blk.attn.qkv.bias),
                               wproj=wp.view(c.hidden_size, H * Dp), bproj=b16(blk.attn.proj.bias),
                               w1=b16(blk.mlp.linear_fc1.weight), b1=b16(blk.mlp.linear_fc1.bias),
                               w2=b16(blk.mlp.linear_fc2.weight), b2=b16(blk.mlp.linear_fc2.bias)))

        def merger(m):
            return dict(nw=b16(m.norm.weight), nb=b16(m.norm.bias), w1=b16(m.linear_fc1.weight),
                        b1=b16(m.linear_fc1.bias), w2=b16(m.linear_fc2.weight), b2=b16(m.linear_fc2.bias),
                        post=m.postshuffle)
        self._native = dict(wpe=b16(self.patch_embed.proj.weight.reshape(c.hidden_size, -1)),
                            bpe=b16(self.patch_embed.proj.bias), table=b16(self.pos_embed.weight), blocks=blocks,
                            merger=merger(self.merger), ds=[merger(m) for m in self.deepstack_merger_list])
        return self

    @torch.no_grad()
    def forward(self, pixels: torch.Tensor, grid_thw):
        from ..ops import C
        from ..train.attention import tile_lists
        c = self.cfg
        if self._native is None:
            self.refresh_native()
        nat, cc = self._native, C()
        grids = _grids(grid_thw)
        dev = pixels.device
        P, Hd, H, Dh, Dp = pixels.shape[0], c.hidden_size, c.num_heads, c.head_dim, 128
        if sum(t * h * w for t, h, w in grids) != P:
            raise ValueError("pixels rows do not match grid_thw")
        b16 = dict(dtype=torch.bfloat16, device=dev)
        # patch embedding (+ bias) + resampled position table
        acc = cc.gemm(pixels.to(torch.bfloat16).contiguous(), nat["wpe"], out_fp32=True)
        idx, wts = vit_interp(grids, c.grid_side, c.spatial_merge_size, torch.bfloat16, dev)
        h = torch.empty(P, Hd, **b16)
        cc.vit_patch_pos(acc, nat["bpe"], nat["table"], idx.to(torch.int32).contiguous(), wts.contiguous(), h)
        del acc
        ang = vision_rope_angles(grids, Dh, c.spatial_merge_size, c.rope_theta, dev)
        cosv, sinv = ang.cos().contiguous(), ang.sin().contiguous()
        seg = [h_ * w_ for t_, h_, w_ in grids for _ in range(t_)]  # attention within each frame
        cu_host = [0]
        for n in seg:
            cu_host.append(cu_host[-1] + n)
        cu = torch.tensor(cu_host, dtype=torch.int32, device=dev)
        fwd_tiles = tile_lists(cu_host, dev)[0]
        q, k, v, o = (torch.empty(P, H, Dp, **b16) for _ in range(4))
        lse = torch.empty(H, P, dtype=torch.float32, device=dev)
        y = torch.empty(P, Hd, **b16)
        qkv = torch.empty(P, 3 * Hd, **b16)
        m = torch.empty(P, c.intermediate_size, **b16)
        scale = 1.0 / math.sqrt(Dh)
        ds = []
        for li, b in enumerate(nat["blocks"]):
            cc.vit_layernorm(h, b["n1w"], b["n1b"], c.eps, y)
            cc.gemm(y, b["wqkv"], out=qkv, bias=b["bqkv"])
            cc.vit_qkv_rope(qkv, cosv, sinv, H, Dh, q, k, v)
            cc.attn_train_fwd(q, k, v, cu, fwd_tiles, scale, o, lse, None, 64, False)
            cc.gemm(o.view(P, H * Dp), b["wproj"], out=h, residual=h, bias=b["bproj"])
            cc.vit_layernorm(h, b["n2w"], b["n2b"], c.eps, y)
            cc.gemm(y, b["w1"], out=m, bias=b["b1"], act=1)
            cc.gemm(m, b["w2"], out=h, residual=h, bias=b["b2"])
            if li in c.deepstack_visual_indexes:
                ds.append(self._merge_native(h, nat["ds"][c.deepstack_visual_indexes.index(li)]))
        return self._merge_native(h, nat["merger"]), ds

    def _merge_native(self, h: torch.Tensor, m: dict) -> torch.Tensor:
        from ..ops import C
        c, cc = self.cfg, C()
        rows = h.shape[0] // c.spatial_merge_size ** 2
        x = h.view(rows, c.merged_dim) if m["post"] else h
        y = torch.empty_like(x)
        cc.vit_layernorm(x, m["nw"], m["nb"], c.eps, y)
        t = cc.gemm(y.view(rows, c.merged_dim), m["w1"], bias=m["b1"], act=2)
        return cc.gemm(t, m["w2"], bias=m["b2"])
