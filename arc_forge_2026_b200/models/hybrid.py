"""The hybrid MoE on the native kernels: decode / speculative verify / prefill forward passes.

Weights live in the layouts the kernels want:

* GDN layers: one fused in-projection ``[q|k|v|z|b|a]`` (``in_proj_qkvz`` and ``in_proj_ba`` stacked), conv
  weight fp32 ``[C, 4]``, ``A_log``/``dt_bias`` fp32, output norm weight, ``out_proj``.
* Attention layers: one fused ``[q+gate | k | v]`` projection (``q_proj`` rows keep the per-head
  ``[q_h | gate_h]`` interleave), q/k norm weights, ``o_proj``.
* MoE: router rows + the shared-expert gate row (``router_ext``), routed experts as an INT3 tile bank, the shared
  expert as ``[gate; up]`` and ``down``.

The residual stream is bf16 and is updated in place by the GEMM epilogues (``out = acc + residual``) and the MoE
combine. With hyper-connections (``hc_count > 1``) it is a stream of G branches ``[N, G, H]`` instead: every sub-layer
reads a mix of the branches and writes its output back to each branch with a gate (``ops/hc.py``). A step over N tokens launches, per layer, 6-9 kernels; the whole decode step is CUDA-graph capturable
(all shapes fixed by the batch layout, all indices on the device).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..config import FULL, ModelConfig
from ..ops import C
from ..ops.attention import PAGE, paged_attention
from ..ops.gdn import GdnScratch, GdnShape, GdnState, gdn_decode
from ..ops.hc import HCWeights, hc_inject_, hc_read
from ..ops.ple import PleServeState, PleServeWeights, ple_serve
from ..ops.moe import Fp8ExpertBank, Int3ExpertBank, MoEWorkspace, moe_forward, router_weight_with_shared_gate
from ..ops.qsa import qsa_attention
from ..parallel.ep import EPMoEWorkspace, moe_forward_ep
from .reference import HybridMoE, rope_cos_sin


@dataclass
class LayerWeights:
    kind: str
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    # attention
    w_qkv: torch.Tensor | None = None
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    w_o: torch.Tensor | None = None
    qsa_q_norm: torch.Tensor | None = None  # QSA indexer norms (w_qkv then also holds the index projection rows)
    qsa_k_norm: torch.Tensor | None = None
    # GDN
    w_in: torch.Tensor | None = None
    conv_w: torch.Tensor | None = None
    A_log: torch.Tensor | None = None
    dt_bias: torch.Tensor | None = None
    g_norm: torch.Tensor | None = None
    w_out: torch.Tensor | None = None
    # MoE
    router_ext: torch.Tensor | None = None
    bank: Int3ExpertBank | None = None
    shared_w13: torch.Tensor | None = None
    shared_w2: torch.Tensor | None = None
    # hyper-connections (hc_count > 1): the read before / write-back after each sub-layer
    hc_attn: HCWeights | None = None
    hc_mlp: HCWeights | None = None
    # per-layer n-gram embedding (the layers of cfg.ple_layer_ids)
    ple: PleServeWeights | None = None


@dataclass
class StepBatch:
    """Device-side description of one forward over ``num_seqs * q_per_seq`` tokens (uniform rows per sequence)."""
    ids: torch.Tensor          # [N] int32
    positions: torch.Tensor    # [N] int32
    slots: torch.Tensor        # [N] int32 KV slot (page * 64 + offset)
    block_table: torch.Tensor  # [S, max_pages] int32
    seq_lens: torch.Tensor     # [S] int32: tokens in the KV cache including this step's rows
    seq_slot: torch.Tensor     # [S] int32 GDN state slot
    n_commit: torch.Tensor     # [slots] int32 accepted rows of the previous cycle
    q_per_seq: int
    parity: int = 0
    commit_current: bool = False
    max_pages: int | None = None  # bound on pages per sequence (split plan)
    attn_bt_row: torch.Tensor | None = None    # prefill: virtual rows -> block-table row
    attn_seq_lens: torch.Tensor | None = None  # prefill: per-virtual-row lengths
    attn_q_per_seq: int | None = None

    @property
    def num_tokens(self) -> int:
        return self.ids.shape[0]


def _random_ple(cfg: ModelConfig, std: float, gen, dev) -> PleServeWeights:
    from ..models.ple import NgramHash
    from ..ops.ple import PleTable
    h = NgramHash(cfg)
    G, H, E = cfg.hc_count, cfg.hidden_size, cfg.ple_embed_dim
    D = E // cfg.ngram_heads
    # e4m3 rows drawn in chunks (a real table is ~51 GB: no full fp32 staging), scale std per 128 x 128 block
    rows = torch.empty(h.rows, D, dtype=torch.float8_e4m3fn, device=dev)
    step = max(1, (1 << 27) // D)
    for r0 in range(0, h.rows, step):
        n = min(step, h.rows - r0)
        rows[r0:r0 + n] = torch.randn(n, D, generator=gen, device=dev).clamp_(-8, 8).to(torch.float8_e4m3fn)
    scale = torch.full(((h.rows + 127) // 128, (D + 127) // 128), std, dtype=torch.float32, device=dev)

    def rn(*s):
        return torch.randn(*s, generator=gen, device=dev) * std
    z = torch.zeros(G * H, device=dev)
    return PleServeWeights(PleTable(h, rows, scale), rn(G * H, E), rn(H, E), z, z.clone(), z.clone(),
                           rn(G * H, cfg.ple_conv_kernel), G, H, cfg.rms_norm_eps, cfg.ple_conv_dilation)


def _ple_from_package(t: dict, prefix: str, cfg: ModelConfig, dev) -> PleServeWeights:
    from ..models.ple import NgramHash
    from ..ops.ple import PleTable
    rows = t[f"{prefix}.table.weight"]
    table = (PleTable(NgramHash(cfg), rows.to(dev), t[f"{prefix}.table.weight_scale_inv"].float().to(dev))
             if rows.dtype == torch.float8_e4m3fn else PleTable(NgramHash(cfg), rows.to(dev, torch.bfloat16), None))
    f = {n: t[f"{prefix}.{n}"].to(dev) for n in ("key_proj", "value_proj", "norm_key", "norm_query", "norm_conv",
                                                  "conv")}
    return PleServeWeights(table, f["key_proj"], f["value_proj"], f["norm_key"], f["norm_query"], f["norm_conv"],
                           f["conv"], cfg.hc_count, cfg.hidden_size, cfg.rms_norm_eps, cfg.ple_conv_dilation)


def _hc_from_package(t: dict, prefix: str, cfg: ModelConfig, dev) -> HCWeights:
    inj = t.get(f"{prefix}.w_inject")
    return HCWeights.from_tensors(t[f"{prefix}.hc_norm.weight"], t[f"{prefix}.w_down"], t[f"{prefix}.w_up"], inj,
                                  cfg.rms_norm_eps, dev)


class HybridModel:
    def __init__(self, cfg: ModelConfig, layers: list[LayerWeights], embed, final_norm, lm_head, device):
        self.cfg = cfg
        self.layers = layers
        self.embed = embed
        self.final_norm = final_norm
        self.lm_head = lm_head
        self.device = torch.device(device)
        c = cfg
        self.gdn_shape = GdnShape(c.linear_num_key_heads, c.linear_key_head_dim, c.linear_num_value_heads,
                                  c.linear_value_head_dim)
        cos, sin = rope_cos_sin(torch.arange(1 << 17, device=self.device), c.rotary_dim, c.rope_theta)
        self.rope_cos, self.rope_sin = cos.contiguous(), sin.contiguous()
        self.ep = None  # ExpertParallel when the routed experts are split over ranks
        self.hc_final: HCWeights | None = None  # the final branch readout of a hyper-connection model

    def enable_expert_parallel(self, world: int, rank: int, T_cap: int, group=None):
        """Split the routed experts over ``world`` ranks (keeps this rank's block) and route every MoE layer
        through the peer-memory exchange. ``T_cap`` bounds the tokens of one forward on any rank and must be the same
        on every rank (the exchange regions are laid out by it; the constructor checks)."""
        from ..parallel.ep import ExpertParallel, expert_range, local_bank
        c = self.cfg
        e0, e1 = expert_range(c.num_experts, world, rank)
        for lw in self.layers:
            if lw.bank.num_experts == c.num_experts:
                lw.bank = local_bank(lw.bank, world, rank)
            elif lw.bank.num_experts != e1 - e0:
                raise ValueError(f"layer holds {lw.bank.num_experts} experts, expected {c.num_experts} or {e1 - e0}")
        self.ep = ExpertParallel(world, rank, T_cap, c.hidden_size, c.num_experts_per_tok, c.num_experts,
                                 self.device, group)
        self.ep.track_waits(c.num_layers)
        return self.ep

    # ------------------------------------------------------------------ construction
    @classmethod
    def random(cls, cfg: ModelConfig, device, seed: int = 0, std: float | None = None, ep_world: int = 1):
        """Random-init weights of ``cfg`` generated directly on the device (INT3 experts as random codes).
        With ``ep_world > 1`` only one rank's block of ``E / ep_world`` experts is made per layer."""
        std = cfg.init_std if std is None else std
        dev = torch.device(device)
        gen = torch.Generator(device=dev).manual_seed(seed)

        def randn(*shape):
            return (torch.randn(*shape, generator=gen, device=dev) * std).to(torch.bfloat16)

        H = cfg.hidden_size
        gs = GdnShape(cfg.linear_num_key_heads, cfg.linear_key_head_dim, cfg.linear_num_value_heads,
                      cfg.linear_value_head_dim)
        layers = []
        for kind in cfg.layer_types:
            lw = LayerWeights(kind, torch.zeros(H, dtype=torch.bfloat16, device=dev),
                              torch.zeros(H, dtype=torch.bfloat16, device=dev))
            if kind == FULL:
                D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_kv_heads
                lw.w_qkv = randn(Hq * 2 * D + 2 * Hkv * D + cfg.qsa_proj_dim, H)
                if cfg.qsa_topk:
                    lw.qsa_q_norm = torch.zeros(cfg.qsa_indexer_dim, dtype=torch.bfloat16, device=dev)
                    lw.qsa_k_norm = torch.zeros(cfg.qsa_indexer_dim, dtype=torch.bfloat16, device=dev)
                lw.q_norm = torch.zeros(D, dtype=torch.bfloat16, device=dev)
                lw.k_norm = torch.zeros(D, dtype=torch.bfloat16, device=dev)
                lw.w_o = randn(H, Hq * D)
            else:
                lw.w_in = randn(gs.mixed_dim, H)
                lw.conv_w = (torch.randn(gs.conv_dim, 4, generator=gen, device=dev) * 0.3).float()
                lw.A_log = torch.log(torch.empty(gs.Hv, device=dev).uniform_(1, 16, generator=gen))
                dt = torch.exp(torch.empty(gs.Hv, device=dev).uniform_(math.log(1e-3), math.log(1e-1),
                                                                        generator=gen))
                lw.dt_bias = dt + torch.log(-torch.expm1(-dt))
                lw.g_norm = torch.ones(gs.Dv, dtype=torch.bfloat16, device=dev)
                lw.w_out = randn(H, gs.Hv * gs.Dv)
            E, I, Is = cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
            lw.router_ext = router_weight_with_shared_gate(randn(E, H), randn(1, H))
            E = E // ep_world
            if cfg.expert_format == "fp8":  # block-FP8 experts (the QAD teacher): e4m3 of N(0, 1), scale std / 1
                def fp8w(rows, k):
                    w = torch.empty(E, rows, k, dtype=torch.float8_e4m3fn, device=dev)
                    for e0 in range(0, E, 32):  # in slices: the fp32 draw of a whole bank would not fit
                        e1 = min(E, e0 + 32)
                        w[e0:e1] = torch.randn(e1 - e0, rows, k, generator=gen, device=dev).to(torch.float8_e4m3fn)
                    return w, torch.full((E, rows // 128, k // 128), std, dtype=torch.float32, device=dev)
                a, sa = fp8w(2 * I, H)
                b, sb = fp8w(H, I)
                lw.bank = Fp8ExpertBank(a, sa, b, sb)
                lw.shared_w13 = randn(2 * Is, H)
                lw.shared_w2 = randn(H, Is)
                if cfg.hc_count > 1:
                    lw.hc_attn, lw.hc_mlp = (HCWeights.random(cfg.hc_count, H, cfg.hc_lowrank, std, cfg.rms_norm_eps,
                                                              True, gen, dev) for _ in range(2))
                layers.append(lw)
                continue
            lw.bank = Int3ExpertBank(
                torch.randint(-2**31, 2**31 - 1, (E, 2 * I // 128, H // 128, 128, 12), dtype=torch.int32,
                              device=dev, generator=gen),
                (torch.randn(E, 2 * I // 128, H // 128, 128, generator=gen, device=dev) * std / 2.3).to(
                    torch.bfloat16),
                torch.randint(-2**31, 2**31 - 1, (E, H // 128, I // 128, 128, 12), dtype=torch.int32, device=dev,
                              generator=gen),
                (torch.randn(E, H // 128, I // 128, 128, generator=gen, device=dev) * std / 2.3).to(
                    torch.bfloat16))
            lw.shared_w13 = randn(2 * Is, H)
            lw.shared_w2 = randn(H, Is)
            layers.append(lw)
        G = cfg.hc_count
        if G > 1:
            for lw in layers:
                lw.hc_attn, lw.hc_mlp = (HCWeights.random(G, H, cfg.hc_lowrank, std, cfg.rms_norm_eps, True, gen, dev)
                                         for _ in range(2))
        for i in cfg.ple_layer_ids:
            layers[i].ple = _random_ple(cfg, std, gen, dev)
        embed = randn(cfg.vocab_size, H)
        m = cls(cfg, layers, embed, torch.zeros(H, dtype=torch.bfloat16, device=dev), randn(cfg.vocab_size, H), dev)
        if G > 1:
            m.hc_final = HCWeights.random(G, H, cfg.hc_lowrank, std, cfg.rms_norm_eps, False, gen, dev)
        return m

    @classmethod
    def from_reference(cls, ref: HybridMoE, device, codes_scales: list | None = None):
        """Convert the oracle model. ``codes_scales``: per layer (w13_codes, w13_scales, w2_codes, w2_scales) of
        INT3-quantised experts; without it the experts are RTN-quantised here."""
        from ..quant.gptq import rtn_quantize
        cfg = ref.cfg
        dev = torch.device(device)
        bf = dict(dtype=torch.bfloat16, device=dev)
        layers = []
        for i, L in enumerate(ref.layers):
            lw = LayerWeights(L.kind, L.input_layernorm.weight.detach().to(**bf),
                              L.post_attention_layernorm.weight.detach().to(**bf))
            m = L.mixer
            if L.kind == FULL:
                idx = [m.index_qk_proj.weight] if cfg.qsa_topk else []  # QSA index rows after q | k | v
                lw.w_qkv = torch.cat([m.q_proj.weight, m.k_proj.weight, m.v_proj.weight, *idx]).detach().to(**bf)
                if cfg.qsa_topk:
                    lw.qsa_q_norm = m.index_q_norm.weight.detach().to(**bf)
                    lw.qsa_k_norm = m.index_k_norm.weight.detach().to(**bf)
                lw.q_norm = m.q_norm.weight.detach().to(**bf)
                lw.k_norm = m.k_norm.weight.detach().to(**bf)
                lw.w_o = m.o_proj.weight.detach().to(**bf).contiguous()
            else:
                lw.w_in = torch.cat([m.in_proj_qkvz.weight, m.in_proj_ba.weight]).detach().to(**bf)
                lw.conv_w = m.conv1d.detach().float().to(dev).contiguous()
                lw.A_log = m.A_log.detach().float().to(dev)
                lw.dt_bias = m.dt_bias.detach().float().to(dev)
                lw.g_norm = m.norm.detach().to(**bf)
                lw.w_out = m.out_proj.weight.detach().to(**bf).contiguous()
            moe = L.mlp
            lw.router_ext = router_weight_with_shared_gate(moe.gate.weight.detach().to(**bf),
                                                           moe.shared_expert_gate.weight.detach().to(**bf))
            if codes_scales is not None:
                c13, s13, c2, s2 = codes_scales[i]
            else:
                c13, s13 = rtn_quantize(moe.w13.detach().float())
                c2, s2 = rtn_quantize(moe.w2.detach().float())
            lw.bank = Int3ExpertBank.from_codes(c13, s13.to(torch.bfloat16), c2, s2.to(torch.bfloat16), dev)
            lw.shared_w13 = torch.cat([moe.shared_gate_proj.weight, moe.shared_up_proj.weight]).detach().to(**bf)
            lw.shared_w2 = moe.shared_down_proj.weight.detach().to(**bf).contiguous()
            if getattr(L, "hc", False):
                lw.hc_attn, lw.hc_mlp = HCWeights.from_module(L.hc_attn, dev), HCWeights.from_module(L.hc_mlp, dev)
            if getattr(L, "ple", None) is not None:
                lw.ple = PleServeWeights.from_module(L.ple, dev)
            layers.append(lw)
        m = cls(cfg, layers, ref.embed_tokens.weight.detach().to(**bf), ref.norm.weight.detach().to(**bf),
                ref.lm_head.weight.detach().to(**bf), dev)
        if cfg.hc_count > 1:
            m.hc_final = HCWeights.from_module(ref.hc_final, dev)
        return m

    @classmethod
    def from_package(cls, pkg_dir, device, verify: bool = True, weight_patch=None, merged=None):
        """Load an INT3 deploy package (``formats/int3_package.py``): uint3 expert packs are re-tiled for the
        expert GEMM, block-FP8 dense modules dequantised to bf16 for the dense GEMMs. ``weight_patch`` / ``merged``:
        an RL weight patch or merged version served over the unchanged package (``read_package``)."""
        from ..formats.int3_package import dense_weight, expert_codes, read_package
        cfg, t = read_package(pkg_dir, verify, weight_patch=weight_patch, merged=merged)
        dev = torch.device(device)
        bf = dict(dtype=torch.bfloat16, device=dev)
        layers = []
        for i, kind in enumerate(cfg.layer_types):
            p = f"model.layers.{i}"
            lw = LayerWeights(kind, t[f"{p}.input_layernorm.weight"].to(**bf),
                              t[f"{p}.post_attention_layernorm.weight"].to(**bf))
            if kind == FULL:
                a = f"{p}.self_attn"
                lw.w_qkv = torch.cat([dense_weight(t, f"{a}.{n}") for n in ("q_proj", "k_proj", "v_proj")]).to(**bf)
                lw.q_norm = t[f"{a}.q_norm.weight"].to(**bf)
                lw.k_norm = t[f"{a}.k_norm.weight"].to(**bf)
                lw.w_o = dense_weight(t, f"{a}.o_proj").to(**bf).contiguous()
            else:
                g = f"{p}.linear_attn"
                lw.w_in = torch.cat([dense_weight(t, f"{g}.in_proj_qkvz"), dense_weight(t, f"{g}.in_proj_ba")]).to(**bf)
                lw.conv_w = t[f"{g}.conv1d.weight"].float().to(dev).contiguous()
                lw.A_log = t[f"{g}.A_log"].float().to(dev)
                lw.dt_bias = t[f"{g}.dt_bias"].float().to(dev)
                lw.g_norm = t[f"{g}.norm.weight"].to(**bf)
                lw.w_out = dense_weight(t, f"{g}.out_proj").to(**bf).contiguous()
            m = f"{p}.mlp"
            lw.router_ext = router_weight_with_shared_gate(dense_weight(t, f"{m}.gate").to(**bf),
                                                           dense_weight(t, f"{m}.shared_expert_gate").to(**bf))
            c13, s13, c2, s2 = expert_codes(t, i, cfg)
            lw.bank = Int3ExpertBank.from_codes(c13, s13, c2, s2, dev)
            lw.shared_w13 = torch.cat([dense_weight(t, f"{m}.shared_expert.gate_proj"),
                                       dense_weight(t, f"{m}.shared_expert.up_proj")]).to(**bf)
            lw.shared_w2 = dense_weight(t, f"{m}.shared_expert.down_proj").to(**bf).contiguous()
            if cfg.hc_count > 1:
                lw.hc_attn, lw.hc_mlp = (_hc_from_package(t, f"{p}.{n}", cfg, dev) for n in ("hc_attn", "hc_mlp"))
            if i in cfg.ple_layer_ids:
                lw.ple = _ple_from_package(t, f"{p}.ple", cfg, dev)
            layers.append(lw)
        m = cls(cfg, layers, t["model.embed_tokens.weight"].to(**bf), t["model.norm.weight"].to(**bf),
                t["lm_head.weight"].to(**bf), dev)
        if cfg.hc_count > 1:
            m.hc_final = _hc_from_package(t, "model.hc_final", cfg, dev)
        m.pkg_dir = str(pkg_dir)
        return m

    def tensors(self):
        """(name, tensor) of every weight the forward reads (layer fields, expert-bank fields, embeddings)."""
        yield "embed", self.embed
        yield "final_norm", self.final_norm
        yield "lm_head", self.lm_head
        if self.hc_final is not None:
            for k, v in vars(self.hc_final).items():
                if isinstance(v, torch.Tensor):
                    yield f"hc_final.{k}", v
        for i, lw in enumerate(self.layers):
            for k, v in vars(lw).items():
                if isinstance(v, torch.Tensor):
                    yield f"layers.{i}.{k}", v
                elif v is not None and hasattr(v, "__dict__"):
                    for bk, bv in vars(v).items():
                        if isinstance(bv, torch.Tensor):
                            yield f"layers.{i}.{k}.{bk}", bv

    @torch.no_grad()
    def update_from_package(self, pkg_dir) -> dict:
        """Replace the weights by those of a deploy package of the same architecture, copying into the existing
        tensors (addresses unchanged: captured CUDA graphs stay valid). ``pkg_dir`` may also be an RL weight patch
        (``patch.json``) or a merged version (``merged_manifest.json``): it is then applied over the package this
        model was loaded from. Expert-parallel models keep their block of experts. Raises before writing anything if
        any tensor differs in shape or dtype."""
        from pathlib import Path
        d = Path(pkg_dir)
        base = getattr(self, "pkg_dir", None)
        if (d / "patch.json").exists() or (d / "merged_manifest.json").exists():
            if base is None:
                raise ValueError(f"{d} patches a package, but this model was not loaded from one")
            kw = {"weight_patch": d} if (d / "patch.json").exists() else {"merged": d}
            new = HybridModel.from_package(base, self.device, **kw)
        else:
            new = HybridModel.from_package(pkg_dir, self.device)
            base = str(pkg_dir)
        if self.ep is not None:
            from ..parallel.ep import local_bank
            for lw in new.layers:
                lw.bank = local_bank(lw.bank, self.ep.world, self.ep.rank)
        mine, theirs = dict(self.tensors()), dict(new.tensors())
        if mine.keys() != theirs.keys():
            raise ValueError(f"package tensors differ: {sorted(set(mine) ^ set(theirs))[:8]}")
        for k, t in mine.items():
            if t.shape != theirs[k].shape or t.dtype != theirs[k].dtype:
                raise ValueError(f"{k}: {tuple(theirs[k].shape)} {theirs[k].dtype} vs {tuple(t.shape)} {t.dtype}")
        for k, t in mine.items():
            t.copy_(theirs[k])
        self.pkg_dir = base
        return {"tensors": len(mine)}

    def nbytes(self) -> int:
        return sum(t.nbytes for _, t in self.tensors())

    # ------------------------------------------------------------------ caches
    def new_kv_cache(self, num_pages: int, kv_dtype: str = "bf16"):
        """Per attention layer (k, v) bf16 pages, or with ``kv_dtype="nvfp4"`` (k, v, kscale, vscale): e2m1 codes
        and e4m3 scales per 16 elements (``ops/attention.py`` ``new_nvfp4_kv``)."""
        c = self.cfg
        if kv_dtype == "nvfp4":
            from ..ops.attention import new_nvfp4_kv
            return [new_nvfp4_kv(num_pages, c.num_kv_heads, c.head_dim, self.device)
                    for _ in range(c.num_attention_layers)]
        if kv_dtype != "bf16":
            raise ValueError(f"kv_dtype {kv_dtype!r}: bf16 or nvfp4")
        shape = (num_pages, c.num_kv_heads, PAGE, c.head_dim)
        return [(torch.zeros(shape, dtype=torch.bfloat16, device=self.device),
                 torch.zeros(shape, dtype=torch.bfloat16, device=self.device)) for _ in range(c.num_attention_layers)]

    def new_qsa_cache(self, num_pages: int, sessions: int, max_pages: int):
        """Per full-attention layer: raw index keys by KV slot [pages*64, 128] and pooled block keys by (session
        row, block index) [sessions * max_pages * 64 / qsa_block, 128]."""
        z = dict(dtype=torch.bfloat16, device=self.device)
        nb = max_pages * (PAGE // self.cfg.qsa_block)
        return [(torch.zeros(num_pages * PAGE, self.cfg.qsa_indexer_dim, **z),
                 torch.zeros(sessions * nb, self.cfg.qsa_indexer_dim, **z))
                for _ in range(self.cfg.num_attention_layers)]

    def new_ple_states(self, slots: int, max_q: int):
        """Side state of every PLE layer (n-gram history, conv inputs, pending rows of the last window)."""
        return [PleServeState(lw.ple, slots, max_q, self.device) for lw in self.layers if lw.ple is not None]

    def new_gdn_states(self, slots: int, max_q: int):
        return [GdnState(self.gdn_shape, slots, max_q, self.device) for _ in range(self.cfg.num_gdn_layers)]

    def new_workspace(self, max_tokens: int):
        return Workspace(self, max_tokens)

    # ------------------------------------------------------------------ forward
    def forward(self, b: StepBatch, kv, gdn, ws: "Workspace", gdn_scratch: GdnScratch | None = None, qsa=None,
                ple=None):
        """Runs the stack over b.ids; returns the final-normed hidden rows [N, H] (a view into the workspace).
        ``qsa`` (a ``QsaState``): the full-attention layers store index keys and, on verify batches, attend to
        their QSA page selection instead of the whole context. ``ple``: the PLE side states (``new_ple_states``) when
        the model has PLE layers."""
        c, cC = self.cfg, C()
        N, H = b.num_tokens, c.hidden_size
        if self.ep is not None:
            self.ep.ctx.begin_step()  # per-layer wait slots restart with the stack
        h = ws.h[:N]
        cC.embedding(b.ids, self.embed, h)
        y = ws.y[:N]
        ai = gi = 0
        D, Hq, Hkv = c.head_dim, c.num_attention_heads, c.num_kv_heads
        G = c.hc_count
        hs = None
        if G > 1:  # branch stream; h becomes the sub-layer output buffer
            hs = ws.hs[:N]
            hs.copy_(h[:, None, :].expand(N, G, H))
        pi = 0
        for lw in self.layers:
            if lw.ple is not None:
                ple_serve(hs if hs is not None else h.view(N, 1, H), b.ids, lw.ple, ple[pi], b.seq_slot, b.n_commit,
                          b.q_per_seq, b.parity, b.commit_current)
                pi += 1
            if hs is not None:
                x, hc_gate = hc_read(hs, lw.hc_attn, G)
                cC.rmsnorm(x, None, lw.in_norm, y, c.rms_norm_eps, True)
            else:
                cC.rmsnorm(h, None, lw.in_norm, y, c.rms_norm_eps, True)
            if lw.kind == FULL:
                qkv = ws.qkv[:N]
                cC.gemm(y, lw.w_qkv, out=qkv)
                kc, vc, *kvs = kv[ai]  # kvs: the NVFP4 scales, or empty for a bf16 cache
                kvs = tuple(kvs) or None
                q = ws.q[:N]
                cC.qk_norm_rope_store(qkv, Hq, Hkv, D, c.rotary_dim, lw.q_norm, lw.k_norm, b.positions, b.slots,
                                      self.rope_cos, self.rope_sin, c.rms_norm_eps, q, kc, vc,
                                      *(kvs or (None, None)))
                attn = ws.attn[:N]
                row_len = qkv.shape[1]
                gate = qkv[:, D:]
                if qsa is not None:
                    raw, key = qsa.cache[ai]
                    cC.qsa_prep(qkv, Hq * 2 * D + 2 * Hkv * D, b.positions, b.slots, lw.qsa_q_norm, self.rope_cos,
                                self.rope_sin, c.rms_norm_eps, c.qsa_indexer_heads, c.rotary_dim, qsa.ws.idx_q, raw)
                if qsa is not None and b.attn_bt_row is None:
                    qsa_attention(q.view(-1, Hq, D), kc, vc, b.block_table, b.seq_lens, qsa.fin, key, qsa.ws,
                                  attn.view(-1, Hq, D), gate=gate, gate_ld=row_len, gate_head_stride=2 * D,
                                  splits=qsa.splits, hs=qsa.hs, layer=ai, replay=qsa.replay, kv_scales=kvs,
                                  raw=raw, k_norm=lw.qsa_k_norm, rope=(self.rope_cos, self.rope_sin),
                                  rot=c.rotary_dim, eps=c.rms_norm_eps)
                elif b.attn_bt_row is not None and qsa is not None and qsa.pf is not None:
                    # prefill under QSA: row sets of attn_q_per_seq positions select their blocks like verify rows
                    qp = b.attn_q_per_seq
                    nv = b.attn_bt_row.shape[0]
                    qsa.prefill_attention(ws.q[: nv * qp].view(-1, Hq, D), kc, vc, b.block_table, b.attn_seq_lens,
                                          b.attn_bt_row, ai, raw, key, lw.qsa_k_norm,
                                          ws.attn[: nv * qp].view(-1, Hq, D), ws.qkv[: nv * qp, D:], row_len, 2 * D,
                                          kv_scales=kvs)
                elif b.attn_bt_row is not None:
                    # prefill: virtual rows of attn_q_per_seq queries; rows past N are padding (scratch)
                    qp = b.attn_q_per_seq
                    nv = b.attn_bt_row.shape[0]
                    paged_attention(ws.q[: nv * qp].view(-1, Hq, D), kc, vc, b.block_table, b.attn_seq_lens, qp,
                                    ws.attn[: nv * qp].view(-1, Hq, D), gate=ws.qkv[: nv * qp, D:], gate_ld=row_len,
                                    gate_head_stride=2 * D, max_pages=b.max_pages, bt_row=b.attn_bt_row, kv_scales=kvs)
                else:
                    paged_attention(q.view(-1, Hq, D), kc, vc, b.block_table, b.seq_lens, b.q_per_seq,
                                    attn.view(-1, Hq, D), gate=gate, gate_ld=row_len, gate_head_stride=2 * D,
                                    max_pages=b.max_pages, kv_scales=kvs)
                cC.gemm(attn, lw.w_o, out=h, residual=None if hs is not None else h)
                ai += 1
            else:
                mixed = ws.mixed[:N]
                cC.gemm(y, lw.w_in, out=mixed)
                o = ws.gdn_out[:N]
                gdn_decode(mixed, self.gdn_shape, gdn[gi], lw.conv_w, lw.A_log, lw.dt_bias, lw.g_norm, b.n_commit,
                           b.seq_slot, o, b.q_per_seq, b.parity, b.commit_current, gdn_scratch, c.rms_norm_eps)
                cC.gemm(o, lw.w_out, out=h, residual=None if hs is not None else h)
                gi += 1
            resid = h
            if hs is not None:
                hc_inject_(hs, h, hc_gate)
                x, hc_gate = hc_read(hs, lw.hc_mlp, G)
                cC.rmsnorm(x, None, lw.post_norm, y, c.rms_norm_eps, True)
                resid = ws.zero[:N]
            else:
                cC.rmsnorm(h, None, lw.post_norm, y, c.rms_norm_eps, True)
            if self.ep is not None:
                moe_forward_ep(y, resid, lw.router_ext, lw.bank, lw.shared_w13, lw.shared_w2, self.ep, ws.moe, out=h,
                               renorm=c.norm_topk_prob)
            else:
                moe_forward(y, resid, lw.router_ext, lw.bank, lw.shared_w13, lw.shared_w2, c.num_experts_per_tok,
                            ws.moe, out=h, renorm=c.norm_topk_prob)
            if hs is not None:
                hc_inject_(hs, h, hc_gate)
        if hs is not None:
            h = hc_read(hs, self.hc_final, G)[0]
        cC.rmsnorm(h, None, self.final_norm, y, c.rms_norm_eps, True)
        return y

    def logits(self, hidden: torch.Tensor, out: torch.Tensor | None = None, fp32: bool = False):
        return C().gemm(hidden, self.lm_head, out=out, out_fp32=fp32)


class Workspace:
    """All per-step activations for up to ``max_tokens`` rows (fixed addresses: CUDA-graph safe)."""

    def __init__(self, model: HybridModel, max_tokens: int):
        c = model.cfg
        dev = model.device
        bf = dict(dtype=torch.bfloat16, device=dev)
        H = c.hidden_size
        self.max_tokens = max_tokens
        self.h = torch.empty(max_tokens, H, **bf)
        self.y = torch.empty(max_tokens, H, **bf)
        if c.hc_count > 1:  # branch stream and the zero residual of the MoE output
            self.hs = torch.empty(max_tokens, c.hc_count, H, **bf)
            self.zero = torch.zeros(max_tokens, H, **bf)
        D, Hq, Hkv = c.head_dim, c.num_attention_heads, c.num_kv_heads
        self.qkv = torch.empty(max_tokens + 8, Hq * 2 * D + 2 * Hkv * D + c.qsa_proj_dim, **bf)
        self.q = torch.empty(max_tokens + 8, Hq * D, **bf)
        self.attn = torch.empty(max_tokens + 8, Hq * D, **bf)
        gs = model.gdn_shape
        self.mixed = torch.empty(max_tokens, gs.mixed_dim, **bf)
        self.gdn_out = torch.empty(max_tokens, gs.Hv * gs.Dv, **bf)
        if model.ep is not None:
            self.moe = EPMoEWorkspace(model.ep, c.moe_intermediate_size, c.shared_expert_intermediate_size, dev)
        else:
            self.moe = MoEWorkspace(max_tokens, c.num_experts, c.num_experts_per_tok, H, c.moe_intermediate_size,
                                    c.shared_expert_intermediate_size, dev)
