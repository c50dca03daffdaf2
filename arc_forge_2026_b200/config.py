"""Typed configuration for every part of the framework.

One dataclass per concern (model shape, serving, speculative decoding, QAD training), each
serialisable to and from JSON, plus an environment-override layer that validates strictly.

The reference has no central config object: argparse per tool, ~40 ``ARC_*`` environment flags
validated by ``_flag`` (``agi2/work/qwen38fn_l4/probes/hostcomm/arc_hostcomm_hook.py:89-94``, raises on
anything but 0/1), JSON presets and module-level mutable dicts. Here the same knobs are fields of
typed dataclasses; :func:`apply_env_overrides` accepts ``AFB_<SECTION>_<FIELD>=value`` and rejects
unknown keys and unparsable values instead of guessing.

Model presets:

* ``tiny_cpu``: 4 layers (3 GDN + 1 gated attention), hidden 256, 32 routed
  experts top-4 + 1 shared, expert FFN 128, vocab 4096.
* ``qwen3next_80b`` -- the Qwen3-Next-80B-A3B shape with 320 routed experts (the gEAN-pruned count):
  48 layers, hidden 2048, GDN:attention 3:1, attention 16Q/2KV x 256, GDN 16 QK / 32 V heads x 128,
  top-10 of 320 experts with intermediate 512 plus a 512-wide shared expert, vocab 151,936.
* ``qwen3next_80b_teacher`` -- the same with 512 experts (QAD teacher, block FP8).
* ``qwen38fn`` -- the reference's own shape (``training/run_records/A4/config/recorded-config-99c11efb.json``):
  hidden 2560, 24Q/2KV x 256, GDN 16 QK / 48 V heads, 512 experts x 640, vocab 248,320, 4 hyper-connections,
  PLE at layer 2, QSA top-512 of 4-token blocks (indexer budget 2048, compress ratio 4, 4 heads x 128).
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any

LINEAR = "linear_attention"
FULL = "full_attention"


@dataclass
class ModelConfig:
    name: str = "tiny_cpu"
    vocab_size: int = 4096
    hidden_size: int = 256
    num_layers: int = 4
    full_attention_interval: int = 4  # every 4th layer is gated attention, the rest are GDN
    # gated attention
    num_attention_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 64
    partial_rotary_factor: float = 0.25
    rope_theta: float = 1.0e7
    # Gated DeltaNet
    linear_num_key_heads: int = 2
    linear_num_value_heads: int = 4
    linear_key_head_dim: int = 64
    linear_value_head_dim: int = 64
    linear_conv_kernel: int = 4
    # MoE
    num_experts: int = 32
    num_experts_per_tok: int = 4
    moe_intermediate_size: int = 128
    shared_expert_intermediate_size: int = 128
    norm_topk_prob: bool = True
    # misc
    rms_norm_eps: float = 1.0e-6
    hc_count: int = 1  # hyper-connection branches; 1 = plain residual stream
    hc_lowrank: int = 320  # rank of the hyper-connection mix projection
    # per-layer n-gram embeddings (PLE): layers (0-based) that add a gated n-gram embedding to the stream
    ple_layer_ids: tuple = ()
    ngram_size: int = 3
    heads_per_ngram: int = 8
    ngram_vocab_size_base: int = 20_000_000
    ple_embed_dim: int = 2560
    ple_conv_kernel: int = 4
    ple_conv_dilation: int = 1
    ngram_seed: int = 1234
    eos_token_id: int = 2
    init_std: float = 0.02
    # QSA sparse attention on the full-attention layers (0 = dense attention)
    qsa_block: int = 0
    qsa_topk: int = 0
    qsa_indexer_heads: int = 4
    qsa_indexer_dim: int = 128
    # storage format of the routed experts: "int3" (uint3 g128), "fp8" (128x128 block), "bf16"
    expert_format: str = "bf16"
    # multimodal RoPE: frequencies of the rotary dims split (temporal, height, width), interleaved; None = text-only
    # 1-D RoPE. With three-row positions (``models/vision.py`` ``mrope_positions``) image tokens rotate by their grid
    # position; text tokens have equal rows and get plain RoPE.
    mrope_section: tuple | None = None

    def __post_init__(self):
        if self.num_attention_heads % self.num_kv_heads:
            raise ValueError("num_attention_heads must be a multiple of num_kv_heads")
        if self.linear_num_value_heads % self.linear_num_key_heads:
            raise ValueError("GDN value heads must be a multiple of key heads")
        if not 1 <= self.num_experts_per_tok <= self.num_experts:
            raise ValueError("invalid top-k")
        if self.qsa_topk and (self.qsa_block not in (4, 8, 16, 32, 64) or self.qsa_indexer_dim != 128
                              or not 1 <= self.qsa_indexer_heads <= 4):
            raise ValueError("QSA needs blocks of 4..64 tokens dividing the 64-token page, 128-dim index heads and "
                             "1..4 of them")
        rot = self.rotary_dim
        if rot <= 0 or rot % 2:
            raise ValueError("rotary dimension must be positive and even")
        if self.mrope_section is not None:
            self.mrope_section = tuple(int(x) for x in self.mrope_section)
            if len(self.mrope_section) != 3 or sum(self.mrope_section) != rot // 2:
                raise ValueError(f"mrope_section {self.mrope_section} must split the {rot // 2} rotary frequencies "
                                 "into (temporal, height, width)")
        if self.expert_format not in ("int3", "fp8", "bf16"):
            raise ValueError(f"expert_format {self.expert_format!r}")
        self.ple_layer_ids = tuple(int(i) for i in self.ple_layer_ids)
        if any(not 0 <= i < self.num_layers for i in self.ple_layer_ids):
            raise ValueError(f"ple_layer_ids {self.ple_layer_ids} outside the {self.num_layers} layers")
        if self.ple_layer_ids and (self.ngram_size < 2 or self.ple_embed_dim % self.ngram_heads
                                   or (self.ple_embed_dim // self.ngram_heads) % 16):
            raise ValueError("PLE: ple_embed_dim must split into ngram heads of a multiple of 16 dims")
        if self.expert_format == "int3" and (self.hidden_size % 128 or self.moe_intermediate_size % 128):
            raise ValueError("uint3 g128 experts need hidden and expert widths divisible by 128")

    @property
    def layer_types(self) -> list[str]:
        return [FULL if (i + 1) % self.full_attention_interval == 0 else LINEAR for i in range(self.num_layers)]

    @property
    def ngram_heads(self) -> int:
        return (self.ngram_size - 1) * self.heads_per_ngram

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def qsa_proj_dim(self) -> int:
        """Columns the attention projection carries for the QSA indexer (index query heads + raw key), 0 if off."""
        return (self.qsa_indexer_heads + 1) * self.qsa_indexer_dim if self.qsa_topk else 0

    @property
    def gdn_conv_dim(self) -> int:
        return 2 * self.linear_num_key_heads * self.linear_key_head_dim + self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def gdn_qkvz_dim(self) -> int:
        return self.gdn_conv_dim + self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def num_attention_layers(self) -> int:
        return sum(t == FULL for t in self.layer_types)

    @property
    def num_gdn_layers(self) -> int:
        return sum(t == LINEAR for t in self.layer_types)

    def kv_bytes_per_token(self, elem_bytes: int = 2) -> int:
        return self.num_attention_layers * 2 * self.num_kv_heads * self.head_dim * elem_bytes

    def gdn_state_bytes(self, elem_bytes: int = 4) -> int:
        """Recurrent state of one sequence over all GDN layers (S is [Hv, Dk, Dv])."""
        per = self.linear_num_value_heads * self.linear_key_head_dim * self.linear_value_head_dim * elem_bytes
        return self.num_gdn_layers * per


@dataclass
class DrafterConfig:
    """DFlash block drafter: plain residual, target-hidden conditioning, injected context K/V."""
    num_layers: int = 8
    hidden_size: int = 2048
    num_attention_heads: int = 16
    num_kv_heads: int = 2
    head_dim: int = 128
    intermediate_size: int = 6144
    window: int = 1024
    block_size: int = 5  # anchor + K proposal slots (verify width K=4)
    rms_norm_eps: float = 1.0e-6
    rope_theta: float = 1.0e7
    # training variants (the serving drafter is plain / dense; train/drafter_tools.py converts the others)
    residual: str = "plain"  # plain | hc (hyper-connection branch stream)
    hc_count: int = 1
    hc_lowrank: int = 64
    ffn: str = "dense"  # dense | dense_shared (a dense SwiGLU plus a sigmoid-gated shared SwiGLU)
    shared_intermediate_size: int = 0
    # candidate selector (0: none, proposals are the unary argmax): re-ranks the top-k draft candidates of each slot
    # with a rank-r bilinear term in the predecessor token and the slot's hidden state (train/drafter_objective.py)
    selector_top_k: int = 0
    selector_rank: int = 64

    @property
    def k(self) -> int:
        return self.block_size - 1


@dataclass
class ServeConfig:
    max_sessions: int = 128
    page_size: int = 64
    max_context: int = 32768
    kv_dtype: str = "bf16"  # target KV cache: bf16 | nvfp4 (e2m1 + e4m3 per 16 elements: 3.6x the tokens per byte)
    gdn_state_dtype: str = "fp32"
    spec_k: int = 4  # 0 disables speculative decoding
    accept_mode: str = "rejection"  # rejection | greedy | bernoulli
    accept_prob: float = 0.7  # for bernoulli mode
    seed: int = 0
    cuda_graphs: bool = True
    temperature: float = 0.0
    qsa_splits: int = 4  # KV splits of the QSA union (per session: W*K + local pages)
    hisparse: bool = False  # KV history of the QSA layers in pinned host memory (needs QSA)
    hisparse_hot_blocks: int = 0  # GPU cache slots per session and layer (0: W * qsa_topk + 32)
    hisparse_fp8: bool = False  # host pool in e4m3 with per-(page, head) scales (half the host memory)
    parallel: str = "single"  # single | ep (EP over the world, DP attention)
    fused_comm: bool = True  # EP dispatch/combine in our peer-memory kernels (False = NCCL baseline)


@dataclass
class QADConfig:
    seq_len: int = 16384
    global_batch: int = 32
    topk: int = 64
    direction: str = "reverse"  # KL direction over the top-k + tail classes
    lr_scale: float = 1.0e-5
    lr_router: float = 3.0e-6
    lr_dense: float = 2.0e-6
    betas: tuple[float, float] = (0.9, 0.95)
    weight_decay: float = 0.0
    optimizer_state_dtype: str = "bf16"
    grad_clip: float = 1.0
    fused_comm: bool = True


PRESETS: dict[str, dict[str, Any]] = {
    "tiny_cpu": dict(name="tiny_cpu"),
    # the tiny shape with the head size the GPU attention kernels take (128)
    "tiny_gpu": dict(name="tiny_gpu", head_dim=128, expert_format="int3"),
    "qwen3next_80b": dict(
        name="qwen3next_80b", vocab_size=151936, hidden_size=2048, num_layers=48, full_attention_interval=4,
        num_attention_heads=16, num_kv_heads=2, head_dim=256, partial_rotary_factor=0.25, rope_theta=1.0e7,
        linear_num_key_heads=16, linear_num_value_heads=32, linear_key_head_dim=128, linear_value_head_dim=128,
        num_experts=320, num_experts_per_tok=10, moe_intermediate_size=512, shared_expert_intermediate_size=512,
        expert_format="int3"),
    "qwen3next_80b_teacher": dict(
        name="qwen3next_80b_teacher", vocab_size=151936, hidden_size=2048, num_layers=48, full_attention_interval=4,
        num_attention_heads=16, num_kv_heads=2, head_dim=256, linear_num_key_heads=16, linear_num_value_heads=32,
        linear_key_head_dim=128, linear_value_head_dim=128, num_experts=512, num_experts_per_tok=10,
        moe_intermediate_size=512, shared_expert_intermediate_size=512, expert_format="fp8"),
    "qwen38fn": dict(
        name="qwen38fn", vocab_size=248320, hidden_size=2560, num_layers=48, full_attention_interval=4,
        num_attention_heads=24, num_kv_heads=2, head_dim=256, linear_num_key_heads=16, linear_num_value_heads=48,
        linear_key_head_dim=128, linear_value_head_dim=128, num_experts=512, num_experts_per_tok=10,
        moe_intermediate_size=640, shared_expert_intermediate_size=640, hc_count=4, ple_layer_ids=(2,), qsa_block=4,
        qsa_topk=512, expert_format="int3"),
}


DRAFTER_PRESETS: dict[str, dict[str, Any]] = {
    "dflash_8l": dict(),
    "tiny": dict(num_layers=2, hidden_size=256, num_attention_heads=4, num_kv_heads=2, head_dim=128,
                 intermediate_size=512),
}


def drafter_preset(name: str, **overrides) -> DrafterConfig:
    kw = dict(DRAFTER_PRESETS[name])
    kw.update(overrides)
    return DrafterConfig(**kw)


def preset(name: str, **overrides) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}")
    kw = dict(PRESETS[name])
    kw.update(overrides)
    return ModelConfig(**kw)


def to_json(cfg) -> str:
    return json.dumps(dataclasses.asdict(cfg), indent=1, sort_keys=True)


def from_json(cls, text: str):
    data = json.loads(text)
    names = {f.name for f in dataclasses.fields(cls)}
    unknown = set(data) - names
    if unknown:
        raise ValueError(f"{cls.__name__}: unknown keys {sorted(unknown)}")
    for f in dataclasses.fields(cls):
        if f.name in data and isinstance(data[f.name], list) and "tuple" in str(f.type):
            data[f.name] = tuple(data[f.name])
    return cls(**data)


def _parse(value: str, typ: Any, key: str):
    t = str(typ)
    if t in ("bool", "<class 'bool'>"):
        if value not in ("0", "1"):
            raise ValueError(f"{key}={value!r}: boolean flags take 0 or 1")
        return value == "1"
    if t in ("int", "<class 'int'>"):
        return int(value)
    if t in ("float", "<class 'float'>"):
        return float(value)
    if t in ("str", "<class 'str'>"):
        return value
    raise ValueError(f"{key}: cannot override a field of type {t} from the environment")


def apply_env_overrides(cfg, section: str, environ: dict[str, str] | None = None):
    """Return a copy of ``cfg`` with ``AFB_<SECTION>_<FIELD>`` variables applied (strict)."""
    environ = os.environ if environ is None else environ
    prefix = f"AFB_{section.upper()}_"
    fields = {f.name.upper(): f for f in dataclasses.fields(cfg)}
    updates = {}
    for key, value in environ.items():
        if not key.startswith(prefix):
            continue
        fname = key[len(prefix):]
        if fname not in fields:
            raise ValueError(f"{key}: {type(cfg).__name__} has no field {fname.lower()!r}")
        f = fields[fname]
        updates[f.name] = _parse(value, f.type, key)
    return dataclasses.replace(cfg, **updates) if updates else cfg


__all__ = ["ModelConfig", "DrafterConfig", "ServeConfig", "QADConfig", "PRESETS", "preset", "drafter_preset",
           "to_json", "from_json",
           "apply_env_overrides", "LINEAR", "FULL", "field"]
