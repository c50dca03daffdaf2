"""arc_forge_2026_b200: a Blackwell-native (sm_100a) framework for hybrid-MoE compression, QAD training and
speculative serving, with the capabilities of ARC-Forge-2026.

Subpackages: ``models`` (reference oracle + GPU inference model + DFlash drafter), ``ops`` (CUDA kernels as
Python ops), ``parallel`` (symmetric memory, fused EP collectives, NCCL baselines), ``quant`` (uint3 g128,
GPTQ, block FP8, saliency/pruning), ``train`` (QAD, RL deltas, losses, optimizers), ``serve`` (engine,
scheduler, spec decode, HiSparse host KV, OpenAI server), ``formats`` (checkpoint and artefact formats),
``utils`` (timing, IO, env flags).
"""
from .config import DrafterConfig, ModelConfig, QADConfig, ServeConfig, preset

__version__ = "0.1.0"
__all__ = ["ModelConfig", "DrafterConfig", "ServeConfig", "QADConfig", "preset", "__version__"]
