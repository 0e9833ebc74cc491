"""B200-native GLM-5.3-Flash MoE block (drop-in for kg36/livglm's ExpertSSDMoE)."""

from .config import CONFIGS, ContractError, MoEConfig
from .moe import DenseMLP, ExpertSSDMoE, ResidentExperts, TopKRouter, build_layer

__all__ = [
    "CONFIGS", "ContractError", "MoEConfig", "DenseMLP", "ExpertSSDMoE", "ResidentExperts",
    "TopKRouter", "build_layer",
]
