"""MoE geometry with the reference's field names.

Mirrors the MoE fields of GLMTextConfig (kg36/livglm
src/glm53flash/model_config.py:11-54) and the checks of its validate()
(model_config.py:142-176) that concern the MoE block.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any


class ContractError(ValueError):
    """Inputs do not satisfy the MoE block's contract (kg36/livglm contract.py:54-55)."""


@dataclass(frozen=True)
class MoEConfig:
    hidden_size: int
    moe_intermediate_size: int
    n_routed_experts: int
    num_experts_per_tok: int
    n_shared_experts: int = 1
    n_group: int = 1
    topk_group: int = 1
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 2.5
    swiglu_limit: float = 10.0
    scoring_func: str = "sigmoid"
    topk_method: str = "noaux_tc"
    hidden_act: str = "silu"

    @classmethod
    def from_text_config(cls, text: dict[str, Any]) -> "MoEConfig":
        """Build from the checkpoint's `text_config` dict (model_config.py:56-140)."""

        def integer(key: str) -> int:
            value = text.get(key)
            if isinstance(value, bool) or not isinstance(value, int):
                raise ContractError(f"configuration field must be an integer: {key}")
            return value

        def number(key: str) -> float:
            value = text.get(key)
            if isinstance(value, bool) or not isinstance(value, (int, float)):
                raise ContractError(f"configuration field must be numeric: {key}")
            return float(value)

        result = cls(
            hidden_size=integer("hidden_size"),
            moe_intermediate_size=integer("moe_intermediate_size"),
            n_routed_experts=integer("n_routed_experts"),
            num_experts_per_tok=integer("num_experts_per_tok"),
            n_shared_experts=integer("n_shared_experts"),
            n_group=integer("n_group"),
            topk_group=integer("topk_group"),
            norm_topk_prob=bool(text.get("norm_topk_prob")),
            routed_scaling_factor=number("routed_scaling_factor"),
            swiglu_limit=number("swiglu_limit"),
            scoring_func=str(text.get("scoring_func")),
            topk_method=str(text.get("topk_method")),
            hidden_act=str(text.get("hidden_act")),
        )
        result.validate()
        return result

    @classmethod
    def from_model_dict(cls, config: dict[str, Any]) -> "MoEConfig":
        text = config.get("text_config")
        if not isinstance(text, dict):
            raise ContractError("config has no text_config object")
        return cls.from_text_config(text)

    def validate(self) -> "MoEConfig":
        if self.hidden_act != "silu":
            raise ContractError(f"v1 supports only SiLU, got {self.hidden_act!r}")
        if self.scoring_func != "sigmoid" or self.topk_method != "noaux_tc":
            raise ContractError("v1 supports only sigmoid/noaux_tc routing")
        if not 1 <= self.num_experts_per_tok <= self.n_routed_experts:
            raise ContractError("invalid routed top-k geometry")
        if self.n_group < 1 or self.n_routed_experts % self.n_group:
            raise ContractError("expert count must be divisible by n_group")
        if not 1 <= self.topk_group <= self.n_group:
            raise ContractError("invalid topk_group")
        if self.n_routed_experts // self.n_group < 2:
            raise ContractError("router groups must contain at least two experts")
        if self.hidden_size % 32 or self.hidden_size <= 0:
            raise ContractError("hidden_size must be a positive multiple of the MXFP4 group (32)")
        if self.moe_intermediate_size % 32 or self.moe_intermediate_size <= 0:
            raise ContractError("expert width is not divisible by 32")
        if self.n_shared_experts < 0:
            raise ContractError("n_shared_experts must be >= 0")
        return self

    @property
    def shared_intermediate_size(self) -> int:
        return self.moe_intermediate_size * self.n_shared_experts

    def replace(self, **kw) -> "MoEConfig":
        return replace(self, **kw)


# The five workloads named by the benchmark plan.  swiglu_limit is GLM's 10.0.
CONFIGS: dict[str, MoEConfig] = {
    "cfg0": MoEConfig(hidden_size=256, moe_intermediate_size=128, n_routed_experts=16,
                      num_experts_per_tok=4, n_shared_experts=1, n_group=4, topk_group=2),
    "cfg1": MoEConfig(hidden_size=4096, moe_intermediate_size=1536, n_routed_experts=128,
                      num_experts_per_tok=8, n_shared_experts=1, n_group=8, topk_group=4),
}
CONFIGS["cfg2"] = CONFIGS["cfg1"]
CONFIGS["cfg3"] = CONFIGS["cfg1"]
CONFIGS["cfg4"] = CONFIGS["cfg1"]
# Real GLM-5.3-Flash routed geometry (kg36/livglm docs/v1-impl.md:118-135).
CONFIGS["glm53flash"] = MoEConfig(hidden_size=4096, moe_intermediate_size=2048,
                                  n_routed_experts=288, num_experts_per_tok=8,
                                  n_shared_experts=1, n_group=1, topk_group=1)
