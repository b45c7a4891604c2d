"""The model-config fields the hot-path layers read (the reference's zonos3.models.config.ModelConfig,
model/src/zonos3/models/config.py: hidden_size, rms_norm_eps, the moe_* fields, get_routed_moe_dim :52,
get_num_experts_per_tok :180), plus the GDN head count / width that the release hard-codes (4 x 128,
servers/sgl/src/zonos3_sgl/models/gdn.py:136-141) and the BASELINE configs change (16 x 128, 4 x 64)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class ModelConfig:
    hidden_size: int
    num_layers: int = 1
    rms_norm_eps: float = 1e-5
    gdn_num_heads: int = 4
    gdn_head_dim: int = 128
    moe_n_experts: int = 64
    moe_topk: int = 8
    moe_intermediate_size: int = 768
    moe_alpha: float = 1.0
    norm_topk_prob: bool = True
    moe_router_type: str = "linear"
    moe_balancing_strategy: str = "quantile"
    moe_router_use_eda: bool = False
    moe_start_from_layer: int = 1
    use_training_router_weights: bool = True  # ZONOS3_USE_TRAINING_ROUTER_WEIGHTS=1 in the server's env.sh

    def get_num_experts_per_tok(self, layer_id: int) -> int:
        return self.moe_topk

    @property
    def routed_dim(self) -> int:
        return max(1, int(round(self.hidden_size * self.moe_alpha)))
