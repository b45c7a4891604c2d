"""The model-config fields the hot-path layers read (the reference's zonos3.models.config.ModelConfig,
model/src/zonos3/models/config.py: hidden_size, rms_norm_eps, the moe_* fields, get_routed_moe_dim :52,
get_num_experts_per_tok :180; the attention, vocabulary and soft-cap fields :82-106, audio_vocab_size :176), plus
the GDN head count / width that the release hard-codes (4 x 128, servers/sgl/src/zonos3_sgl/models/gdn.py:136-141)
and the benchmark configs change (16 x 128, 4 x 64)."""

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
    # layer pattern: "gdnN_global1" = N gated-DeltaNet layers then one global-attention layer, repeated
    # (TransformerBlock, servers/sgl/src/zonos3_sgl/models/zonos3.py:896-899); "global" = attention everywhere
    attention_pattern: str = "gdn3_global1"
    num_qo_heads: int = 16
    num_kv_heads: int = 4
    head_dim: int = 128
    rope_theta: float = 10000.0
    intermediate_size: int = 0  # dense FFN width of the layers before moe_start_from_layer
    n_codebooks: int = 9
    codebook_size: int = 1024
    text_vocab: int | None = None
    text_extra_tokens: int = 0
    audio_pad_id: int = 1025
    loss_softcap: float = 15.0

    def get_num_experts_per_tok(self, layer_id: int) -> int:
        return self.moe_topk

    @property
    def routed_dim(self) -> int:
        return max(1, int(round(self.hidden_size * self.moe_alpha)))

    @property
    def audio_vocab_size(self) -> int:
        """Codes 0..codebook_size-1, the end-of-audio id, then the pad id (config.py:58-60, :176)."""
        return self.codebook_size + 2

    def uses_gdn(self, layer_id: int) -> bool:
        """gdnN_global1: every (N + 1)-th layer is global attention, the others gated DeltaNet."""
        pattern = self.attention_pattern
        if pattern == "global":
            return False
        if pattern.startswith("gdn") and pattern.endswith("_global1"):
            period = int(pattern[3:-len("_global1")]) + 1
            return (layer_id + 1) % period != 0
        raise ValueError(f"unsupported attention_pattern {pattern!r}")

    def is_moe(self, layer_id: int) -> bool:
        return layer_id >= self.moe_start_from_layer
