"""MoE layer modules with the reference's forward signatures and checkpoint names, on the B200 kernels.

* ``Router(config, layer_id).forward(hidden_states, router_states=None) -> (weights fp32 [T, k], ids int32 [T, k],
  hidden_states_next)`` — servers/sgl/src/zonos3_sgl/models/zonos3.py:787-828 (linear router, quantile balancing:
  top-k of logits - balancing_biases; weights = softmax over the selected logits with
  ZONOS3_USE_TRAINING_ROUTER_WEIGHTS, else the selected entries of the full softmax). One fused kernel
  (zb_moe_router) computes rmsnorm_eda, the router GEMM, the selection and the weights.
* ``FusedGroupedExperts(config, layer_id).forward(x, router_logits=None, *, topk_weights, topk_ids)`` —
  zonos3.py:450-637 + FusedMoE.forward (layers/moe/fused_moe/layer.py:132-177): renormalisation
  (norm_topk_prob), permutation, gather, tcgen05 grouped GEMMs with SwiGLU / routing weight, combine.
  Checkpoints: gate_up_proj [E, 2I, D] (or w1 / w3, or SonicMoE's interleaved w13) and down_proj [E, D, I] (or w2).
* ``MoEFeedForward(config, layer_id).forward(x, router_states=None) -> (out, router_states_next)`` — zonos3.py:853-882.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops
from .base import BaseOP, Weight, _key


class Router(BaseOP):
    _fp32 = ("balancing_biases",)

    def __init__(self, config, layer_id: int):
        if getattr(config, "moe_router_type", "linear") != "linear" or getattr(config, "moe_router_use_eda", False):
            raise ValueError("the B200 router implements the release's linear router without EDA")
        self.hidden_size = config.hidden_size
        self.num_experts = config.moe_n_experts
        self.top_k = config.get_num_experts_per_tok(layer_id)
        self._eps = config.rms_norm_eps
        self._training_weights = bool(getattr(config, "use_training_router_weights", True))
        self._layer_id = layer_id
        self.router_linear = Weight((self.num_experts, self.hidden_size))
        self.rmsnorm_eda = Weight((self.hidden_size,))
        self.balancing_biases = torch.zeros(self.num_experts, dtype=torch.float32)

    def forward(self, hidden_states: torch.Tensor, router_states: torch.Tensor | None = None, *, ids=None,
                weights=None, logits=None, renormalize: bool = False):
        """``renormalize``: divide the k weights by their sum + 1e-8 in the router kernel (the experts' own
        renormalisation, fused by MoEFeedForward); the reference's Router returns them unnormalised."""
        ids, w = ops.moe_router(
            hidden_states, self.rmsnorm_eda.weight, self._eps, self.router_linear.weight, self.balancing_biases,
            self.top_k, weights="selected_softmax" if self._training_weights else "full_softmax",
            renormalize=renormalize, ids=ids, topk_weights=weights, logits=logits)
        # the states the next layer's EDA would blend in; the release routes without EDA, so no copy is made
        return w, ids, hidden_states


class FusedGroupedExperts(BaseOP):
    def __init__(self, config, layer_id: int):
        self.num_experts = config.moe_n_experts
        self.hidden_size = config.routed_dim
        self.intermediate_size = config.moe_intermediate_size
        self.top_k = config.get_num_experts_per_tok(layer_id)
        self._renormalize = bool(getattr(config, "norm_topk_prob", True))
        self.gate_up_proj = torch.empty(self.num_experts, 2 * self.intermediate_size, self.hidden_size)
        self.down_proj = torch.empty(self.num_experts, self.hidden_size, self.intermediate_size)
        self._workspaces: dict = {}

    def load_state_dict(self, state_dict, *, prefix: str = "", _internal: bool = False) -> None:
        """gate_up_proj / down_proj directly, from unfused w1 / w3 / w2, or from SonicMoE's interleaved w13
        (zonos3.py:552-618): the same formats the reference accepts."""
        gu, dn = _key(prefix, "gate_up_proj"), _key(prefix, "down_proj")
        w1, w2, w3, w13 = (_key(prefix, n) for n in ("w1.weight", "w2.weight", "w3.weight", "w13"))
        if gu not in state_dict and w13 in state_dict:
            inter = state_dict.pop(w13)
            state_dict[gu] = torch.cat([inter[:, 0::2, :], inter[:, 1::2, :]], dim=1)
        elif gu not in state_dict and w1 in state_dict and w3 in state_dict:
            state_dict[gu] = torch.cat([state_dict.pop(w1), state_dict.pop(w3)], dim=1)
        if dn not in state_dict:
            for alt in (_key(prefix, "w2"), w2):
                if alt in state_dict:
                    state_dict[dn] = state_dict.pop(alt)
                    break
        super().load_state_dict(state_dict, prefix=prefix, _internal=_internal)

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor | None = None, *, topk_weights=None,
                topk_ids=None, out=None, weights_normalized: bool = False) -> torch.Tensor:
        if topk_weights is None or topk_ids is None:
            if router_logits is None:
                raise ValueError("router_logits must be provided when top-k routing is not precomputed.")
            topk_ids, topk_weights = ops.moe_select(router_logits.contiguous(), None, self.top_k,
                                                    weights="full_softmax", renormalize=self._renormalize)
        else:
            topk_weights = topk_weights.to(torch.float32)
            if self._renormalize and not weights_normalized:
                topk_weights = topk_weights / (topk_weights.sum(dim=-1, keepdim=True) + 1e-8)
        topk_ids = topk_ids.to(torch.int32).contiguous()
        ws = ops.MoEWorkspace.for_shape(self._workspaces, x.shape[0], topk_ids.shape[1], self.num_experts,
                                        self.hidden_size, self.intermediate_size, x.device)
        return ops.moe_experts(x.contiguous(), self.gate_up_proj, self.down_proj, topk_ids,
                               topk_weights.contiguous(), ws, out=out)


class MoEFeedForward(BaseOP):
    def __init__(self, config, layer_id: int):
        self.router = Router(config, layer_id)
        self.hidden_size = config.hidden_size
        self.routed_dim = config.routed_dim
        self.use_latent_moe = self.routed_dim < self.hidden_size
        self.experts = FusedGroupedExperts(config, layer_id)
        if self.use_latent_moe:
            self.latent_down = Weight((self.routed_dim, self.hidden_size))
            self.latent_up = Weight((self.hidden_size, self.routed_dim))

    def forward(self, x: torch.Tensor, router_states: torch.Tensor | None = None):
        num_tokens, hidden = x.shape
        # the experts' renormalisation of the top-k weights runs inside the router kernel
        weights, ids, states_next = self.router.forward(x, router_states, renormalize=self.experts._renormalize)
        routed = F.linear(x, self.latent_down.weight) if self.use_latent_moe else x
        out = self.experts.forward(routed, topk_weights=weights, topk_ids=ids, weights_normalized=True)
        if self.use_latent_moe:
            out = F.linear(out, self.latent_up.weight)
        return out.view(num_tokens, hidden), states_next
