"""zonos3-mini B200: the ZONOS3-Mini LM-backbone hot path (gated DeltaNet, MoE router + SwiGLU experts, Full
AttnRes) as hand-written sm_100a CUDA kernels behind a C ABI, with host modules that keep the reference layers'
forward signatures.

The directory name is not a Python identifier, so it is imported under the alias ``zonos3_mini_b200``
(``__graft_entry__.load_package`` registers it).
"""

from . import _lib, attention, attnres, base, config, core, gdn, model, moe, ops, replicas, vocoder  # noqa: F401

__all__ = ["attention", "attnres", "base", "config", "core", "gdn", "model", "moe", "ops", "replicas", "vocoder"]
