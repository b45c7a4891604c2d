"""Host side of the whole-model module (CPU): the checkpoint names and shapes of Zonos3ForCausalLM equal those of
the oracle LM (and so the reference's lm.py module tree) at the cfg5 and cfg1 shapes, loading is strict, the layer
pattern follows gdnN_global1, and the bench's algorithmic-byte count adds up."""

from __future__ import annotations

import pytest
import torch

from oracle import lm as olm


def _pair(zb, layers, moe_start=0):
    mc = zb.config.ModelConfig(hidden_size=2048, num_layers=layers, gdn_num_heads=16, gdn_head_dim=128,
                               moe_n_experts=64, moe_topk=8, moe_intermediate_size=768, moe_start_from_layer=moe_start,
                               intermediate_size=4096, n_codebooks=10, codebook_size=4096, text_vocab=8192,
                               audio_pad_id=4097)
    oc = olm.LMConfig(dim=2048, n_layers=layers, gdn_period=4, gdn_heads=16, gdn_head_dim=128, n_heads=16,
                      n_kv_heads=4, head_dim=128, n_experts=64, topk=8, moe_hidden=768, moe_routed_dim=2048,
                      n_codebooks=10, codebook_size=4096, text_rows=8193, dense_first_layer=moe_start > 0,
                      ffn_hidden=4096)
    return mc, oc


@pytest.mark.parametrize("layers,moe_start", [(8, 0), (4, 1)])
def test_checkpoint_names_match_the_reference_module_tree(zb, layers, moe_start):
    mc, oc = _pair(zb, layers, moe_start)
    with torch.device("meta"):
        model = zb.model.Zonos3ForCausalLM(mc)
    got = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    want = {k: tuple(v) for k, v in olm.weight_shapes(oc).items()}
    assert got == want


def test_strict_load_and_layer_pattern(zb):
    mc = zb.config.ModelConfig(hidden_size=64, num_layers=8, gdn_num_heads=2, gdn_head_dim=32, moe_n_experts=4,
                               moe_topk=2, moe_intermediate_size=128, moe_start_from_layer=0, num_qo_heads=4,
                               num_kv_heads=2, head_dim=16, n_codebooks=2, codebook_size=16, text_vocab=8,
                               audio_pad_id=17)
    model = zb.model.Zonos3ForCausalLM(mc)
    kinds = [type(layer.attention).__name__ for layer in model.layers.op_list]
    assert kinds == ["OriginalGDN"] * 3 + ["Attention"] + ["OriginalGDN"] * 3 + ["Attention"]
    assert model.attention_layer_ids() == [3, 7]
    state = {k: torch.zeros_like(v) for k, v in model.state_dict().items()}
    model.load_state_dict(dict(state))
    with pytest.raises(RuntimeError, match="Unexpected keys"):
        model.load_state_dict({**state, "speaker_projection.weight": torch.zeros(1)})
    assert zb.config.ModelConfig(hidden_size=8, attention_pattern="gdn2_global1").uses_gdn(2) is False


def test_decode_step_bytes(zb):
    import bench

    inner = 16 * 128
    per_gdn_state = 256 * 16 * 128 * 128 * 4 * 2
    total = bench.cfg5_step_bytes(256, 878)
    experts = 24 * 64 * 3 * 768 * 2048 * 2
    kv = 6 * 256 * 879 * 4 * 128 * 2 * 2
    assert experts + 18 * per_gdn_state + kv < total < experts + 18 * per_gdn_state + kv + 3e9
    # one more cached key per stream adds its K and V rows in the 6 GQA layers and its page-table entry
    assert bench.cfg5_step_bytes(256, 879) - total == 6 * 256 * (4 * 128 * 2 * 2 + 4)
    assert inner == 2048


def test_prefill_layout_and_chunk_tables(zb):
    """PrefillLayout.build([1, 0, 2]) lays requests out as 128, 64 and 192 padded rows; chunk_tables gives the
    reference's cu_seqlens and (sequence, chunk) indices (servers/sgl/src/zonos3_sgl/models/gdn.py:49-59)."""
    layout = zb.gdn.PrefillLayout.build([1, 0, 2], "cpu")
    assert layout.rows == 384
    assert layout.starts.tolist() == [0, 128, 192] and layout.cu_seqlens.tolist() == [0, 128, 192, 384]
    assert layout.seq_of_token.tolist() == [0] * 128 + [1] * 64 + [2] * 192
    assert layout.row_in_seq.tolist() == list(range(128)) + list(range(64)) + list(range(192))
    assert layout.fresh.tolist() == [1, 1, 1] and len(layout.tensors()) == 5
    cu, chunks = zb.gdn.chunk_tables([70, 2, 129], "cpu")
    assert cu.tolist() == [0, 70, 72, 201]
    assert chunks.tolist() == [[0, 0], [0, 1], [1, 0], [2, 0], [2, 1], [2, 2]]
