"""Host-side logic of the reference-mirroring API (no GPU)."""
import copy
import types

import pytest

from lagunalab_b200 import laguna
from lagunalab_b200.cache import DequantKVCache, make_quantized_cache

TINY = dict(
    model_type="laguna", vocab_size=100352, hidden_size=128, intermediate_size=256,
    num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
    rms_norm_eps=1e-6, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
    shared_expert_intermediate_size=64, norm_topk_prob=True, mlp_only_layers=[0],
    gating="per-head", moe_routed_scaling_factor=2.5, rope_parameters={"rope_theta": 1e6},
    decoder_sparse_step=1,
)


@pytest.mark.parametrize("bad", [
    {"moe_router_logit_softcapping": 30.0},
    {"swa_attention_sink_enabled": True},
    {"moe_apply_router_weight_on_input": True},
    {"gating": False},
])
def test_unsupported_config_raises(bad):
    with pytest.raises(ValueError):
        laguna.ModelArgs.from_dict({**copy.deepcopy(TINY), **bad})


def test_from_dict_ignores_unknown_keys_and_fills_defaults():
    a = laguna.ModelArgs.from_dict(copy.deepcopy(TINY))
    assert a.layer_types == ["full_attention"] * 4
    assert a.num_attention_heads_per_layer == [4] * 4
    assert a.rope_for("full_attention") == {"rope_theta": 1e6}


def _model(head_dim):
    return types.SimpleNamespace(args=laguna.ModelArgs.from_dict({**TINY, "head_dim": head_dim}))


def test_quantized_cache_rejects_indivisible_head_dim():
    with pytest.raises(ValueError, match="head_dim"):
        make_quantized_cache(_model(16), 8)


def test_fused_decode_needs_8bit():
    with pytest.raises(ValueError, match="8-bit"):
        make_quantized_cache(_model(128), 4, fused_decode=True)


def test_cache_has_no_bits_attribute_before_a_quantized_step():
    c = DequantKVCache(bits=8, quantized_decode=True)
    assert not hasattr(c, "bits") and c.kv_bits == 8 and c.group_size == 64
    assert c.empty() and c.nbytes == 0 and c.offset == 0


def test_layout_follows_layer_types():
    caches = make_quantized_cache(_model(128), bits=4)
    assert len(caches) == 4 and all(isinstance(c, DequantKVCache) for c in caches)
    assert all(c.kv_bits == 4 and not hasattr(c, "bits") for c in caches)
