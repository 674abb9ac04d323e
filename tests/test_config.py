"""Model specs from transformers configs, and the shape checks the kernels rely on (CPU)."""

from __future__ import annotations

import dataclasses

import pytest

from strands_decider_b200 import config


def _hf_config(spec):
    transformers = pytest.importorskip("transformers")
    return transformers.Qwen3_5TextConfig(
        vocab_size=spec.vocab, hidden_size=spec.hidden, intermediate_size=spec.inter,
        num_hidden_layers=spec.n_layers, num_attention_heads=spec.attn_heads,
        num_key_value_heads=spec.attn_kv_heads, head_dim=spec.head_dim,
        linear_num_key_heads=spec.gdn_heads, linear_num_value_heads=spec.gdn_heads,
        linear_key_head_dim=spec.gdn_dk, linear_value_head_dim=spec.gdn_dv,
        linear_conv_kernel_dim=spec.conv_width, layer_types=list(spec.layer_types), rms_norm_eps=spec.eps,
        tie_word_embeddings=True,
        rope_parameters={"rope_type": "default", "rope_theta": spec.rope_theta,
                         "partial_rotary_factor": spec.partial_rotary})


@pytest.mark.parametrize("spec", [config.TINY, config.REDUCED_1024, config.HYBRID_2B])
def test_spec_round_trips_through_a_transformers_config(spec):
    got = config.ModelSpec.from_hf_config(_hf_config(spec), weight_format=spec.weight_format, name=spec.name,
                                          max_positions=spec.max_positions)
    assert got == spec


def test_unsupported_shapes_are_refused():
    with pytest.raises(ValueError, match="GDN head dims"):
        dataclasses.replace(config.TINY, gdn_dk=64).validate()
    with pytest.raises(ValueError, match="head_dim"):
        dataclasses.replace(config.TINY, head_dim=96).validate()
    with pytest.raises(ValueError, match="conv width"):
        dataclasses.replace(config.TINY, conv_width=3).validate()
    cfg = _hf_config(config.TINY)
    cfg.linear_num_value_heads = 4
    with pytest.raises(ValueError, match="value head"):
        config.ModelSpec.from_hf_config(cfg)


def test_workload_shapes():
    w = config.HYBRID_2B_WORKLOAD
    assert (w.n_requests, w.state_len, w.n_questions, w.question_len) == (1024, (512, 512), 3, 32)
    p = config.PREFIX_CACHE_WORKLOAD
    assert (p.n_requests, p.state_len, p.n_questions, p.question_len, p.option_range) == (512, (64, 2048), 32, 48,
                                                                                          (2, 5))
    lat = config.LATENCY_WORKLOAD
    assert lat.state_len[0] + lat.question_len == 96 and lat.n_questions == 1
