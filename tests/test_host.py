"""Host-side logic of the CUDA backend that needs no GPU: config, step description,
weights naming, argument checks, the host KV cache."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

from nanocompile_b200 import quantize as q
from nanocompile_b200.qwen2 import (QWEN2_0_5B, TINY, KVCache, Qwen2Config, build_qwen2, quantize, synthetic_cache,
                                    synthetic_prompt, synthetic_weights)
from nanocompile_b200.runtime import InterpreterError, check_arguments

REFERENCE = Path(os.environ.get("NANOCOMPILE_REFERENCE", "/root/reference"))


def test_config_from_dict_and_derived_sizes():
    c = Qwen2Config.from_dict({"architectures": ["Qwen2ForCausalLM"], "vocab_size": 151936, "hidden_size": 896,
                               "intermediate_size": 4864, "num_hidden_layers": 24, "num_attention_heads": 14,
                               "num_key_value_heads": 2, "rms_norm_eps": 1e-6, "rope_theta": 1e6,
                               "tie_word_embeddings": True})
    assert c == QWEN2_0_5B and c.head_dim == 64 and c.kv_group_size == 7
    with pytest.raises(ValueError, match="not a Qwen2 config"):
        Qwen2Config.from_dict({"architectures": ["Llama"]})
    with pytest.raises(ValueError):
        Qwen2Config(256, 64, 128, 2, 3, 2, 1e-6, 1e6, True)


def test_weight_names_and_shapes():
    g = quantize(build_qwen2(TINY, last_only=True), "int8", keep=("lm_head.weight",))
    w = g.weights
    assert w["model.layers.0.self_attn.q_proj.weight@int8"] == (np.dtype(np.int8), (64, 64))
    assert w["model.layers.1.mlp.down_proj.weight@scales"] == (np.dtype(np.float32), (64,))
    assert "model.embed_tokens.weight" in w and "model.layers.0.self_attn.q_proj.weight" not in w
    assert g.name == "qwen2_last"
    f = build_qwen2(TINY)
    assert "model.layers.0.self_attn.q_proj.weight" in f.weights and f.name == "qwen2"


@pytest.mark.skipif(not REFERENCE.exists(), reason="the reference checkout is not present")
def test_weight_list_matches_the_reference_graph():
    """The weights a step reads, by name, dtype and shape, are the reference graph's."""
    sys.path.insert(1, str(REFERENCE))
    from nanocompile import quantize as rq
    from nanocompile.models.qwen2 import Qwen2Config as RC, build_qwen2 as rbuild

    rc = RC(*[getattr(TINY, f) for f in TINY.__dataclass_fields__])
    for activations in (None, "int8"):
        ref = rbuild(rc, last_only=True)
        mine = build_qwen2(TINY, last_only=True)
        if activations:
            ref = rq.quantize(ref, activations, keep=("lm_head.weight",))
            mine = quantize(mine, activations, keep=("lm_head.weight",))
        theirs = {n: (node.dtype.numpy, tuple(node.shape)) for n, node in ref.weights.items()}
        assert {n: (np.dtype(d), s) for n, (d, s) in mine.weights.items()} == \
               {n: (np.dtype(d), s) for n, (d, s) in theirs.items()}


def test_quantized_weights_make_int8_and_scales():
    g = quantize(build_qwen2(TINY), "int8", keep=("lm_head.weight",))
    w = synthetic_weights(TINY, seed=0)
    out = q.quantized_weights(g, w)
    assert set(out) == set(g.weights)
    name = "model.layers.0.mlp.gate_proj.weight"
    values, scales = q.quantize_int8(w[name])
    assert np.array_equal(out[q.int8_name(name)], values) and np.array_equal(out[q.scales_name(name)], scales)
    with pytest.raises(KeyError):
        q.quantized_weights(g, {})


def test_synthetic_inputs_are_deterministic():
    a, b = synthetic_weights(TINY, seed=3), synthetic_weights(TINY, seed=3)
    assert all(np.array_equal(a[k], b[k]) for k in a)
    assert synthetic_prompt(256, 8) == synthetic_prompt(256, 8)
    k1, v1, t1 = synthetic_cache(TINY, 5, 7)
    k2, v2, t2 = synthetic_cache(TINY, 5, 7)
    assert np.array_equal(k1, k2) and np.array_equal(v1, v2) and t1 == t2 and k1.shape == (2, 2, 7, 16)


def test_check_arguments_uses_the_interpreters_messages():
    g = build_qwen2(TINY, last_only=True)
    w = synthetic_weights(TINY, seed=0)
    zeros = np.zeros((2, 2, 3, 16), np.float32)
    ids = np.array([1, 2], np.int64)
    assert check_arguments(g, {"token_ids": ids, "past_keys": zeros, "past_values": zeros}, w) == {"seq": 2, "past": 3}
    with pytest.raises(InterpreterError, match="missing"):
        check_arguments(g, {"token_ids": ids}, w)
    with pytest.raises(InterpreterError, match="already bound"):
        check_arguments(g, {"token_ids": ids, "past_keys": zeros, "past_values": zeros[:, :, :2]}, w)
    with pytest.raises(InterpreterError, match="expected i64"):
        check_arguments(g, {"token_ids": ids.astype(np.int32), "past_keys": zeros, "past_values": zeros}, w)
    with pytest.raises(InterpreterError, match="missing weights"):
        check_arguments(g, {"token_ids": ids, "past_keys": zeros, "past_values": zeros}, {})


def test_host_kv_cache_growth_preserves_contents():
    cache = KVCache(TINY, capacity=2)
    rng = np.random.default_rng(0)
    chunks = [rng.standard_normal((2, 2, n, 16)).astype(np.float32) for n in (1, 3, 2)]
    for c in chunks:
        cache.append(c, -c)
    keys, values = cache.past()
    assert np.array_equal(keys, np.concatenate(chunks, 2)) and np.array_equal(values, -keys)
    assert cache.capacity >= 6
