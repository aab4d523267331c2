"""Host-side logic of the CUDA backend that needs no GPU: the model shape, weight naming, the
host quantizer, and the CUDA target's reading of the reference's own graphs."""

from __future__ import annotations

import numpy as np
import pytest

from nanocompile_b200 import quantize as q
from nanocompile_b200.model import QWEN2_0_5B, SMALL, TINY, ModelShape, synthetic_cache, synthetic_prompt, synthetic_weights


def test_shape_from_a_config_and_derived_sizes():
    fields = {"vocab_size": 151936, "hidden_size": 896, "intermediate_size": 4864, "num_hidden_layers": 24,
              "num_attention_heads": 14, "num_key_value_heads": 2, "rms_norm_eps": 1e-6, "rope_theta": 1e6,
              "tie_word_embeddings": True}
    assert ModelShape.of(fields) == QWEN2_0_5B
    assert QWEN2_0_5B.q_rows == 896 and QWEN2_0_5B.kv_rows == 128 and QWEN2_0_5B.attention_scale == np.float32(0.125)
    with pytest.raises(NotImplementedError, match="tied"):
        ModelShape.of(fields | {"tie_word_embeddings": False})
    with pytest.raises(ValueError):
        ModelShape(256, 64, 128, 2, 3, 2, 16)
    assert ModelShape(**{k: getattr(TINY, k) for k in TINY.__dataclass_fields__}) == TINY


def test_weight_shapes_name_every_array():
    w = TINY.weight_shapes(quantized=True)
    assert w["model.layers.0.self_attn.q_proj.weight@int8"] == ("int8", (64, 64))
    assert w["model.layers.1.mlp.down_proj.weight@scales"] == ("float32", (64,))
    assert "model.embed_tokens.weight" in w and "model.layers.0.self_attn.q_proj.weight" not in w
    assert "model.layers.0.self_attn.q_proj.weight" in TINY.weight_shapes(quantized=False)


def test_weight_shapes_match_the_reference_graph(reference):
    """The arrays a step reads, by name, dtype and shape, are the reference graph's."""
    from nanocompile import quantize as rq
    from nanocompile.models.qwen2 import Qwen2Config, build_qwen2

    for quantized in (False, True):
        graph = build_qwen2(Qwen2Config(**TINY.config_fields()), last_only=True)
        if quantized:
            graph = rq.quantize(graph, "int8", keep=("lm_head.weight",))
        theirs = {n: (node.dtype.numpy.name, tuple(node.shape)) for n, node in graph.weights.items()}
        assert TINY.weight_shapes(quantized) == theirs


def test_int8_projection_weights_quantize_the_projections_only():
    w = synthetic_weights(TINY, seed=0)
    out = q.int8_projection_weights(w, TINY)
    assert set(out) == set(TINY.weight_shapes(quantized=True))
    name = "model.layers.0.mlp.gate_proj.weight"
    values, scales = q.quantize_int8(w[name])
    assert np.array_equal(out[q.int8_name(name)], values) and np.array_equal(out[q.scales_name(name)], scales)
    assert out["model.embed_tokens.weight"] is w["model.embed_tokens.weight"]
    assert q.int8_projection_weights(out, TINY).keys() == out.keys()          # already quantized: kept
    with pytest.raises(KeyError):
        q.int8_projection_weights({}, TINY)


def test_int8_projection_weights_are_the_references(reference):
    """The host quantizer's bytes are the reference's ``quantized_weights`` of its own graph."""
    from nanocompile import quantize as rq
    from nanocompile.models.qwen2 import Qwen2Config, build_qwen2

    w = synthetic_weights(TINY, seed=2)
    graph = rq.quantize(build_qwen2(Qwen2Config(**TINY.config_fields())), "int8", keep=("lm_head.weight",))
    theirs = rq.quantized_weights(graph, w)
    mine = q.int8_projection_weights(w, TINY)
    assert theirs.keys() == mine.keys()
    for name in theirs:
        assert np.array_equal(np.asarray(theirs[name]).view(np.uint8), np.asarray(mine[name]).view(np.uint8)), name


def test_synthetic_inputs_are_deterministic():
    a, b = synthetic_weights(TINY, seed=3), synthetic_weights(TINY, seed=3)
    assert all(np.array_equal(a[k], b[k]) for k in a)
    assert synthetic_prompt(256, 8) == synthetic_prompt(256, 8)
    k1, v1, t1 = synthetic_cache(TINY, 5, 7)
    k2, v2, t2 = synthetic_cache(TINY, 5, 7)
    assert np.array_equal(k1, k2) and np.array_equal(v1, v2) and t1 == t2 and k1.shape == (2, 2, 7, 16)


# -- the CUDA target over the reference's graphs ---------------------------------------------------


def _graph(shape: ModelShape, activations, last_only=True, **kwargs):
    from nanocompile import quantize as rq
    from nanocompile.models.qwen2 import Qwen2Config, build_qwen2

    graph = build_qwen2(Qwen2Config(**(shape.config_fields() | kwargs)), last_only=last_only)
    if activations is not None:
        graph = rq.quantize(graph, activations, keep=("lm_head.weight",))
    return graph


@pytest.mark.parametrize("activations", [None, "int8", "f32"])
@pytest.mark.parametrize("last_only", [True, False])
def test_target_reads_the_step_off_the_reference_graph(reference, activations, last_only):
    from nanocompile_b200.target import lower_cuda

    cuda = lower_cuda(_graph(TINY, activations, last_only))
    assert cuda.shape == TINY and cuda.activations == activations and cuda.last_only == last_only
    assert np.array_equal(cuda.rope_rates.view(np.uint32), TINY.rope_rates().view(np.uint32))
    covered = sorted(c for g in cuda.groups for c in g.calls)
    assert covered == list(range(cuda.calls))                         # every reference call is in one group
    kinds = {g.kind for g in cuda.groups}
    assert {"gather", "rms_norm", "qkv_projection", "attention", "o_projection", "gate_up_projection",
            "down_projection", "lm_head", "kv_output", "rope"} <= kinds
    assert ("block_quantize" in kinds) == (activations == "int8")
    for layer in range(TINY.layers):
        calls = [c for g in cuda.groups if g.layer == layer and g.kind == "gate_up_projection" for c in g.calls]
        assert len(calls) == 1                                       # gate and up in one fused call
    assert "matmul_i8_vnni" in cuda.source() if activations == "int8" else True


def test_target_reads_the_05b_graph_and_its_rates(reference):
    from nanocompile_b200.target import lower_cuda

    cuda = lower_cuda(_graph(QWEN2_0_5B, "int8"))
    assert cuda.shape == QWEN2_0_5B and cuda.calls > 24 * 30
    assert np.array_equal(cuda.rope_rates.view(np.uint32), QWEN2_0_5B.rope_rates().view(np.uint32))
    other = lower_cuda(_graph(SMALL, "int8", rope_theta=10000.0))      # another theta: its own rates
    assert np.array_equal(other.rope_rates, ModelShape(**{**SMALL.__dict__, "theta": 10000.0}).rope_rates())


def test_target_refuses_what_the_kernels_do_not_implement(reference):
    from nanocompile import quantize as rq
    from nanocompile.models.qwen2 import Qwen2Config, build_qwen2
    from nanocompile.frontend import GraphBuilder
    from nanocompile import dtypes

    from nanocompile_b200.target import TargetError, lower_cuda

    with pytest.raises(TargetError, match="tied"):
        lower_cuda(build_qwen2(Qwen2Config(**(TINY.config_fields() | {"tie_word_embeddings": False}))))
    coarse = rq.quantize(build_qwen2(Qwen2Config(**TINY.config_fields())), "int8", block=64, keep=("lm_head.weight",))
    with pytest.raises(TargetError, match="line"):
        lower_cuda(coarse)                                            # block-64 activation scales
    b = GraphBuilder("not_qwen2")
    seq = b.symbol("seq")
    x = b.input("x", dtypes.f32, (seq, 4))
    with pytest.raises(TargetError, match="token_ids"):
        lower_cuda(b.build({"y": x * x}))


def test_compiled_graph_without_a_gpu_lowers_and_lists_the_program(reference):
    from nanocompile_b200.runtime import CUDABackend

    backend = CUDABackend()
    graph = _graph(TINY, "int8")
    compiled = backend.compiled(graph)
    assert backend.compiled(graph) is compiled                        # once per graph, as CBackend
    assert compiled.program.calls and compiled.cached and compiled.compile_seconds > 0
    assert "gate_up_projection" in compiled.source and "model.layers.1.mlp.down_proj.weight@int8" in compiled.source
