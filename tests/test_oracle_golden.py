"""The CPU oracle pinned against the reference's own outputs (tests/golden, made by nanocompile's CBackend).

The oracle is what the GPU parity tests compare against, so before it is trusted it must
reproduce the reference bit for bit: every logit, every quantized activation, every key.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from nanocompile_b200 import quantize as q
from nanocompile_b200.model import QWEN2_0_5B, TINY, ModelShape, synthetic_weights
from oracle import oracle
from tests.conftest import bits, golden


def tiny_weights(activations):
    w = synthetic_weights(TINY, seed=0)
    if activations is None:
        return w
    return q.int8_projection_weights(w, TINY)


@pytest.mark.parametrize("tag,activations", [("fp32", None), ("vnni", "int8")])
def test_oracle_tiny_greedy_is_the_references_bitwise(tag, activations):
    g = golden("tiny")
    model = oracle.OracleModel(TINY, tiny_weights(activations), activations)
    tokens, logits = model.greedy(list(g["prompt"]), 16, return_logits=True)
    assert tokens == list(g[f"{tag}_tokens"])
    assert np.array_equal(bits(logits), bits(g[f"{tag}_logits"]))


@pytest.mark.parametrize("tag,activations", [("fp32", None), ("vnni", "int8")])
def test_oracle_tiny_full_and_chunked_passes(tag, activations):
    g = golden("tiny")
    model = oracle.OracleModel(TINY, tiny_weights(activations), activations)
    prompt = list(g["prompt"])
    zeros = np.zeros((TINY.layers, TINY.kv_heads, 0, TINY.head_dim), np.float32)
    full, keys, values = model.step(prompt, zeros, zeros, last_only=False)
    assert np.array_equal(bits(full), bits(g[f"{tag}_full_logits"]))
    assert np.array_equal(bits(keys), bits(g[f"{tag}_keys"]))
    assert np.array_equal(bits(values), bits(g[f"{tag}_values"]))
    first, k5, v5 = model.step(prompt[:5], zeros, zeros, last_only=False)
    rows = [first]
    pk, pv = k5, v5
    for t in prompt[5:]:
        lg, k, v = model.step([t], pk, pv, last_only=False)
        rows.append(lg)
        pk, pv = np.concatenate([pk, k], 2), np.concatenate([pv, v], 2)
    assert np.array_equal(bits(np.concatenate(rows)), bits(g[f"{tag}_chunked_logits"]))


def test_inverse_frequencies_are_the_references():
    assert np.array_equal(bits(TINY.rope_rates()), bits(golden("tiny")["inv_freq"]))
    assert np.array_equal(bits(QWEN2_0_5B.rope_rates()), bits(golden("qwen05b_vnni")["inv_freq"]))


def test_quantize_int8_is_the_references_byte_for_byte():
    g = golden("proj")
    values, scales = q.quantize_int8(g["qi8_w"])
    assert values.dtype == np.int8 and np.array_equal(values, g["qi8_values"])
    assert np.array_equal(bits(scales), bits(g["qi8_scales"]))
    assert scales[3] == 1.0 and not values[3].any()


WIDTHS = [(896, 72), (4864, 24), (160, 40), (96, 24)]


@pytest.mark.parametrize("k,n", WIDTHS)
@pytest.mark.parametrize("tokens", [1, 3, 7])
def test_oracle_projection_is_the_references_bitwise(k, n, tokens):
    """Quantized activations, scales, offset and output of one int8-vnni projection."""
    g = golden("proj")
    tag = f"k{k}_n{n}_t{tokens}"
    rng = np.random.default_rng(k + tokens)               # the fixture's weight, regenerated
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    values, scales = q.quantize_int8(w)
    assert np.array_equal(values, g[f"{tag}_q"]) and np.array_equal(bits(scales), bits(g[f"{tag}_scales"]))
    xq, xs, off, sums = oracle.quantize_blocks(g[f"{tag}_x"])
    assert np.array_equal(xq, g[f"{tag}_xq"].reshape(xq.shape))
    assert np.array_equal(bits(xs), bits(g[f"{tag}_xs"].reshape(xs.shape)))
    assert np.array_equal(bits(off), bits(g[f"{tag}_offset"].reshape(off.shape)))
    y, lanes = oracle.matmul_i8_vnni(xq, xs, off, values, scales, lanes=True)
    assert np.array_equal(bits(y), bits(g[f"{tag}_y"]))
    # the integer layer, independently of any float order: NumPy int64
    w64 = values.astype(np.int64) + 128
    x64 = xq.astype(np.int64)
    expect_lanes = np.einsum("nkj,mkj->mnk", w64.reshape(n, k // 4, 4), x64.reshape(tokens, k // 4, 4))
    assert np.array_equal(lanes, expect_lanes)
    assert np.array_equal(sums, x64.reshape(tokens, k // 32, 32).sum(-1))


def test_expf_restatement_is_glibc_on_a_sweep_of_floats():
    """The table-driven expf the kernels use gives glibc's bits (a strided sweep of all floats)."""
    u = np.arange(0, 2**32, 1021, dtype=np.uint64).astype(np.uint32)
    x = u.view(np.float32)
    x = x[np.isfinite(x)]
    x = np.concatenate([x, np.array([-np.inf, np.inf, np.nan, 0.0, -0.0, 88.72, -103.97, -103.9, 88.7], np.float32)])
    a, b = oracle.expf_libm(x), oracle.expf_restated(x)
    same = (bits(a) == bits(b)) | (np.isnan(a) & np.isnan(b))
    assert same.all(), x[~same][:5]


def sha1(a: np.ndarray) -> np.ndarray:
    return np.frombuffer(hashlib.sha1(np.ascontiguousarray(a).tobytes()).digest(), np.uint8)


@pytest.mark.slow
def test_oracle_05b_int8_vnni_first_steps_are_the_references(qwen05b_vnni_weights):
    g = golden("qwen05b_vnni")
    model = oracle.OracleModel(QWEN2_0_5B, qwen05b_vnni_weights, "int8", threads=8)
    tokens, logits = model.greedy(list(g["prompt"]), 2, return_logits=True)
    assert tokens == list(g["tokens"][:2])
    assert np.array_equal(bits(logits), bits(g["first_logits"]))
    assert all(np.array_equal(sha1(logits[i]), g["sha1"][i]) for i in range(2))


# -- int8 weights with float32 activations (matmul_i8, nanocompile/lower.py:320-356) ----------------

WIDTHS_I8 = [(896, 72), (4864, 24), (160, 40), (96, 24), (136, 16), (100, 8)]


@pytest.mark.parametrize("k,n", WIDTHS_I8)
@pytest.mark.parametrize("tokens", [1, 3, 7])
def test_oracle_int8_f32_projection_is_the_references_bitwise(k, n, tokens):
    g = golden("int8_f32")
    tag = f"k{k}_n{n}_t{tokens}"
    rng = np.random.default_rng(3 * k + tokens)          # the fixture's weight, regenerated
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    values, scales = q.quantize_int8(w)
    assert np.array_equal(values, g[f"{tag}_q"]) and np.array_equal(bits(scales), bits(g[f"{tag}_scales"]))
    assert np.array_equal(bits(oracle.matmul_i8(g[f"{tag}_x"], values, scales)), bits(g[f"{tag}_y"]))


def test_oracle_tiny_int8_f32_greedy_is_the_references_bitwise():
    g = golden("int8_f32")
    model = oracle.OracleModel(TINY, q.int8_projection_weights(synthetic_weights(TINY, seed=0), TINY), "f32")
    tokens, logits = model.greedy(list(g["tiny_prompt"]), 16, return_logits=True)
    assert tokens == list(g["tiny_tokens"]) and np.array_equal(bits(logits), bits(g["tiny_logits"]))
    zeros = np.zeros((TINY.layers, TINY.kv_heads, 0, TINY.head_dim), np.float32)
    full, _, _ = model.step(list(g["tiny_prompt"]), zeros, zeros, last_only=False)
    assert np.array_equal(bits(full), bits(g["tiny_full_logits"]))


@pytest.mark.slow
def test_oracle_05b_int8_f32_first_steps_are_the_references(qwen05b_vnni_weights):
    g = golden("qwen05b_int8")
    model = oracle.OracleModel(QWEN2_0_5B, qwen05b_vnni_weights, "f32", threads=8)
    tokens, logits = model.greedy(list(g["prompt"]), 3, return_logits=True)
    assert tokens == list(g["tokens"][:3])
    assert np.array_equal(bits(logits[:2]), bits(g["first_logits"]))
    assert all(np.array_equal(sha1(logits[i]), g["sha1"][i]) for i in range(3))
