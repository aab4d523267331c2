"""The whole step on the B200 through the public API, against the reference's own outputs.

Golden vectors come from nanocompile's CBackend on the same seeded weights (tests/golden);
the GPU must give the same tokens and the same logits to the bit.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from nanocompile_b200.qwen2 import QWEN2_0_5B, SMALL, TINY, Qwen2, greedy, synthetic_cache, synthetic_weights
from tests.conftest import bits, golden

pytestmark = pytest.mark.gpu


def sha1(a) -> np.ndarray:
    return np.frombuffer(hashlib.sha1(np.ascontiguousarray(a, np.float32).tobytes()).digest(), np.uint8)


@pytest.fixture(scope="module")
def tiny_models(cuda):
    w = synthetic_weights(TINY, seed=0)
    backend = cuda.CUDABackend(device=0, capacity=64, slots=4, max_rows=16)
    return {"fp32": Qwen2(TINY, w, run=backend, quantization=None),
            "vnni": Qwen2(TINY, w, run=backend, quantization="int8-vnni")}


@pytest.mark.parametrize("tag", ["fp32", "vnni"])
def test_tiny_greedy_tokens_and_logits_are_the_references(tiny_models, tag):
    g = golden("tiny")
    model = tiny_models[tag]
    prompt = list(g["prompt"])
    assert greedy(model, prompt, 16) == list(g[f"{tag}_tokens"])
    cache = model.new_cache(32)
    pending, logits = prompt, []
    for _ in range(16):
        lg = model.forward(pending, cache=cache, last_only=True)
        logits.append(lg[0])
        pending = [int(np.argmax(lg[0]))]
    assert np.array_equal(bits(np.stack(logits)), bits(g[f"{tag}_logits"]))


@pytest.mark.parametrize("tag", ["fp32", "vnni"])
def test_tiny_full_chunked_and_stateless_steps(tiny_models, tag):
    g = golden("tiny")
    model = tiny_models[tag]
    prompt = list(g["prompt"])
    assert np.array_equal(bits(model.forward(prompt)), bits(g[f"{tag}_full_logits"]))
    cache = model.new_cache(32)
    rows = [model.forward(prompt[:5], cache=cache)] + [model.forward([t], cache=cache) for t in prompt[5:]]
    assert np.array_equal(bits(np.concatenate(rows)), bits(g[f"{tag}_chunked_logits"]))
    keys, values = cache.past()
    assert np.array_equal(bits(keys), bits(g[f"{tag}_keys"])) and np.array_equal(bits(values), bits(g[f"{tag}_values"]))
    # the reference's stateless Runner contract: host KV in, new KV out
    from nanocompile_b200.qwen2 import KVCache

    host = KVCache(TINY, 4)
    rows = [model.forward(prompt[:5], cache=host)] + [model.forward([t], cache=host) for t in prompt[5:]]
    assert np.array_equal(bits(np.concatenate(rows)), bits(g[f"{tag}_chunked_logits"]))
    hk, hv = host.past()
    assert np.array_equal(bits(hk), bits(g[f"{tag}_keys"])) and np.array_equal(bits(hv), bits(g[f"{tag}_values"]))


def test_bad_token_ids_raise_kernel_error(tiny_models, cuda):
    model = tiny_models["vnni"]
    with pytest.raises(cuda.KernelError, match="index 256"):
        model.forward([1, 256])
    with pytest.raises(cuda.KernelError, match="index -1"):
        model.forward([-1])
    assert greedy(model, [1, 2], 2) == greedy(model, [1, 2], 2)      # the model still works after


def oracle_decode(oracle, first, keys, values, steps):
    """Greedy tokens of one sequence after its cached history, step by step on the CPU oracle."""
    out, token = [], first
    for _ in range(steps):
        logits, k, v = oracle.step([token], keys, values)
        keys, values = np.concatenate([keys, k], 2), np.concatenate([values, v], 2)
        token = int(np.argmax(logits[0]))
        out.append(token)
    return out


@pytest.mark.parametrize("rows", [1, 2, 4])
def test_small_persistent_step_is_the_oracles(cuda, rows):
    """SMALL through the persistent step + int8 LM head (1..4 rows), against the oracle."""
    from oracle.oracle import OracleModel

    w = synthetic_weights(SMALL, seed=3)
    backend = cuda.CUDABackend(device=0, capacity=200, slots=4, max_rows=8)
    model = Qwen2(SMALL, w, run=backend, quantization="int8-vnni")
    oracle = OracleModel(SMALL, model.weights, "int8")
    first, keys, values = [], [], []
    for b in range(rows):
        k, v, t = synthetic_cache(SMALL, 7 + b, 37 + 29 * b)
        keys.append(k)
        values.append(v)
        first.append(t)
    tokens = cuda.batched_greedy(model, first, keys, values, 24)     # ragged histories, one replay per step
    for b in range(rows):
        assert list(tokens[b]) == oracle_decode(oracle, first[b], keys[b], values[b], 24), b
    compiled = backend.compiled(model.graph_last, model.weights)
    kinds = compiled.model.profile(first, list(range(rows)), [k.shape[2] for k in keys], 1)
    assert "persistent_layers" in kinds and "lm_head_argmax" in kinds, kinds


@pytest.fixture(scope="module")
def vnni_05b(cuda, qwen05b_weights):
    backend = cuda.CUDABackend(device=0, capacity=1100, slots=2, max_rows=64)
    return Qwen2(QWEN2_0_5B, qwen05b_weights, run=backend, quantization="int8-vnni")


def test_05b_int8_vnni_greedy_993_tokens_are_the_references(vnni_05b):
    """Config 3: 32-token prompt, greedy decode up to past = 1024, CUDA-graph replays."""
    g = golden("qwen05b_vnni")
    assert greedy(vnni_05b, list(g["prompt"]), 993) == list(g["tokens"])


def test_05b_int8_vnni_step_logits_are_the_references(vnni_05b):
    g = golden("qwen05b_vnni")
    cache = vnni_05b.new_cache(1100)
    pending = list(g["prompt"])
    for step in range(48):
        lg = vnni_05b.forward(pending, cache=cache, last_only=True)[0]
        assert np.array_equal(sha1(lg), g["sha1"][step]), step
        pending = [int(g["tokens"][step])]
    assert np.array_equal(bits(g["samples"][47]), bits(lg[::1009]))


def test_05b_prefill_512_is_the_references(vnni_05b):
    """Config 4: one step over 512 prompt tokens at past 0."""
    g = golden("prefill")
    cache = vnni_05b.new_cache(600)
    lg = vnni_05b.forward(list(g["ids"]), cache=cache, last_only=True)[0]
    assert np.array_equal(bits(lg), bits(g["logits"]))
    keys, values = cache.past()
    for layer in range(QWEN2_0_5B.num_hidden_layers):
        assert np.array_equal(sha1(keys[layer]), g["keys_sha1"][layer])
        assert np.array_equal(sha1(values[layer]), g["values_sha1"][layer])


def test_05b_batched_decode_is_the_references(cuda, qwen05b_weights):
    """Config 5: 64 sequences from N(0,1) caches of 2048 positions, 64 greedy steps each."""
    g = golden("batch")
    past = int(g["past"])
    backend = cuda.CUDABackend(device=0, capacity=past + 64, slots=64, max_rows=64)
    model = Qwen2(QWEN2_0_5B, qwen05b_weights, run=backend, quantization="int8-vnni")
    first, keys, values = [], [], []
    for b in range(64):
        k, v, t = synthetic_cache(QWEN2_0_5B, b, past)
        keys.append(k)
        values.append(v)
        first.append(t)
    tokens = cuda.batched_greedy(model, first, keys, values, 64)
    expected = g["tokens"]
    assert np.array_equal(np.asarray(first), expected[:, 0])
    assert np.array_equal(tokens, expected[:, 1:])


@pytest.mark.parametrize("rows", [1, 3, 4])
def test_05b_small_batched_decode_is_the_references(cuda, qwen05b_weights, rows):
    """A few of config 5's sequences at once: the persistent decode step (up to four rows)."""
    g = golden("batch")
    past = int(g["past"])
    backend = cuda.CUDABackend(device=0, capacity=past + 64, slots=8, max_rows=8)
    model = Qwen2(QWEN2_0_5B, qwen05b_weights, run=backend, quantization="int8-vnni")
    pick = [5, 17, 40, 63][:rows]
    first, keys, values = [], [], []
    for b in pick:
        k, v, t = synthetic_cache(QWEN2_0_5B, b, past)
        keys.append(k)
        values.append(v)
        first.append(t)
    tokens = cuda.batched_greedy(model, first, keys, values, 64)
    assert np.array_equal(tokens, g["tokens"][pick, 1:])


def test_05b_fp32_greedy_is_the_references(cuda, qwen05b_weights):
    """Config 2: float32 projections, 32-token prompt, 128 greedy steps."""
    g = golden("qwen05b_fp32")
    backend = cuda.CUDABackend(device=0, capacity=200, slots=2, max_rows=64)
    model = Qwen2(QWEN2_0_5B, qwen05b_weights, run=backend, quantization=None)
    assert greedy(model, list(g["prompt"]), 128) == list(g["tokens"])
    cache = model.new_cache(200)
    lg = model.forward(list(g["prompt"]), cache=cache, last_only=True)[0]
    assert np.array_equal(bits(lg), bits(g["first_logits"][0]))
