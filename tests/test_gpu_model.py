"""The whole step on the B200, driven through the reference's own ``Qwen2`` and ``Runner`` API.

``nanocompile.models.qwen2.Qwen2(config, weights, run=CUDABackend(), quantization=...)`` is the
reference's driver, unchanged (the copy ``oracle/build_ref.py`` ships); the CUDA backend is the
only thing swapped in. Golden vectors come from the reference's CBackend on the same seeded
weights (tests/golden): the GPU must give the same tokens, and the same logits to the bit.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from nanocompile_b200.model import QWEN2_0_5B, SMALL, TINY, synthetic_cache, synthetic_weights
from tests.conftest import bits, golden

pytestmark = pytest.mark.gpu


def sha1(a) -> np.ndarray:
    return np.frombuffer(hashlib.sha1(np.ascontiguousarray(a, np.float32).tobytes()).digest(), np.uint8)


def ref_model(reference, cuda, shape, weights, quantization, **backend):
    from nanocompile.models.qwen2 import Qwen2, Qwen2Config

    return Qwen2(Qwen2Config(**shape.config_fields()), weights, run=cuda.CUDABackend(device=0, **backend),
                 quantization=quantization)


@pytest.fixture(scope="module")
def tiny_models(reference, cuda):
    w = synthetic_weights(TINY, seed=0)
    return {"fp32": ref_model(reference, cuda, TINY, w, None, capacity=64, slots=4, max_rows=16),
            "vnni": ref_model(reference, cuda, TINY, w, "int8-vnni", capacity=64, slots=4, max_rows=16)}


@pytest.mark.parametrize("tag", ["fp32", "vnni"])
def test_tiny_reference_greedy_tokens_and_logits(tiny_models, tag):
    """The reference's own greedy loop and host KVCache over the CUDA runner."""
    from nanocompile.models.qwen2 import greedy

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
def test_tiny_full_chunked_and_device_cache_steps(tiny_models, cuda, tag):
    g = golden("tiny")
    model = tiny_models[tag]
    prompt = list(g["prompt"])
    assert np.array_equal(bits(model.forward(prompt)), bits(g[f"{tag}_full_logits"]))
    host = model.new_cache(4)                                    # the reference's KVCache, grown by doubling
    rows = [model.forward(prompt[:5], cache=host)] + [model.forward([t], cache=host) for t in prompt[5:]]
    assert np.array_equal(bits(np.concatenate(rows)), bits(g[f"{tag}_chunked_logits"]))
    hk, hv = host.past()
    assert np.array_equal(bits(hk), bits(g[f"{tag}_keys"])) and np.array_equal(bits(hv), bits(g[f"{tag}_values"]))
    device = cuda.new_device_cache(model, 32)                    # the history stays in HBM
    rows = [device.forward(prompt[:5])] + [device.forward([t]) for t in prompt[5:]]
    assert np.array_equal(bits(np.concatenate(rows)), bits(g[f"{tag}_chunked_logits"]))
    dk, dv = device.past()
    assert np.array_equal(bits(dk), bits(g[f"{tag}_keys"])) and np.array_equal(bits(dv), bits(g[f"{tag}_values"]))
    assert cuda.device_greedy(model, prompt, 16) == list(g[f"{tag}_tokens"])


def test_bad_token_ids_raise_the_references_kernel_error(tiny_models, cuda):
    from nanocompile.runtime import KernelError
    from nanocompile.models.qwen2 import greedy

    model = tiny_models["vnni"]
    with pytest.raises(KernelError, match="gather index 256 is outside 0..255"):
        model.forward([1, 256])
    with pytest.raises(cuda.KernelError, match="gather index -1 is outside 0..255"):
        model.forward([-1])
    assert greedy(model, [1, 2], 2) == cuda.device_greedy(model, [1, 2], 2)      # the model still works after


def test_argument_errors_are_the_interpreters(tiny_models):
    from nanocompile.interpreter import InterpreterError

    model = tiny_models["vnni"]
    zeros = np.zeros((2, 2, 3, 16), np.float32)
    step = model.run.compiled(model.graph_last)
    with pytest.raises(InterpreterError, match="already bound"):
        step({"token_ids": np.array([1], np.int64), "past_keys": zeros, "past_values": zeros[:, :, :2]}, model.weights)
    with pytest.raises(InterpreterError, match="missing"):
        step({"token_ids": np.array([1], np.int64)}, model.weights)
    big = np.zeros((2, 2, 64, 16), np.float32)                   # past + seq beyond the backend's capacity
    with pytest.raises(InterpreterError, match="capacity"):
        step({"token_ids": np.array([1], np.int64), "past_keys": big, "past_values": big}, model.weights)


def test_profile_and_plan_of_a_stateless_call(tiny_models):
    model = tiny_models["vnni"]
    step = model.run.compiled(model.graph)
    zeros = np.zeros((2, 2, 0, 16), np.float32)
    profile: dict[str, float] = {}
    out = step({"token_ids": np.array([3, 1, 4], np.int64), "past_keys": zeros, "past_values": zeros}, model.weights,
               profile=profile)
    assert out["logits"].shape == (3, 256) and out["keys"].shape == (2, 2, 3, 16)
    assert {"gather", "attention", "lm_head_argmax"} <= set(profile) and all(v > 0 for v in profile.values())
    plan = step.last_plan
    assert plan.rows == 3 and plan.past == 0 and plan.kv_bytes_out == 3 * 2 * 2 * 16 * 4 * 2 and plan.arena_bytes > 0


@pytest.mark.parametrize("rows", [1, 2, 4])
def test_small_persistent_step_is_the_oracles(cuda, rows):
    """SMALL through the persistent step + int8 LM head (1..4 rows), against the oracle."""
    from nanocompile_b200 import quantize as q
    from oracle.oracle import OracleModel

    w = q.int8_projection_weights(synthetic_weights(SMALL, seed=3), SMALL)
    model = cuda.DeviceModel(SMALL, w, "int8", max_rows=8, slots=4, capacity=200)
    oracle = OracleModel(SMALL, w, "int8")
    first, keys, values = [], [], []
    for b in range(rows):
        k, v, t = synthetic_cache(SMALL, 7 + b, 37 + 29 * b)
        model.kv_write(b, 0, k, v)
        keys.append(k)
        values.append(v)
        first.append(t)
    tokens, _ = model.decode(first, list(range(rows)), [k.shape[2] for k in keys], 24)   # ragged histories
    for b in range(rows):
        assert list(tokens[:, b]) == oracle.greedy([first[b]], 24, keys[b], values[b]), b
    kinds = model.profile(first, list(range(rows)), [k.shape[2] for k in keys], 1)
    assert "persistent_layers" in kinds and "lm_head_argmax" in kinds, kinds


@pytest.fixture(scope="module")
def vnni_05b(reference, cuda, qwen05b_weights):
    return ref_model(reference, cuda, QWEN2_0_5B, qwen05b_weights, "int8-vnni", capacity=1100, slots=2, max_rows=512)


def test_05b_int8_vnni_greedy_993_tokens_are_the_references(vnni_05b, cuda):
    """Configuration 3: 32-token prompt, greedy to past 1024 -- the reference's greedy over the
    stateless runner (its host KVCache each step), and the device-resident decode."""
    from nanocompile.models.qwen2 import greedy

    g = golden("qwen05b_vnni")
    assert cuda.device_greedy(vnni_05b, list(g["prompt"]), 993) == list(g["tokens"])
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


def test_05b_int8_vnni_every_step_logits_through_the_device_cache(vnni_05b, cuda):
    """All 993 steps of configuration 3 with the history in HBM (the persistent decode step for
    the one-row steps): the SHA-1 of every step's float32 logits is the reference's."""
    g = golden("qwen05b_vnni")
    cache = cuda.new_device_cache(vnni_05b, 1100)
    pending = list(g["prompt"])
    for step in range(len(g["tokens"])):
        lg = cache.forward(pending, last_only=True)[0]
        assert np.array_equal(sha1(lg), g["sha1"][step]), step
        pending = [int(g["tokens"][step])]


def test_05b_prefill_512_is_the_references(vnni_05b, cuda):
    """Configuration 4: one step over 512 prompt tokens at past 0, host and device caches."""
    g = golden("prefill")
    for cache in (vnni_05b.new_cache(600), cuda.new_device_cache(vnni_05b, 600)):
        if hasattr(cache, "forward"):
            lg = cache.forward(list(g["ids"]), last_only=True)[0]
        else:
            lg = vnni_05b.forward(list(g["ids"]), cache=cache, last_only=True)[0]
        assert np.array_equal(bits(lg), bits(g["logits"]))
        keys, values = cache.past()
        for layer in range(QWEN2_0_5B.layers):
            assert np.array_equal(sha1(keys[layer]), g["keys_sha1"][layer])
            assert np.array_equal(sha1(values[layer]), g["values_sha1"][layer])


def test_05b_batched_decode_is_the_references(reference, cuda, qwen05b_weights):
    """Configuration 5: 64 sequences from N(0,1) caches of 2048 positions, 64 greedy steps each."""
    g = golden("batch")
    past = int(g["past"])
    model = ref_model(reference, cuda, QWEN2_0_5B, qwen05b_weights, "int8-vnni", capacity=past + 64, slots=64,
                      max_rows=64)
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


def test_05b_batched_decode_logits_are_the_references(cuda, qwen05b_vnni_weights):
    """Configuration 5's logits, not only its tokens: every row of the first and of the 64th batched
    step has the SHA-1 of the reference's float32 logits (the step then takes the exact float32 LM
    head, so this holds the 24 layers and the final norm of all 64 sequences to the bit)."""
    import hashlib

    g = golden("batch")
    past = int(g["past"])
    model = cuda.DeviceModel(QWEN2_0_5B, qwen05b_vnni_weights, "int8", max_rows=64, slots=64, capacity=past + 72)
    first = []
    for b in range(64):
        k, v, t = synthetic_cache(QWEN2_0_5B, b, past)
        model.kv_write(b, 0, k, v)
        first.append(t)
    for steps in (1, 64):
        tokens, logits = model.decode(first, list(range(64)), [past] * 64, steps, want_logits=True)
        assert np.array_equal(tokens.T, g["tokens"][:, 1:steps + 1])
        for b in range(64):
            digest = np.frombuffer(hashlib.sha1(np.ascontiguousarray(logits[b]).tobytes()).digest(), np.uint8)
            assert np.array_equal(digest, g["sha1"][b, steps - 1]), (steps, b)
    model.close()


def test_05b_batched_decode_on_tensor_core_projections(cuda, qwen05b_vnni_weights, monkeypatch):
    """Configuration 5's first 16 steps with the tcgen05 kind::i8 projections (NC_TC_I8=1)."""
    monkeypatch.setenv("NC_TC_I8", "1")
    g = golden("batch")
    past = int(g["past"])
    model = cuda.DeviceModel(QWEN2_0_5B, qwen05b_vnni_weights, "int8", max_rows=64, slots=64, capacity=past + 32)
    first = []
    for b in range(64):
        k, v, t = synthetic_cache(QWEN2_0_5B, b, past)
        model.kv_write(b, 0, k, v)
        first.append(t)
    kinds = model.profile(first, list(range(64)), [past] * 64, 1)
    tokens, _ = model.decode(first, list(range(64)), [past] * 64, 16)
    assert np.array_equal(tokens.T, g["tokens"][:, 1:17])
    assert "gate_up_projection" in kinds
    model.close()


@pytest.mark.parametrize("rows", [1, 3, 4])
def test_05b_small_batched_decode_is_the_references(cuda, qwen05b_vnni_weights, rows):
    """A few of configuration 5's sequences at once: the persistent decode step (up to four rows)."""
    g = golden("batch")
    past = int(g["past"])
    model = cuda.DeviceModel(QWEN2_0_5B, qwen05b_vnni_weights, "int8", max_rows=8, slots=8, capacity=past + 64)
    pick = [5, 17, 40, 63][:rows]
    first = []
    for b, sequence in enumerate(pick):
        k, v, t = synthetic_cache(QWEN2_0_5B, sequence, past)
        model.kv_write(b, 0, k, v)
        first.append(t)
    tokens, _ = model.decode(first, list(range(rows)), [past] * rows, 64)
    assert np.array_equal(tokens.T, g["tokens"][pick, 1:])
    model.close()


def test_persistent_step_phase_table(cuda, qwen05b_vnni_weights):
    """The persistent step's globaltimer phase table: every phase boundary reached, in the
    order the phases run, within one layer's time; the stamps leave the decoded tokens alone; a
    batch the persistent kernel does not serve is refused."""
    g = golden("batch")
    past = int(g["past"])
    model = cuda.DeviceModel(QWEN2_0_5B, qwen05b_vnni_weights, "int8", max_rows=8, slots=8, capacity=past + 64)
    k, v, t = synthetic_cache(QWEN2_0_5B, 5, past)
    model.kv_write(0, 0, k, v)
    phases = model.phase_times([t], [0], [past], 2)
    assert list(phases) == list(model.PHASES)
    order = ["input words in", "input norm", "q/k/v rows out", "q/k/v words in", "scores", "softmax",
             "attention out", "attention blocks in", "o rows out", "residual words in", "post norm",
             "gate/up staged", "SwiGLU out", "SwiGLU in", "down rows out"]
    times = [phases[name] for name in order]
    assert all(0.0 <= a <= b for a, b in zip(times, times[1:])), phases
    assert 0.0 < phases["down rows out"] < 1000.0
    tokens, _ = model.decode([t], [0], [past], 8)
    assert np.array_equal(tokens[:, 0], g["tokens"][5, 1:9])
    with pytest.raises(cuda.InterpreterError, match="persistent decode kernel does not serve"):
        model.phase_times([t] * 5, list(range(5)), [past] * 5, 1)
    model.close()


def test_05b_device_quantized_weights_decode_the_same(cuda, qwen05b_weights, qwen05b_vnni_weights):
    """float32 projections uploaded and quantized on the device give the host quantizer's bytes:
    the same 24 greedy tokens as the golden run."""
    g = golden("qwen05b_vnni")
    model = cuda.DeviceModel(QWEN2_0_5B, qwen05b_weights, "int8", max_rows=64, slots=1, capacity=128)
    _, tok = model.run(np.asarray(g["prompt"], np.int64), 0, 0, last_only=True, want_logits=False)
    more, _ = model.decode([int(tok[0])], [0], [len(g["prompt"])], 23)
    assert [int(tok[0])] + [int(t) for t in more[:, 0]] == list(g["tokens"][:24])
    model.close()


def test_05b_fp32_greedy_is_the_references(reference, cuda, qwen05b_weights):
    """Configuration 2: float32 projections, 32-token prompt, 128 greedy steps."""
    from nanocompile.models.qwen2 import greedy

    g = golden("qwen05b_fp32")
    model = ref_model(reference, cuda, QWEN2_0_5B, qwen05b_weights, None, capacity=200, slots=2, max_rows=64)
    assert cuda.device_greedy(model, list(g["prompt"]), 128) == list(g["tokens"])
    cache = model.new_cache(200)
    lg = model.forward(list(g["prompt"]), cache=cache, last_only=True)[0]
    assert np.array_equal(bits(lg), bits(g["first_logits"][0]))
    assert greedy(model, list(g["prompt"]), 8) == list(g["tokens"][:8])


def test_tiny_int8_f32_through_the_reference_api(reference, cuda):
    """quantization="int8" (int8 weights, float32 activations): the reference's greedy and full
    logits over the CUDA runner, against its CBackend's."""
    from nanocompile.models.qwen2 import greedy

    g = golden("int8_f32")
    model = ref_model(reference, cuda, TINY, synthetic_weights(TINY, seed=0), "int8", capacity=64, slots=2, max_rows=16)
    prompt = list(g["tiny_prompt"])
    assert greedy(model, prompt, 16) == list(g["tiny_tokens"])
    assert cuda.device_greedy(model, prompt, 16) == list(g["tiny_tokens"])
    assert np.array_equal(bits(model.forward(prompt)), bits(g["tiny_full_logits"]))


def test_05b_int8_f32_greedy_is_the_references(reference, cuda, qwen05b_weights):
    """The 0.5B model with quantization="int8": 48 greedy tokens and every step's logits (SHA-1)."""
    g = golden("qwen05b_int8")
    model = ref_model(reference, cuda, QWEN2_0_5B, qwen05b_weights, "int8", capacity=128, slots=2, max_rows=64)
    assert cuda.device_greedy(model, list(g["prompt"]), 48) == list(g["tokens"])
    cache = model.new_cache(128)
    pending = list(g["prompt"])
    for step in range(8):
        lg = model.forward(pending, cache=cache, last_only=True)[0]
        assert np.array_equal(sha1(lg), g["sha1"][step]), step
        pending = [int(g["tokens"][step])]
