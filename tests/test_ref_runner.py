"""The reference's own compiled step, replayed from oracle/_ref, against the golden run and the
oracle: the CPU baseline bench.py times is the reference's algorithm, bit for bit."""

import numpy as np
import pytest

from tests.conftest import bits, golden
from nanocompile_b200.model import QWEN2_0_5B, synthetic_cache
from oracle import oracle

ref_runner = pytest.importorskip("oracle.ref_runner")
if not (ref_runner.REF / "plan.json").exists():
    pytest.skip("oracle/_ref not built (needs the reference checkout)", allow_module_level=True)


@pytest.fixture(scope="module")
def reference(qwen05b_vnni_weights):
    return ref_runner.ReferenceModel(ref_runner.REF, qwen05b_vnni_weights, threads=8)


def test_replayed_reference_reproduces_the_golden_run(reference):
    g = golden("qwen05b_vnni")
    logits, keys, values = reference.step(list(g["prompt"]), np.zeros((24, 2, 0, 64), np.float32),
                                          np.zeros((24, 2, 0, 64), np.float32))
    assert np.array_equal(bits(logits[0]), bits(g["first_logits"][0]))
    assert np.array_equal(bits(keys[0, :, :, :]), bits(g["prompt_keys_layer0"]))
    assert reference.greedy(list(g["prompt"]), 8) == list(g["tokens"][:8])


def test_replayed_reference_equals_the_oracle_on_a_long_cache(reference, qwen05b_vnni_weights):
    keys, values, first = synthetic_cache(QWEN2_0_5B, 3, 96)
    port = oracle.OracleModel(QWEN2_0_5B, qwen05b_vnni_weights, "int8", threads=8)
    a = reference.step([first], keys, values)
    b = port.step([first], keys, values, last_only=True)
    for x, y in zip(a, b):
        assert np.array_equal(bits(np.asarray(x).reshape(-1)), bits(np.asarray(y).reshape(-1)))
