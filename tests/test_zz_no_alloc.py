"""The allocation-free LM head entry point (collected last: a failure here comes after every other test).

nc_lm_head_argmax_noalloc is for callers that cannot call cudaMalloc -- a host that fixes the
library's device-memory budget, a thread next to a global-mode graph capture, a loop that
cannot afford an allocation's implicit synchronization.  Its scratch is a static device array,
so two calls in a row must still match the entry point that takes caller-provided scratch,
bit for bit, and sizes past the array's limit must be refused with a clear error.

Rows 1..4 run the few-row kernel; 17..27 run the many-row kernel, which counts finished CTAs over
a two-dimensional grid and lays its partial results out differently; 27 rows is the most the
static array takes for Qwen2's 151,936-token vocabulary (27 * 1187 <= 32768 < 28 * 1187).
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import bits
from tests.gpu_util import DeviceArray, call

pytestmark = pytest.mark.gpu

VOCAB, HIDDEN = 151936, 896


@pytest.fixture(scope="module")
def embedding(cuda):
    rng = np.random.default_rng(7)
    embed = (rng.standard_normal((VOCAB, HIDDEN)) * 0.02).astype(np.float32)
    embed[VOCAB - 3] = embed[5]                       # a tie for the first-index rule
    return DeviceArray(cuda, embed)


@pytest.mark.parametrize("rows", [1, 3, 17, 27])
def test_noalloc_lm_head_matches_the_scratch_entry_point_twice(cuda, embedding, rows):
    rng = np.random.default_rng(100 + rows)
    x = rng.standard_normal((rows, HIDDEN)).astype(np.float32)
    dx = DeviceArray(cuda, x)
    ref_logits = DeviceArray(cuda, shape=(rows, VOCAB), dtype=np.float32)
    ref_tokens = DeviceArray(cuda, shape=(rows,), dtype=np.int64)
    scratch = DeviceArray(cuda, shape=(cuda.library().nc_lm_head_scratch_bytes(rows, VOCAB),), dtype=np.uint8, fill=0)
    call(cuda, "nc_lm_head_argmax", [ref_logits, dx, embedding, ref_tokens, scratch], [rows, VOCAB, HIDDEN])
    want_logits, want_tokens = ref_logits.numpy(), ref_tokens.numpy()
    for _ in range(2):
        logits = DeviceArray(cuda, shape=(rows, VOCAB), dtype=np.float32)
        tokens = DeviceArray(cuda, np.full(rows, -1, np.int64))
        call(cuda, "nc_lm_head_argmax_noalloc", [logits, dx, embedding, tokens], [rows, VOCAB, HIDDEN])
        assert np.array_equal(bits(logits.numpy()), bits(want_logits))
        assert np.array_equal(tokens.numpy(), want_tokens)


@pytest.mark.parametrize("rows", [28, 64, 1 << 40])
def test_noalloc_lm_head_refuses_more_rows_than_its_scratch(cuda, embedding, rows):
    dx = DeviceArray(cuda, shape=(64, HIDDEN), dtype=np.float32, fill=0)
    tokens = DeviceArray(cuda, shape=(64,), dtype=np.int64)
    with pytest.raises(cuda.InterpreterError, match="static scratch holds"):
        call(cuda, "nc_lm_head_argmax_noalloc", [None, dx, embedding, tokens], [rows, VOCAB, HIDDEN])
