"""The allocation-free LM head entry point (collected last: a failure here comes after every other test).

nc_lm_head_argmax_noalloc is for callers that cannot call cudaMalloc -- a host that fixes the
library's device-memory budget, a thread next to a global-mode graph capture, a loop that
cannot afford an allocation's implicit synchronization.  Its scratch is a static device array,
so two calls in a row must still match the entry point that takes caller-provided scratch,
bit for bit, and sizes past the array's limit must be refused with a clear error.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.conftest import bits
from tests.gpu_util import DeviceArray, call

pytestmark = pytest.mark.gpu


def test_noalloc_lm_head_matches_the_scratch_entry_point_twice(cuda):
    rng = np.random.default_rng(7)
    rows, vocab, hidden = 3, 151936, 896
    x = rng.standard_normal((rows, hidden)).astype(np.float32)
    embed = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    embed[vocab - 3] = embed[5]                       # a tie for the first-index rule
    dx, de = DeviceArray(cuda, x), DeviceArray(cuda, embed)
    ref_logits = DeviceArray(cuda, shape=(rows, vocab), dtype=np.float32)
    ref_tokens = DeviceArray(cuda, shape=(rows,), dtype=np.int64)
    scratch = DeviceArray(cuda, shape=(cuda.library().nc_lm_head_scratch_bytes(rows, vocab),), dtype=np.uint8, fill=0)
    call(cuda, "nc_lm_head_argmax", [ref_logits, dx, de, ref_tokens, scratch], [rows, vocab, hidden])
    want_logits, want_tokens = ref_logits.numpy(), ref_tokens.numpy()
    for _ in range(2):
        logits = DeviceArray(cuda, shape=(rows, vocab), dtype=np.float32)
        tokens = DeviceArray(cuda, np.full(rows, -1, np.int64))
        call(cuda, "nc_lm_head_argmax_noalloc", [logits, dx, de, tokens], [rows, vocab, hidden])
        assert np.array_equal(bits(logits.numpy()), bits(want_logits))
        assert np.array_equal(tokens.numpy(), want_tokens)


def test_noalloc_lm_head_refuses_more_rows_than_its_scratch(cuda):
    dx = DeviceArray(cuda, shape=(64, 896), dtype=np.float32, fill=0)
    de = DeviceArray(cuda, shape=(151936, 896), dtype=np.float32, fill=0)
    tokens = DeviceArray(cuda, shape=(64,), dtype=np.int64)
    with pytest.raises(cuda.InterpreterError, match="static scratch holds"):
        call(cuda, "nc_lm_head_argmax_noalloc", [None, dx, de, tokens], [64, 151936, 896])
