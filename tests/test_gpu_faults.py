"""Failure detection on the GPU without a GPU fault: bounded waits made to run out.

Each device-side wait of the library gives up after a number of SM cycles, records a fault word
and lets its kernel stop cleanly (drain its copies and MMAs, free its TMEM); the host reports the
fault as KernelError. Here the limit is made short (nc_set_wait_limit) so that waits run out on
purpose -- against a condition that never comes true, and inside a real projection and a real
decode step -- and the next call, at the default limit, must be correct to the bit.
"""

from __future__ import annotations

import numpy as np
import pytest

from nanocompile_b200 import quantize as q
from nanocompile_b200.model import SMALL, synthetic_cache, synthetic_weights
from oracle import oracle
from tests.conftest import bits
from tests.gpu_util import DeviceArray, call, packed_int8

pytestmark = pytest.mark.gpu


@pytest.fixture()
def short_waits(cuda):
    cuda.device_faults()                               # start clean
    yield cuda
    cuda.set_wait_limit(0)                             # back to the default, whatever happened
    try:
        cuda.device_faults()
    except cuda.KernelError:
        pass


@pytest.mark.parametrize("kind,what", [(0, "hand-over word"), (1, "pipeline stage")])
def test_a_wait_that_never_ends_reports_a_kernel_error(short_waits, kind, what):
    cuda = short_waits
    cuda.set_wait_limit(200_000)                       # ~0.1 ms
    with pytest.raises(cuda.KernelError, match=what):
        cuda.selftest_wait(kind)
    cuda.device_faults()                               # reported once, then clear


def _projection(cuda, rows=64, n=896, k=4864, seed=3):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, k)) * 2).astype(np.float32)
    xq, xs, off, _ = oracle.quantize_blocks(x)
    w, s = q.quantize_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    expect = oracle.matmul_i8_vnni(xq, xs, off, w, s)
    args = [DeviceArray(cuda, shape=(rows, n), dtype=np.float32, fill=0), DeviceArray(cuda, xq), DeviceArray(cuda, xs),
            DeviceArray(cuda, off[:, 0]), packed_int8(cuda, w), DeviceArray(cuda, s)]
    return args, expect, [rows, n, k, 0, 0, 0]


def test_tensor_core_projection_stops_on_a_short_wait_and_recovers(short_waits):
    cuda = short_waits
    args, expect, sizes = _projection(cuda)
    cuda.set_wait_limit(1)                             # every stage wait that is not already satisfied gives up
    call(cuda, "nc_matmul_i8_tc", args + [None] * 6, sizes)
    with pytest.raises(cuda.KernelError, match="wait limit"):
        cuda.device_faults()
    cuda.set_wait_limit(0)
    call(cuda, "nc_matmul_i8_tc", args + [None] * 6, sizes)
    cuda.device_faults()
    assert np.array_equal(bits(args[0].numpy()), bits(expect))


def test_batched_decode_step_fault_is_reported_and_the_retry_is_exact(short_waits, monkeypatch):
    """Eight sequences on the tensor-core projections: a decode with waits cut short fails with
    KernelError; the same decode again, at the default limit, gives the oracle's tokens."""
    cuda = short_waits
    monkeypatch.setenv("NC_TC_I8", "1")
    w = q.int8_projection_weights(synthetic_weights(SMALL, seed=3), SMALL)
    model = cuda.DeviceModel(SMALL, w, "int8", max_rows=8, slots=8, capacity=128)
    first, starts = [], []
    for b in range(8):
        k, v, t = synthetic_cache(SMALL, 20 + b, 30 + b)
        model.kv_write(b, 0, k, v)
        first.append(t)
        starts.append(k.shape[2])
    model.decode(first, list(range(8)), starts, 1)     # capture the decode graph at the default limit
    cuda.set_wait_limit(1)
    with pytest.raises(cuda.KernelError):
        model.decode(first, list(range(8)), starts, 4)
    cuda.set_wait_limit(0)
    tokens, _ = model.decode(first, list(range(8)), starts, 6)
    ref = oracle.OracleModel(SMALL, w, "int8")
    for b in range(8):
        k, v, t = synthetic_cache(SMALL, 20 + b, 30 + b)
        assert list(tokens[:, b]) == ref.greedy([t], 6, k, v), b
    model.close()


def test_device_cache_capacity_overflow_is_refused(cuda, reference):
    from nanocompile.models.qwen2 import Qwen2, Qwen2Config

    model = Qwen2(Qwen2Config(**SMALL.config_fields()), synthetic_weights(SMALL, seed=1),
                  run=cuda.CUDABackend(capacity=32, slots=2, max_rows=8), quantization="int8-vnni")
    cache = cuda.new_device_cache(model, 16)
    cache.forward(list(range(10)))
    with pytest.raises(cuda.InterpreterError, match="holds 16 positions"):
        cache.forward(list(range(7)))
    with pytest.raises(cuda.InterpreterError, match="capacity"):
        cuda.new_device_cache(model, 64)
    assert cache.length == 10                          # the refused step changed nothing
