"""Shared fixtures. ``-m gpu`` tests need a CUDA device and the built library; the rest run on CPU."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libnc_cuda.so")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


def bits(a: np.ndarray) -> np.ndarray:
    """float32 bit patterns, for bitwise comparison."""
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def golden(name: str) -> dict[str, np.ndarray]:
    path = GOLDEN / f"{name}.npz"
    if not path.exists():
        pytest.skip(f"golden fixture {path.name} not generated")
    with np.load(path) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def qwen05b_weights():
    from nanocompile_b200.model import QWEN2_0_5B, synthetic_weights

    return synthetic_weights(QWEN2_0_5B, seed=0)


@pytest.fixture(scope="session")
def qwen05b_vnni_weights(qwen05b_weights):
    from nanocompile_b200 import quantize as q
    from nanocompile_b200.model import QWEN2_0_5B

    return q.int8_projection_weights(qwen05b_weights, QWEN2_0_5B)


@pytest.fixture(scope="session")
def reference():
    """The reference's own nanocompile package (the copy oracle/build_ref.py ships in oracle/_ref/py)."""
    from oracle import reference as ref

    if not ref.available():
        pytest.skip("the reference's package was not copied to oracle/_ref/py (run oracle/build_ref.py)")
    return ref.import_reference()


@pytest.fixture(scope="session")
def cuda():
    """The CUDA runtime module, or skip when no device is visible."""
    from nanocompile_b200 import runtime

    try:
        n = runtime.device_count()
    except Exception as error:  # no driver / no device
        pytest.skip(f"no CUDA device: {error}")
    if n < 1:
        pytest.skip("no CUDA device")
    return runtime
