"""The C ABI: the library loads without a GPU and exports every entry point include/nc_cuda.h declares."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "nc_cuda.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(nc_\w+)\s*\(", text)))


def test_header_declares_the_fused_groups_and_the_runtime():
    names = declared()
    for required in ("nc_matmul_i8_vnni", "nc_rms_norm_quantize", "nc_attention", "nc_lm_head_argmax",
                     "nc_qwen2_create", "nc_qwen2_step", "nc_qwen2_decode", "nc_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from nanocompile_b200 import build, runtime

    if not runtime.LIBRARY_PATH.exists():
        build.build()
    lib = ctypes.CDLL(str(runtime.LIBRARY_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from nanocompile_b200 import runtime

    monkeypatch.setattr(runtime, "_LIB", None)
    monkeypatch.setattr(runtime, "LIBRARY_PATH", tmp_path / "absent.so")
    with pytest.raises(ImportError, match="missing"):
        runtime.library()


def test_oracle_library_exports_its_header():
    from oracle import oracle

    lib = oracle.lib()
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "oracle" / "nc_oracle.h").read_text(), flags=re.S)
    for name in set(re.findall(r"\b(orc_\w+)\s*\(", text)):
        assert hasattr(lib, name), name
