"""Build libnc_cuda.so in-tree for sm_100a: ``python -m nanocompile_b200.build``.

``-fmad=false`` keeps every multiply and add that the reference's C keeps apart
(``nanocompile/codegen_c.py:50`` compiles with ``-ffp-contract=off``); fused
multiply-adds appear only where the kernels spell them, as the reference's
``fmaf`` does. Division and square root stay IEEE (no fast-math flags).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SOURCES = [HERE / "csrc" / "nc_cuda.cu"]
DEPENDS = SOURCES + [HERE / "csrc" / "nc_kernels.cuh", HERE / "csrc" / "nc_gemm_i8.cuh", HERE / "csrc" / "nc_gemm_f32.cuh", HERE / "csrc" / "nc_lm_head_tc.cuh", HERE / "csrc" / "nc_lm_head_q8.cuh", HERE / "csrc" / "nc_decode_mk.cuh", HERE / "csrc" / "nc_attention.cuh", HERE / "csrc" / "nc_common.cuh", ROOT / "include" / "nc_cuda.h"]
TARGET = HERE / "libnc_cuda.so"
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-fmad=false",
              "-Xcompiler", "-fPIC", "-shared"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libnc_cuda.so")
    return found


def build(force: bool = False, verbose: bool = False) -> Path:
    newest = max(p.stat().st_mtime for p in DEPENDS)
    if TARGET.exists() and TARGET.stat().st_mtime >= newest and not force:
        return TARGET
    tmp = TARGET.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd))
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{result.stderr[-6000:]}")
    os.replace(tmp, TARGET)
    return TARGET


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
