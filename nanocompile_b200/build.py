"""Build libnc_cuda.so in-tree for sm_100a: ``python -m nanocompile_b200.build [--force]``.

``-fmad=false`` keeps every multiply and add that the reference's C keeps apart
(``nanocompile/codegen_c.py:50`` compiles with ``-ffp-contract=off``); fused
multiply-adds appear only where the kernels spell them, as the reference's
``fmaf`` does. Division and square root stay IEEE (no fast-math flags).

A stamp next to the library records a hash of the nvcc command, of every source
and header it reads, and of this file; the library is rebuilt whenever that hash
changes (or with ``force``), so a library built from other sources or flags is
never reused.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SOURCES = [HERE / "csrc" / "nc_cuda.cu"]
TARGET = HERE / "libnc_cuda.so"
STAMP = TARGET.with_name(TARGET.name + ".stamp")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-fmad=false",
              "-Xcompiler", "-fPIC", "-shared"]


def depends() -> list[Path]:
    """Every file the library is built from: the sources, their headers, the C ABI, this recipe."""
    return sorted({*SOURCES, *(HERE / "csrc").glob("*.cuh"), *(ROOT / "include").glob("*.h"), Path(__file__).resolve()})


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libnc_cuda.so")
    return found


def fingerprint() -> str:
    h = hashlib.sha256(" ".join(NVCC_FLAGS).encode())
    for path in depends():
        h.update(path.name.encode())
        h.update(path.read_bytes())
    return h.hexdigest()


def up_to_date() -> bool:
    return TARGET.exists() and STAMP.exists() and STAMP.read_text().strip() == fingerprint()


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return TARGET
    stamp = fingerprint()
    tmp = TARGET.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd))
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{result.stderr[-6000:]}")
    os.replace(tmp, TARGET)
    STAMP.write_text(stamp + "\n")
    return TARGET


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
