"""Build the reference's own CPU implementation of the decode step into oracle/_ref (TEST
INFRASTRUCTURE: the CPU baseline of bench.py, and a second oracle for the tests).

    python oracle/build_ref.py [--reference PATH]

Runs only where the nanocompile checkout is present (this build container). It asks the
reference to compile its int8-vnni Qwen2.5-0.5B step exactly as ``Qwen2(..., run=CBackend(),
quantization="int8-vnni")`` does (``nanocompile/models/qwen2.py:291-311``,
``nanocompile/runtime.py:182-207``), and writes into ``oracle/_ref/`` (git-ignored; it travels to
the GPU box with the snapshot):

* ``libnc_ref_step.so`` -- the library the reference's gcc build produced, and
  ``step.c`` -- its generated C, to rebuild it if the host CPU differs;
* ``libnc_pool.so`` -- the reference's thread pool, compiled from ``nanocompile/pool.c`` where it
  lies;
* ``plan.json`` / ``consts.npz`` -- the compiled program's buffers, calls and constants, so
  ``oracle/ref_runner.py`` can replay the call loop of ``CompiledGraph.__call__`` without the
  reference's Python;
* ``py/nanocompile/`` -- the reference's Python package as it is, so the tests that drive the CUDA
  backend through the reference's own ``Qwen2`` and ``CBackend``-style ``Runner`` API can import it
  on a machine without the checkout (the GPU box).

Nothing from the reference's source tree is committed: ``oracle/_ref/`` is git-ignored. The
checkout is found through ``NANOCOMPILE_REFERENCE`` or, without it, the ``reference_path`` that
``BASELINE.json`` records.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
PACKAGE = OUT / "py"


def reference_checkout() -> Path | None:
    """The nanocompile checkout: ``NANOCOMPILE_REFERENCE``, else BASELINE.json's ``reference_path``."""
    configured = os.environ.get("NANOCOMPILE_REFERENCE")
    if not configured:
        baseline = HERE.parent / "BASELINE.json"
        try:
            configured = json.loads(baseline.read_text()).get("reference_path")
        except (OSError, ValueError):
            configured = None
    if not configured:
        return None
    path = Path(configured)
    return path if (path / "nanocompile" / "__init__.py").exists() else None


def copy_package(reference: Path, out: Path = PACKAGE) -> Path:
    """The reference's ``nanocompile`` package (its .py files and pool.c) under ``out``."""
    source = Path(reference) / "nanocompile"
    target = out / "nanocompile"
    if target.exists():
        shutil.rmtree(target)
    for path in source.rglob("*"):
        if path.suffix in (".py", ".c") and "__pycache__" not in path.parts:
            dest = target / path.relative_to(source)
            dest.parent.mkdir(parents=True, exist_ok=True)
            shutil.copyfile(path, dest)
    return target


def _poly(d) -> list:
    """A dimension (int or the reference's polynomial) as [[symbols, coeff], ...]."""
    if isinstance(d, int):
        return [[[], int(d)]]
    return [[list(m), int(c)] for m, c in d._terms.items()]


def build(reference: Path, out: Path = OUT) -> Path:
    reference = Path(reference)
    if not (reference / "nanocompile").exists():
        raise FileNotFoundError(f"no nanocompile checkout at {reference}")
    sys.path.insert(1, str(reference))
    os.environ.setdefault("NANOCOMPILE_CACHE", tempfile.mkdtemp(prefix="nanocompile-cache-"))
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
    from nanocompile import codegen_c, quantize
    from nanocompile.models.qwen2 import Qwen2Config, build_qwen2
    from nanocompile.runtime import CompiledGraph

    out.mkdir(parents=True, exist_ok=True)
    cfg = Qwen2Config(151936, 896, 4864, 24, 14, 2, 1e-6, 1e6, True)
    graph = quantize.quantize(build_qwen2(cfg, last_only=True), "int8", keep=("lm_head.weight",))
    compiled = CompiledGraph(graph)
    program = compiled.program

    buffers = {id(b): i for i, b in enumerate(program.buffers)}
    consts = {}
    plan = {"symbols": list(program.symbols), "kernels": len(program.kernels), "cflags": list(codegen_c.CFLAGS),
            "buffers": [], "calls": [], "outputs": {n: buffers[id(b)] for n, b in program.outputs.items()},
            "inputs": list(graph.input_names)}
    for i, b in enumerate(program.buffers):
        plan["buffers"].append({"kind": b.kind, "name": b.name, "dtype": b.dtype.numpy.str,
                                "shape": [_poly(d) for d in b.shape]})
        if b.kind == "const":
            consts[f"b{i}"] = np.asarray(b.value)
    for c, call in enumerate(program.calls):
        packed = {}
        for j, param in enumerate(program.kernels[call.kernel].params[1:]):
            if param.packed is not None:
                packed[str(j)] = int(param.packed)
        plan["calls"].append({"kernel": call.kernel, "output": buffers[id(call.output)],
                              "operands": [{"buffer": buffers[id(v.buffer)], "offset": _poly(v.offset)}
                                           for v in call.operands],
                              "primitive": call.primitive, "packed": packed})
    (out / "plan.json").write_text(json.dumps(plan))
    np.savez(out / "consts.npz", **consts)
    (out / "step.c").write_text(compiled.source)
    shutil.copyfile(compiled.library_path, out / "libnc_ref_step.so")
    subprocess.run(["gcc", *codegen_c.CFLAGS, "-pthread", "-fPIC", "-shared", "-o", str(out / "libnc_pool.so"),
                    str(reference / "nanocompile" / "pool.c")], check=True)
    (out / "cpu.txt").write_text(_cpu_identity())
    copy_package(reference, out / "py")
    return out


def _cpu_identity() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("flags"):
                return line
    except OSError:
        pass
    return ""


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", default=None, help="the nanocompile checkout (default: "
                        "NANOCOMPILE_REFERENCE, else BASELINE.json's reference_path)")
    args = parser.parse_args()
    reference = Path(args.reference) if args.reference else reference_checkout()
    if reference is None:
        parser.error("no nanocompile checkout: pass --reference or set NANOCOMPILE_REFERENCE")
    print(build(reference))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
