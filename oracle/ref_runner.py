"""Replays the reference's compiled decode step from oracle/_ref (TEST INFRASTRUCTURE: the CPU
baseline of bench.py; the product never imports this module).

``oracle/build_ref.py`` saved the program the reference compiled -- its generated kernels
(``libnc_ref_step.so``), its thread pool, and the list of calls with their buffers and symbolic
offsets. This module is a restatement of ``CompiledGraph.__call__``
(``nanocompile/runtime.py:245-301``): bind the symbols, give every buffer an address, and call
the kernels ``int32_t nc_kN(void **p, const int64_t *s)`` in order, with the pool bound
(``nanocompile/runtime.py:200-207``) and packed weights made once (``runtime.py:157-164``). The
driver loop around it is the reference's ``Qwen2.forward`` with a ``KVCache`` whose filled region
is handed over as a view and made contiguous every step, as the reference does.
"""

from __future__ import annotations

import ctypes
import json
import os
import subprocess
from collections.abc import Mapping, Sequence
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = HERE / "_ref"
_KERNEL = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int64))


def _eval(poly, bound: Mapping[str, int]) -> int:
    total = 0
    for symbols, coeff in poly:
        term = coeff
        for s in symbols:
            term *= bound[s]
        total += term
    return total


def _load_step_library(ref: Path) -> ctypes.CDLL:
    """The reference's compiled kernels; rebuilt from their generated C if this CPU rejects them."""
    lib = ref / "libnc_ref_step.so"
    try:
        return ctypes.CDLL(str(lib))
    except OSError:
        plan = json.loads((ref / "plan.json").read_text())
        rebuilt = ref / "libnc_ref_step_local.so"
        subprocess.run(["gcc", *plan["cflags"], "-fPIC", "-shared", "-o", str(rebuilt), str(ref / "step.c")], check=True)
        return ctypes.CDLL(str(rebuilt))


class ReferenceModel:
    """The reference's int8-vnni Qwen2.5-0.5B step (last row's logits), on the host cores."""

    def __init__(self, ref: Path, weights: Mapping[str, np.ndarray], threads: int | None = None):
        ref = Path(ref)
        self.plan = json.loads((ref / "plan.json").read_text())
        with np.load(ref / "consts.npz") as c:
            self.consts = {int(k[1:]): np.ascontiguousarray(c[k]) for k in c.files}
        self.pool = ctypes.CDLL(str(ref / "libnc_pool.so"))
        self.pool.nc_pool_set_threads.argtypes = [ctypes.c_int]
        self.pool.nc_pool_set_threads(int(threads or os.cpu_count() or 1))
        self.lib = _load_step_library(ref)
        self.lib.nc_bind_pool.argtypes = [ctypes.c_void_p]
        self.lib.nc_bind_pool(ctypes.cast(self.pool.nc_pool_run, ctypes.c_void_p))
        self.kernels = [_KERNEL((f"nc_k{i}", self.lib)) for i in range(self.plan["kernels"])]
        self.weights = {}
        for b in self.plan["buffers"]:
            if b["kind"] == "weight":
                self.weights[b["name"]] = np.ascontiguousarray(weights[b["name"]])
        self._packs: dict[tuple[int, int], np.ndarray] = {}
        self.vocab = int(self.plan["buffers"][self.plan["outputs"]["logits"]]["shape"][-1][0][1])

    def set_threads(self, threads: int) -> None:
        """Threads of the reference's pool (its NANOCOMPILE_THREADS), the calling thread included."""
        self.pool.nc_pool_set_threads(int(threads))

    def _packed(self, buffer: int, block: int) -> np.ndarray:
        key = (buffer, block)
        if key not in self._packs:
            src = self.weights[self.plan["buffers"][buffer]["name"]]
            rows, cols = src.shape
            self._packs[key] = np.ascontiguousarray(src.reshape(rows // block, block, cols).transpose(0, 2, 1))
        return self._packs[key]

    def step(self, ids: Sequence[int], past_keys: np.ndarray, past_values: np.ndarray, last_only: bool = True):
        """``(logits, keys, values)`` for ``ids`` after the cached ``past_*``; last row only."""
        ids = np.ascontiguousarray(np.asarray(ids, np.int64))
        inputs = {"token_ids": ids, "past_keys": np.ascontiguousarray(past_keys, np.float32),
                  "past_values": np.ascontiguousarray(past_values, np.float32)}
        bound = {"seq": ids.size, "past": inputs["past_keys"].shape[2]}
        syms = (ctypes.c_int64 * max(1, len(self.plan["symbols"])))(*[bound[s] for s in self.plan["symbols"]])
        arrays: dict[int, np.ndarray] = {}
        for i, b in enumerate(self.plan["buffers"]):
            if b["kind"] == "input":
                arrays[i] = inputs[b["name"]]
            elif b["kind"] == "weight":
                arrays[i] = self.weights[b["name"]]
            elif b["kind"] == "const":
                arrays[i] = self.consts[i]
            else:
                shape = tuple(_eval(d, bound) for d in b["shape"])
                arrays[i] = np.empty(shape, np.dtype(b["dtype"]))
        for call in self.plan["calls"]:
            pointers = [arrays[call["output"]].ctypes.data]
            for j, op in enumerate(call["operands"]):
                block = call["packed"].get(str(j))
                if block is not None:
                    pointers.append(self._packed(op["buffer"], block).ctypes.data)
                    continue
                a = arrays[op["buffer"]]
                pointers.append(a.ctypes.data + _eval(op["offset"], bound) * a.itemsize)
            args = (ctypes.c_void_p * len(pointers))(*pointers)
            status = self.kernels[call["kernel"]](args, syms)
            if status != 0:
                raise IndexError(f"reference kernel for {call['primitive']} failed with {status}")
        out = {n: arrays[i] for n, i in self.plan["outputs"].items()}
        return out["logits"], out["keys"], out["values"]

    def greedy(self, prompt: Sequence[int], steps: int, past_keys=None, past_values=None):
        """The reference's greedy loop (``models/qwen2.py:348-368``) with its doubling KVCache."""
        length = 0 if past_keys is None else past_keys.shape[2]
        layers, kv, _, d = (past_keys.shape if past_keys is not None else (24, 2, 0, 64))
        capacity = max(1, length + len(prompt) + steps)
        keys = np.zeros((layers, kv, capacity, d), np.float32)
        values = np.zeros((layers, kv, capacity, d), np.float32)
        if length:
            keys[:, :, :length] = past_keys
            values[:, :, :length] = past_values
        pending, tokens = list(prompt), []
        for _ in range(steps):
            logits, k, v = self.step(pending, keys[:, :, :length], values[:, :, :length])
            n = k.shape[2]
            keys[:, :, length:length + n] = k
            values[:, :, length:length + n] = v
            length += n
            tok = int(np.argmax(logits[0]))
            tokens.append(tok)
            pending = [tok]
        return tokens
