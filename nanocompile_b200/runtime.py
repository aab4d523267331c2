"""The CUDA runtime: one ``libnc_cuda.so`` over ctypes, behind nanocompile's ``Runner`` API.

This is the CUDA twin of ``nanocompile/runtime.py``:

* :class:`CUDABackend` is a ``Runner`` for the reference's ``Qwen2``
  (``nanocompile/models/qwen2.py:229``), as ``CBackend`` is (``nanocompile/runtime.py:321-337``):
  ``Qwen2(config, weights, run=CUDABackend(), quantization="int8-vnni")``. It compiles each graph
  once, on first use, through the CUDA target (``nanocompile_b200.target``).
* :class:`CompiledGraph` plays the reference's ``CompiledGraph`` (``nanocompile/runtime.py:167-318``):
  ``program`` (the reference's fused ``Program``), ``groups`` (the CUDA fused groups its calls map
  to), ``source``, ``library_path``, ``cached``, ``compile_seconds``, ``last_plan``, and
  ``__call__(inputs, weights, bindings=None, profile=None)``. Arguments are checked by the
  reference's own ``interpreter.check_arguments``, so both backends accept and refuse the same
  calls with the same messages; a failing kernel raises the reference's ``KernelError``.
* :class:`DeviceModel` is the model resident on one GPU: the arena, the weights, the KV cache of
  its sequence slots; :func:`device_greedy`, :class:`DeviceCache` and :func:`batched_greedy` keep
  the KV history in HBM (the reference's phase 7), so a decode step moves only token ids in and
  tokens out and replays one captured CUDA graph.

There is no CPU path: without the compiled library every entry point raises.
"""

from __future__ import annotations

import ctypes
import time
from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from nanocompile_b200.model import ModelShape
from nanocompile_b200.quantize import int8_name, scales_name

LIBRARY_PATH = Path(__file__).resolve().parent / "libnc_cuda.so"

NC_OK, NC_ERR_KERNEL, NC_ERR_ARGUMENT, NC_ERR_CUDA, NC_ERR_STATE = 0, 1, 2, 3, 4
QUANT_CODES = {None: 0, "int8": 1, "f32": 2}


class KernelError(RuntimeError):
    """A kernel rejected its input (an out-of-range gather index): ``nanocompile/runtime.py:49``."""


class InterpreterError(RuntimeError):
    """Arguments that do not fit the model (sizes, slots, capacity)."""


class CUDAError(RuntimeError):
    """The CUDA runtime or the library failed."""


class NCConfig(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_int64), ("hidden", ctypes.c_int64), ("inter", ctypes.c_int64),
                ("layers", ctypes.c_int64), ("heads", ctypes.c_int64), ("kv_heads", ctypes.c_int64),
                ("head_dim", ctypes.c_int64), ("eps", ctypes.c_float), ("attn_scale", ctypes.c_float),
                ("quant", ctypes.c_int32), ("max_rows", ctypes.c_int32), ("slots", ctypes.c_int32),
                ("capacity", ctypes.c_int32), ("device", ctypes.c_int32)]


_LIB: ctypes.CDLL | None = None
_vp, _i64, _i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
_P64, _P32, _PF = ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float)

# Fused-group entry points: int32_t f(void **p, const int64_t *s, void *stream).
GROUP_ENTRY_POINTS = ("nc_gather_rows", "nc_rms_norm_quantize", "nc_quantize_blocks", "nc_matmul_i8_vnni",
                      "nc_matmul_i8_tc", "nc_matmul_i8_f32", "nc_matmul_f32", "nc_lm_head_argmax",
                      "nc_lm_head_argmax_noalloc", "nc_attention", "nc_attention_cache", "nc_expf_exact",
                      "nc_lm_head_q8_prepare", "nc_lm_head_q8_argmax", "nc_quantize_int8_rows")


def library() -> ctypes.CDLL:
    """The compiled CUDA library; raises if it was not built (there is no fallback)."""
    global _LIB
    if _LIB is None:
        if not LIBRARY_PATH.exists():
            raise ImportError(f"{LIBRARY_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; "
                              f"g.build()'` or `python -m nanocompile_b200.build`")
        L = ctypes.CDLL(str(LIBRARY_PATH))
        L.nc_last_error.argtypes = [ctypes.c_char_p, _i64]
        L.nc_last_error.restype = _i32
        for name in GROUP_ENTRY_POINTS:
            fn = getattr(L, name)
            fn.argtypes = [ctypes.POINTER(_vp), _P64, _vp]
            fn.restype = _i32
        signatures = {
            "nc_device_faults": ([], _i32),
            "nc_set_wait_limit": ([_i64], _i32),
            "nc_selftest_wait": ([_i32], _i32),
            "nc_selfcheck_div127": ([_P64], _i32),
            "nc_lm_head_scratch_bytes": ([_i64, _i64], _i64),
            "nc_lm_head_q8_scratch_bytes": ([_i64, _i64], _i64),
            "nc_device_count": ([_P32], _i32),
            "nc_set_device": ([_i32], _i32),
            "nc_device_alloc": ([_i64, ctypes.POINTER(_vp)], _i32),
            "nc_device_free": ([_vp], _i32),
            "nc_copy_to_device": ([_vp, _vp, _i64], _i32),
            "nc_copy_to_host": ([_vp, _vp, _i64], _i32),
            "nc_device_synchronize": ([], _i32),
            "nc_pack_int8_weights": ([_vp, _vp, _i64], _i32),
            "nc_qwen2_create": ([ctypes.POINTER(NCConfig), _PF, ctypes.POINTER(_vp)], _i32),
            "nc_qwen2_destroy": ([_vp], _i32),
            "nc_qwen2_arena_bytes": ([_vp], _i64),
            "nc_qwen2_upload": ([_vp, ctypes.c_char_p, _vp, _i64], _i32),
            "nc_qwen2_upload_quantize": ([_vp, ctypes.c_char_p, _vp, _i64], _i32),
            "nc_qwen2_missing_weights": ([_vp, _P32], _i32),
            "nc_qwen2_kv_write": ([_vp, _i32, _i64, _i64, _PF, _PF], _i32),
            "nc_qwen2_kv_read": ([_vp, _i32, _i64, _i64, _PF, _PF], _i32),
            "nc_qwen2_step": ([_vp, _i32, _P64, _P32, _P32, _i32, _P32, _PF, _P64, _P32], _i32),
            "nc_qwen2_decode": ([_vp, _i32, _P32, _P64, _P32, _i32, _i32, _P64, _PF], _i32),
            "nc_qwen2_decode_timed": ([_vp, _i32, _P32, _P64, _P32, _i32, _PF], _i32),
            "nc_qwen2_profile": ([_vp, _i32, _P32, _P64, _P32, _i32, _PF, _P32], _i32),
            "nc_qwen2_phase_times": ([_vp, _i32, _P32, _P64, _P32, _i32, _PF], _i32),
            "nc_qwen2_probe": ([_vp, _i32, _PF, _P32], _i32),
            "nc_qwen2_step_timed": ([_vp, _i32, _P64, _P32, _P32, _i32, _PF], _i32),
        }
        for name, (args, res) in signatures.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _LIB = L
    return _LIB


def last_error() -> str:
    buf = ctypes.create_string_buffer(2048)
    library().nc_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    """Turn a library status into the matching exception."""
    if status == NC_OK:
        return
    message = last_error()
    if status == NC_ERR_KERNEL:
        raise KernelError(message)
    if status in (NC_ERR_ARGUMENT, NC_ERR_STATE):
        raise InterpreterError(message)
    raise CUDAError(message)


def device_count() -> int:
    n = ctypes.c_int32(0)
    check(library().nc_device_count(ctypes.byref(n)))
    return n.value


def set_wait_limit(cycles: int) -> None:
    """Bound the abandonable device-side waits on the current device to ``cycles`` SM cycles
    (``<= 0``: the default 2^31). A wait that runs out stops its kernel cleanly and is reported
    by the next :func:`device_faults` or model call as a :class:`KernelError`."""
    check(library().nc_set_wait_limit(int(cycles)))


def device_faults() -> None:
    """Raise :class:`KernelError` if a device-side wait gave up since the last check (and clear it)."""
    check(library().nc_device_faults())


def selftest_wait(kind: int) -> None:
    """Make one of the bounded waits run out against a condition that never comes true (0: a
    hand-over word, 1: a pipeline stage); raises the :class:`KernelError` it reports."""
    check(library().nc_selftest_wait(int(kind)))


def _p(a: np.ndarray | None, kind):
    return ctypes.cast(None, kind) if a is None else a.ctypes.data_as(kind)


# -- the device model ------------------------------------------------------------------------


class DeviceModel:
    """One model resident on one GPU: weights, the KV cache of ``slots`` sequences, activations.

    ``activations`` is ``None`` (float32 projections), ``"int8"`` (int8-vnni: block-32 int8
    activations) or ``"f32"`` (int8 weights with float32 activations). ``weights`` are by
    checkpoint name; int8 modes take ``W@int8`` / ``W@scales`` pairs, or a float32 ``W`` that is
    then quantized on the device (``nc_qwen2_upload_quantize``, the same bytes as the host
    scheme). ``rope_rates`` default to the shape's ``theta``.
    """

    KINDS = ("gather", "qkv_projection", "attention", "o_projection", "gate_up_projection", "down_projection",
             "rms_norm", "block_quantize", "lm_head_argmax", "persistent_layers")

    def __init__(self, shape: ModelShape, weights: Mapping[str, np.ndarray], activations: str | None,
                 max_rows: int = 64, slots: int = 1, capacity: int = 2048, device: int = 0,
                 rope_rates: np.ndarray | None = None):
        if activations not in QUANT_CODES:
            raise ValueError(f"activations must be one of {sorted(QUANT_CODES, key=str)}, got {activations!r}")
        L = library()
        self.shape = shape
        self.activations = activations
        self.max_rows, self.slots, self.capacity, self.device = max_rows, slots, capacity, device
        self.rope_rates = np.ascontiguousarray(shape.rope_rates() if rope_rates is None else rope_rates, np.float32)
        s = shape
        cfg = NCConfig(s.vocab, s.hidden, s.inter, s.layers, s.heads, s.kv_heads, s.head_dim, np.float32(s.eps),
                       s.attention_scale, QUANT_CODES[activations], max_rows, slots, capacity, device)
        handle = _vp()
        check(L.nc_qwen2_create(ctypes.byref(cfg), _p(self.rope_rates, _PF), ctypes.byref(handle)))
        self._h = handle
        self.weights_source = weights
        started = time.perf_counter()
        self.upload(weights)
        self.upload_seconds = time.perf_counter() - started

    def upload(self, weights: Mapping[str, np.ndarray]) -> None:
        """Copy every array the step reads to the arena (float32 projections of an int8 model are
        quantized on the device)."""
        L = library()
        for name, array in weights.items():
            a = np.ascontiguousarray(array)
            quantize_here = (self.activations is not None and a.dtype == np.float32 and a.ndim == 2
                             and name.endswith("_proj.weight") and int8_name(name) not in weights)
            if quantize_here:
                check(L.nc_qwen2_upload_quantize(self._h, name.encode(), a.ctypes.data, a.nbytes))
            else:
                check(L.nc_qwen2_upload(self._h, name.encode(), a.ctypes.data, a.nbytes))
        missing = ctypes.c_int32(0)
        check(L.nc_qwen2_missing_weights(self._h, ctypes.byref(missing)))
        if missing.value:
            raise InterpreterError(f"missing weights: {last_error()}")

    @property
    def arena_bytes(self) -> int:
        return int(library().nc_qwen2_arena_bytes(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            library().nc_qwen2_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # KV cache of one slot, host arrays [layers, kv_heads, count, head_dim]
    def kv_write(self, slot: int, start: int, keys: np.ndarray, values: np.ndarray) -> None:
        k = np.ascontiguousarray(keys, np.float32)
        v = np.ascontiguousarray(values, np.float32)
        check(library().nc_qwen2_kv_write(self._h, slot, start, k.shape[2], _p(k, _PF), _p(v, _PF)))

    def kv_read(self, slot: int, start: int, count: int) -> tuple[np.ndarray, np.ndarray]:
        s = self.shape
        dims = (s.layers, s.kv_heads, count, s.head_dim)
        k = np.empty(dims, np.float32)
        v = np.empty(dims, np.float32)
        check(library().nc_qwen2_kv_read(self._h, slot, start, count, _p(k, _PF), _p(v, _PF)))
        return k, v

    def step(self, ids: Sequence[int], slot: Sequence[int], pos: Sequence[int], logit_rows: Sequence[int],
             want_logits: bool = True) -> tuple[np.ndarray | None, np.ndarray]:
        """One fused step on the device; returns (logits of ``logit_rows``, their argmax)."""
        ids = np.ascontiguousarray(ids, np.int64)
        slot = np.ascontiguousarray(slot, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        rows = np.ascontiguousarray(logit_rows, np.int32)
        logits = np.empty((rows.size, self.shape.vocab), np.float32) if want_logits else None
        tokens = np.empty(rows.size, np.int64)
        bad = ctypes.c_int32(-1)
        check(library().nc_qwen2_step(self._h, ids.size, _p(ids, _P64), _p(slot, _P32), _p(pos, _P32), rows.size,
                                      _p(rows, _P32), _p(logits, _PF), _p(tokens, _P64), ctypes.byref(bad)))
        return logits, tokens

    def run(self, ids: np.ndarray, slot: int, start: int, last_only: bool, want_logits: bool = True
            ) -> tuple[np.ndarray | None, np.ndarray | None]:
        """``ids`` at positions ``start..`` of ``slot``, in chunks of ``max_rows`` rows; returns the
        logits (of the last row with ``last_only``) and the argmax of the last chunk's logit rows."""
        out, tokens = [], None
        n = ids.size
        for lo in range(0, n, self.max_rows):
            chunk = ids[lo: lo + self.max_rows]
            rows = chunk.size
            logit_rows = ([rows - 1] if lo + rows == n else []) if last_only else list(range(rows))
            try:
                lg, tk = self.step(chunk, [slot] * rows, np.arange(start + lo, start + lo + rows), logit_rows,
                                   want_logits)
            except KernelError:
                bad = ids[(ids < 0) | (ids >= self.shape.vocab)]
                if bad.size:
                    raise KernelError(f"gather index {bad.flat[0]} is outside 0..{self.shape.vocab - 1}") from None
                raise
            if logit_rows:
                out.append(lg)
                tokens = tk
        return (np.concatenate(out) if want_logits else None), tokens

    def decode(self, first: Sequence[int], slot: Sequence[int], start: Sequence[int], steps: int,
               per_step: bool = False, want_logits: bool = False) -> tuple[np.ndarray, np.ndarray | None]:
        """Greedy decode of ``len(first)`` sequences for ``steps`` tokens each: tokens [steps, batch]."""
        first = np.ascontiguousarray(first, np.int64)
        slot = np.ascontiguousarray(slot, np.int32)
        start = np.ascontiguousarray(start, np.int32)
        tokens = np.empty((steps, first.size), np.int64)
        logits = np.empty((first.size, self.shape.vocab), np.float32) if want_logits else None
        check(library().nc_qwen2_decode(self._h, first.size, _p(slot, _P32), _p(first, _P64), _p(start, _P32), steps,
                                        1 if per_step else 0, _p(tokens, _P64), _p(logits, _PF)))
        return tokens, logits

    def profile(self, first: Sequence[int], slot: Sequence[int], start: Sequence[int], steps: int
                ) -> dict[str, tuple[float, int]]:
        """Per fused-group kind: (total milliseconds, launches) over ``steps`` eager decode steps
        with a CUDA event pair around every launch."""
        first = np.ascontiguousarray(first, np.int64)
        slot = np.ascontiguousarray(slot, np.int32)
        start = np.ascontiguousarray(start, np.int32)
        ms = np.zeros(len(self.KINDS), np.float32)
        n = np.zeros(len(self.KINDS), np.int32)
        check(library().nc_qwen2_profile(self._h, first.size, _p(slot, _P32), _p(first, _P64), _p(start, _P32), steps,
                                         _p(ms, _PF), _p(n, _P32)))
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(self.KINDS) if n[i]}

    PHASES = ("layer start", "input words in", "input norm", "q/k/v rows out", "q/k/v words in", "scores",
              "softmax", "attention out", "attention blocks in", "o rows out", "residual words in", "post norm",
              "gate/up staged", "SwiGLU out", "SwiGLU in", "down rows out")

    def phase_times(self, first: Sequence[int], slot: Sequence[int], start: Sequence[int], steps: int
                    ) -> dict[str, float]:
        """The persistent decode kernel's phase table over ``steps`` eager decode steps:
        microseconds from a layer's start to the last CTA reaching each event, averaged over layers
        and steps (globaltimer stamps)."""
        first = np.ascontiguousarray(first, np.int64)
        slot = np.ascontiguousarray(slot, np.int32)
        start = np.ascontiguousarray(start, np.int32)
        us = np.zeros(len(self.PHASES), np.float32)
        check(library().nc_qwen2_phase_times(self._h, first.size, _p(slot, _P32), _p(first, _P64), _p(start, _P32),
                                             steps, _p(us, _PF)))
        return {k: round(float(us[i]), 2) for i, k in enumerate(self.PHASES) if us[i] >= 0}

    def step_timed(self, ids: Sequence[int], slot: int, start: int, iters: int) -> float:
        """Average device milliseconds of ``iters`` eager steps of ``ids`` at positions ``start..``
        of ``slot`` (the last row's token only), timed with CUDA events on the model's stream."""
        ids = np.ascontiguousarray(ids, np.int64)
        slots = np.full(ids.size, slot, np.int32)
        pos = np.arange(start, start + ids.size, dtype=np.int32)
        ms = ctypes.c_float(0)
        check(library().nc_qwen2_step_timed(self._h, ids.size, _p(ids, _P64), _p(slots, _P32), _p(pos, _P32), iters,
                                            ctypes.byref(ms)))
        return float(ms.value)

    def probe(self, on: bool) -> dict[str, tuple[float, int]]:
        """Start (``on``) or stop timing every launch of the following :meth:`step` calls; stopping
        returns (milliseconds, launches) per fused-group kind since the start."""
        ms = np.zeros(len(self.KINDS), np.float32)
        n = np.zeros(len(self.KINDS), np.int32)
        check(library().nc_qwen2_probe(self._h, 1 if on else 0, _p(ms, _PF), _p(n, _P32)))
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(self.KINDS) if n[i]}

    def decode_timed(self, first: Sequence[int], slot: Sequence[int], start: Sequence[int], steps: int) -> float:
        """Milliseconds for ``steps`` graph replays, timed with CUDA events on the model's stream."""
        first = np.ascontiguousarray(first, np.int64)
        slot = np.ascontiguousarray(slot, np.int32)
        start = np.ascontiguousarray(start, np.int32)
        ms = ctypes.c_float(0)
        check(library().nc_qwen2_decode_timed(self._h, first.size, _p(slot, _P32), _p(first, _P64), _p(start, _P32),
                                              steps, ctypes.byref(ms)))
        return float(ms.value)


# -- the reference-facing compiled graph and backend -------------------------------------------


def _reference_errors():
    """The reference's exception classes, each also an instance of this module's own."""
    from nanocompile.interpreter import InterpreterError as RefInterpreterError
    from nanocompile.runtime import KernelError as RefKernelError

    kernel = type("KernelError", (RefKernelError, KernelError), {"__module__": __name__})
    interp = type("InterpreterError", (RefInterpreterError, InterpreterError), {"__module__": __name__})
    return kernel, interp


@dataclass(frozen=True)
class StepPlan:
    """What one call used: the device arena, the rows run, the KV history moved in and out."""

    arena_bytes: int
    rows: int
    past: int
    chunks: int
    kv_bytes_in: int
    kv_bytes_out: int


class CompiledGraph:
    """A reference step graph lowered by the CUDA target: call it like ``interpreter.run``.

    The twin of ``CompiledGraph`` (``nanocompile/runtime.py:167-318``). The weights arrive with
    the first call, as they do there; the device model they are uploaded into is shared by every
    graph of the same model on one backend (a model's ``graph`` and ``graph_last``).
    """

    def __init__(self, graph, backend: "CUDABackend"):
        from nanocompile_b200.target import lower_cuda

        started = time.perf_counter()
        self.graph = graph
        self.backend = backend
        self.cuda = lower_cuda(graph)
        self.program = self.cuda.program
        self.groups = self.cuda.groups
        self.source = self.cuda.source()
        self.library_path = LIBRARY_PATH
        self.cached = True                  # the kernels are compiled ahead of time, once
        self.last_plan: StepPlan | None = None
        self.compile_seconds = time.perf_counter() - started

    def device_model(self, weights: Mapping[str, np.ndarray]) -> DeviceModel:
        return self.backend.device_model(self.cuda, weights)

    def __call__(self, inputs: Mapping[str, np.ndarray], weights: Mapping[str, np.ndarray],
                 bindings: Mapping[str, int] | None = None, profile: dict[str, float] | None = None
                 ) -> dict[str, np.ndarray]:
        """One stateless step: the past KV comes from ``inputs`` (host) and the new KV goes back.
        ``profile``, if given, accumulates device seconds per CUDA fused-group kind."""
        from nanocompile.interpreter import check_arguments

        ref_kernel_error, ref_interpreter_error = _reference_errors()
        bound = check_arguments(self.graph, inputs, weights, bindings)
        seq, past = bound["seq"], bound["past"]
        model = self.device_model(weights)
        if seq == 0:
            raise ref_interpreter_error("a step needs at least one token")
        if past + seq > model.capacity:
            raise ref_interpreter_error(f"past {past} + seq {seq} exceeds the device cache capacity {model.capacity}; "
                                        f"give CUDABackend a larger capacity")
        ids = np.ascontiguousarray(inputs["token_ids"], np.int64)
        try:
            if past:
                model.kv_write(0, 0, inputs["past_keys"], inputs["past_values"])
            if profile is not None:
                model.probe(True)
            try:
                logits, _ = model.run(ids, slot=0, start=past, last_only=self.cuda.last_only)
            finally:
                if profile is not None:
                    for kind, (ms, _) in model.probe(False).items():
                        profile[kind] = profile.get(kind, 0.0) + ms / 1e3
            keys, values = model.kv_read(0, past, seq)
        except KernelError as error:
            raise ref_kernel_error(str(error)) from None
        except InterpreterError as error:
            raise ref_interpreter_error(str(error)) from None
        row_bytes = model.shape.layers * model.shape.kv_heads * model.shape.head_dim * 4 * 2
        self.last_plan = StepPlan(model.arena_bytes, seq, past, -(-seq // model.max_rows), past * row_bytes,
                                  seq * row_bytes)
        return {"logits": logits, "keys": keys, "values": values}


class CUDABackend:
    """A ``Runner`` for the reference's ``Qwen2``: compiles each graph once, on first use.

    ``nanocompile/runtime.py:321-337`` ``CBackend``, for the GPU. ``capacity`` bounds the
    positions a sequence may reach, ``slots`` how many device caches one model serves at once,
    ``max_rows`` the token rows of one launch (longer prompts run in chunks).
    """

    def __init__(self, device: int = 0, capacity: int = 2048, slots: int = 4, max_rows: int = 512):
        self.device, self.capacity, self.slots, self.max_rows = device, capacity, slots, max_rows
        self._compiled: dict[int, tuple[object, CompiledGraph]] = {}
        self._models: dict[tuple, tuple[Mapping, DeviceModel]] = {}

    def compiled(self, graph) -> CompiledGraph:
        entry = self._compiled.get(id(graph))
        if entry is None or entry[0] is not graph:
            entry = (graph, CompiledGraph(graph, self))
            self._compiled[id(graph)] = entry
        return entry[1]

    def __call__(self, graph, inputs, weights) -> dict[str, np.ndarray]:
        return self.compiled(graph)(inputs, weights)

    def device_model(self, cuda, weights: Mapping[str, np.ndarray]) -> DeviceModel:
        """The model for ``cuda``'s shape and mode with ``weights`` uploaded; made once per weights object."""
        key = (cuda.shape, cuda.activations, cuda.rope_rates.tobytes())
        entry = self._models.get(key)
        if entry is None or entry[0] is not weights:
            if entry is not None:
                entry[1].close()
            model = DeviceModel(cuda.shape, weights, cuda.activations, max_rows=self.max_rows, slots=self.slots,
                                capacity=self.capacity, device=self.device, rope_rates=cuda.rope_rates)
            entry = (weights, model)
            self._models[key] = entry
        return entry[1]

    def model_for(self, model) -> DeviceModel:
        """The device model behind a reference ``Qwen2`` that runs on this backend."""
        return self.compiled(model.graph_last).device_model(model.weights)


# -- device-resident decoding for a reference ``Qwen2`` ---------------------------------------------


def _backend_of(model) -> CUDABackend:
    backend = getattr(model, "run", None)
    if not isinstance(backend, CUDABackend):
        raise TypeError("device decoding needs a Qwen2 whose runner is a CUDABackend")
    return backend


class DeviceCache:
    """One sequence's keys and values in a slot of the device arena.

    The device twin of the reference's ``KVCache`` (``nanocompile/models/qwen2.py:232-271``):
    :meth:`forward` is ``Qwen2.forward`` with this cache, without moving the history.
    """

    def __init__(self, model, slot: int, capacity: int):
        backend = _backend_of(model)
        self.qwen2 = model
        self.device = backend.model_for(model)
        if not 0 <= slot < self.device.slots:
            raise InterpreterError(f"slot {slot} outside the backend's {self.device.slots} slots")
        if capacity > self.device.capacity:
            raise InterpreterError(f"a cache of {capacity} positions exceeds the backend's capacity "
                                   f"{self.device.capacity}")
        self.slot = slot
        self.length = 0
        self.capacity = capacity

    def _check_room(self, n: int) -> None:
        if self.length + n > self.capacity:
            raise InterpreterError(f"the device cache holds {self.capacity} positions; {self.length} + {n} do not fit")

    def past(self) -> tuple[np.ndarray, np.ndarray]:
        """Host copies of the filled region, ``[layers, kv_heads, length, head_dim]``."""
        return self.device.kv_read(self.slot, 0, self.length)

    def forward(self, token_ids: Sequence[int] | np.ndarray, last_only: bool = False) -> np.ndarray:
        ids = np.asarray(token_ids, np.int64)
        if ids.ndim != 1 or ids.size == 0:
            raise ValueError(f"expected a non-empty 1-D sequence of token IDs, got {ids.shape}")
        self._check_room(ids.size)
        logits, _ = self.device.run(ids, self.slot, self.length, last_only)
        self.length += ids.size
        return logits

    def greedy(self, prompt: Sequence[int], max_new_tokens: int) -> list[int]:
        """The prompt as one step, then ``max_new_tokens - 1`` replays of the captured decode graph."""
        if max_new_tokens <= 0:
            return []
        ids = np.asarray(prompt, np.int64)
        self._check_room(ids.size + max_new_tokens - 1)
        _, tokens = self.device.run(ids, self.slot, self.length, last_only=True, want_logits=False)
        self.length += ids.size
        generated = [int(tokens[0])]
        if max_new_tokens > 1:
            more, _ = self.device.decode(generated, [self.slot], [self.length], max_new_tokens - 1)
            generated += [int(t) for t in more[:, 0]]
            self.length += max_new_tokens - 1
        return generated


def new_device_cache(model, capacity: int, slot: int = 1) -> DeviceCache:
    """A device cache of ``capacity`` positions in ``slot`` of ``model``'s device arena (slot 0
    is the stateless runner's)."""
    return DeviceCache(model, slot if _backend_of(model).slots > 1 else 0, capacity)


def device_greedy(model, prompt_ids: Sequence[int], max_new_tokens: int) -> list[int]:
    """The reference's ``greedy`` (``nanocompile/models/qwen2.py:348-368``) with the history in HBM
    and the argmax on the device: the same tokens, one graph replay per token."""
    if not prompt_ids:
        raise ValueError("cannot generate from an empty prompt")
    return new_device_cache(model, len(prompt_ids) + max_new_tokens).greedy(prompt_ids, max_new_tokens)


def batched_greedy(model, first: Sequence[int], past_keys: Sequence[np.ndarray],
                   past_values: Sequence[np.ndarray], steps: int) -> np.ndarray:
    """Greedy decode of independent sequences together, one token each per step.

    Sequence ``b`` starts from ``first[b]`` after its history ``past_keys[b]`` /
    ``past_values[b]`` (``[layers, kv_heads, past, head_dim]``). Returns the tokens,
    ``[batch, steps]``. Each step is one replay of a captured graph over the batch.
    """
    backend = _backend_of(model)
    batch = len(first)
    if batch > backend.slots or batch > backend.max_rows:
        raise InterpreterError(f"{batch} sequences need a backend with at least that many slots and rows")
    device = backend.model_for(model)
    starts = []
    for b in range(batch):
        device.kv_write(b, 0, past_keys[b], past_values[b])
        starts.append(past_keys[b].shape[2])
    tokens, _ = device.decode(first, list(range(batch)), starts, steps)
    return tokens.T.copy()
