"""The CUDA runtime: one ``libnc_cuda.so`` over ctypes, with nanocompile's runtime API.

This is the CUDA twin of ``nanocompile/runtime.py``:

* :class:`CUDABackend` is a ``Runner`` for :class:`~nanocompile_b200.qwen2.Qwen2`, as
  ``CBackend`` is (``nanocompile/runtime.py:321-337``): it compiles each step graph once,
  on first use, and is then called per step with host arrays.
* :class:`CompiledStep` plays ``CompiledGraph`` (``nanocompile/runtime.py:167-318``):
  ``step(inputs, weights) -> {"logits", "keys", "values"}``, argument errors raised
  with the interpreter's messages, a failing kernel raised as :class:`KernelError`
  with the reference's text.
* :class:`DeviceKVCache` is what the reference's phase 7 planned: the KV history lives in
  the device arena, so a cached step moves only token ids in and logits out, and greedy
  decode replays one captured CUDA graph per token with the argmax fused into the LM head.

There is no CPU path: without the compiled library on a machine with a GPU, every
entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import time
from collections.abc import Mapping, Sequence
from pathlib import Path

import numpy as np

from nanocompile_b200.qwen2 import Qwen2, Qwen2Config, StepGraph, attention_scale, inverse_frequencies

LIBRARY_PATH = Path(__file__).resolve().parent / "libnc_cuda.so"

NC_OK, NC_ERR_KERNEL, NC_ERR_ARGUMENT, NC_ERR_CUDA, NC_ERR_STATE = 0, 1, 2, 3, 4


class KernelError(RuntimeError):
    """A kernel rejected its input (an out-of-range gather index): ``nanocompile/runtime.py:49``."""


class InterpreterError(RuntimeError):
    """Inputs that do not fit the graph: the reference's ``interpreter.InterpreterError`` messages."""


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
        for name in ("nc_gather_rows", "nc_rms_norm_quantize", "nc_quantize_blocks", "nc_matmul_i8_vnni",
                     "nc_matmul_f32", "nc_lm_head_argmax", "nc_lm_head_argmax_noalloc", "nc_attention",
                     "nc_attention_cache", "nc_expf_exact", "nc_lm_head_q8_prepare", "nc_lm_head_q8_argmax"):
            fn = getattr(L, name)
            fn.argtypes = [ctypes.POINTER(_vp), _P64, _vp]
            fn.restype = _i32
        L.nc_device_faults.argtypes = []
        L.nc_device_faults.restype = _i32
        L.nc_selfcheck_div127.argtypes = [_P64]
        L.nc_selfcheck_div127.restype = _i32
        L.nc_lm_head_scratch_bytes.argtypes = [_i64, _i64]
        L.nc_lm_head_scratch_bytes.restype = _i64
        L.nc_lm_head_q8_scratch_bytes.argtypes = [_i64, _i64]
        L.nc_lm_head_q8_scratch_bytes.restype = _i64
        L.nc_device_count.argtypes = [_P32]
        L.nc_set_device.argtypes = [_i32]
        L.nc_device_alloc.argtypes = [_i64, ctypes.POINTER(_vp)]
        L.nc_device_free.argtypes = [_vp]
        L.nc_copy_to_device.argtypes = [_vp, _vp, _i64]
        L.nc_copy_to_host.argtypes = [_vp, _vp, _i64]
        L.nc_pack_int8_weights.argtypes = [_vp, _vp, _i64]
        L.nc_qwen2_create.argtypes = [ctypes.POINTER(NCConfig), _PF, ctypes.POINTER(_vp)]
        L.nc_qwen2_destroy.argtypes = [_vp]
        L.nc_qwen2_arena_bytes.argtypes = [_vp]
        L.nc_qwen2_arena_bytes.restype = _i64
        L.nc_qwen2_upload.argtypes = [_vp, ctypes.c_char_p, _vp, _i64]
        L.nc_qwen2_missing_weights.argtypes = [_vp, _P32]
        L.nc_qwen2_kv_write.argtypes = [_vp, _i32, _i64, _i64, _PF, _PF]
        L.nc_qwen2_kv_read.argtypes = [_vp, _i32, _i64, _i64, _PF, _PF]
        L.nc_qwen2_step.argtypes = [_vp, _i32, _P64, _P32, _P32, _i32, _P32, _PF, _P64, _P32]
        L.nc_qwen2_decode.argtypes = [_vp, _i32, _P32, _P64, _P32, _i32, _i32, _P64, _PF]
        L.nc_qwen2_decode_timed.argtypes = [_vp, _i32, _P32, _P64, _P32, _i32, _PF]
        L.nc_qwen2_profile.argtypes = [_vp, _i32, _P32, _P64, _P32, _i32, _PF, _P32]
        L.nc_qwen2_profile.restype = _i32
        for fn in ("nc_device_count", "nc_set_device", "nc_device_alloc", "nc_device_free", "nc_copy_to_device",
                   "nc_copy_to_host", "nc_pack_int8_weights", "nc_qwen2_create", "nc_qwen2_destroy",
                   "nc_qwen2_upload", "nc_qwen2_missing_weights", "nc_qwen2_kv_write", "nc_qwen2_kv_read",
                   "nc_qwen2_step", "nc_qwen2_decode", "nc_qwen2_decode_timed", "nc_device_synchronize"):
            getattr(L, fn).restype = _i32
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


def _p(a: np.ndarray | None, kind):
    return ctypes.cast(None, kind) if a is None else a.ctypes.data_as(kind)


# -- the device model ----------------------------------------------------------------------


class DeviceModel:
    """One model resident on one GPU: weights, the KV cache of ``slots`` sequences, activations.

    ``activations`` is ``None`` (float32 projections) or ``"int8"`` (int8-vnni).
    """

    def __init__(self, config: Qwen2Config, weights: Mapping[str, np.ndarray], activations: str | None,
                 max_rows: int = 64, slots: int = 1, capacity: int = 2048, device: int = 0):
        if activations not in (None, "int8"):
            raise NotImplementedError("the CUDA target implements float32 and int8-vnni projections; "
                                      "int8 weights with float32 activations (matmul_i8) are not implemented")
        if not config.tie_word_embeddings:
            raise NotImplementedError("the CUDA target implements the tied LM head of Qwen2.5-0.5B")
        L = library()
        c = config
        self.config = c
        self.activations = activations
        self.max_rows, self.slots, self.capacity, self.device = max_rows, slots, capacity, device
        self.inv_freq = inverse_frequencies(c.head_dim, c.rope_theta)
        cfg = NCConfig(c.vocab_size, c.hidden_size, c.intermediate_size, c.num_hidden_layers, c.num_attention_heads,
                       c.num_key_value_heads, c.head_dim, np.float32(c.rms_norm_eps), attention_scale(c.head_dim),
                       1 if activations == "int8" else 0, max_rows, slots, capacity, device)
        handle = _vp()
        check(L.nc_qwen2_create(ctypes.byref(cfg), _p(self.inv_freq, _PF), ctypes.byref(handle)))
        self._h = handle
        self.weights_source = weights
        started = time.perf_counter()
        for name, array in weights.items():
            if name == "lm_head.weight":
                continue
            a = np.ascontiguousarray(array)
            check(L.nc_qwen2_upload(self._h, name.encode(), a.ctypes.data, a.nbytes))
        missing = ctypes.c_int32(0)
        check(L.nc_qwen2_missing_weights(self._h, ctypes.byref(missing)))
        if missing.value:
            raise InterpreterError(f"missing weights: {last_error()}")
        self.upload_seconds = time.perf_counter() - started

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
        c = self.config
        shape = (c.num_hidden_layers, c.num_key_value_heads, count, c.head_dim)
        k = np.empty(shape, np.float32)
        v = np.empty(shape, np.float32)
        check(library().nc_qwen2_kv_read(self._h, slot, start, count, _p(k, _PF), _p(v, _PF)))
        return k, v

    def step(self, ids: Sequence[int], slot: Sequence[int], pos: Sequence[int], logit_rows: Sequence[int],
             want_logits: bool = True) -> tuple[np.ndarray | None, np.ndarray]:
        """One fused step on the device; returns (logits of ``logit_rows``, their argmax)."""
        ids = np.ascontiguousarray(ids, np.int64)
        slot = np.ascontiguousarray(slot, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        rows = np.ascontiguousarray(logit_rows, np.int32)
        logits = np.empty((rows.size, self.config.vocab_size), np.float32) if want_logits else None
        tokens = np.empty(rows.size, np.int64)
        bad = ctypes.c_int32(-1)
        check(library().nc_qwen2_step(self._h, ids.size, _p(ids, _P64), _p(slot, _P32), _p(pos, _P32), rows.size,
                                      _p(rows, _P32), _p(logits, _PF), _p(tokens, _P64), ctypes.byref(bad)))
        return logits, tokens

    def decode(self, first: Sequence[int], slot: Sequence[int], start: Sequence[int], steps: int,
               per_step: bool = False, want_logits: bool = False) -> tuple[np.ndarray, np.ndarray | None]:
        """Greedy decode of ``len(first)`` sequences for ``steps`` tokens each: tokens [steps, batch]."""
        first = np.ascontiguousarray(first, np.int64)
        slot = np.ascontiguousarray(slot, np.int32)
        start = np.ascontiguousarray(start, np.int32)
        tokens = np.empty((steps, first.size), np.int64)
        logits = np.empty((first.size, self.config.vocab_size), np.float32) if want_logits else None
        check(library().nc_qwen2_decode(self._h, first.size, _p(slot, _P32), _p(first, _P64), _p(start, _P32), steps,
                                        1 if per_step else 0, _p(tokens, _P64), _p(logits, _PF)))
        return tokens, logits

    KINDS = ("gather", "qkv_projection", "attention", "o_projection", "gate_up_projection", "down_projection",
             "rms_norm", "block_quantize", "lm_head_argmax", "persistent_layers")

    def profile(self, first: Sequence[int], slot: Sequence[int], start: Sequence[int], steps: int
                ) -> dict[str, tuple[float, int]]:
        """Per fused-group kind: (total milliseconds, launches) over ``steps`` eager steps with a
        CUDA event pair around every launch."""
        first = np.ascontiguousarray(first, np.int64)
        slot = np.ascontiguousarray(slot, np.int32)
        start = np.ascontiguousarray(start, np.int32)
        ms = np.zeros(len(self.KINDS), np.float32)
        n = np.zeros(len(self.KINDS), np.int32)
        check(library().nc_qwen2_profile(self._h, first.size, _p(slot, _P32), _p(first, _P64), _p(start, _P32), steps,
                                         _p(ms, _PF), _p(n, _P32)))
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


# -- argument checks with the reference interpreter's messages -------------------------------

_DTYPE_NAMES = {np.dtype(np.int64): "i64", np.dtype(np.float32): "f32", np.dtype(np.int8): "i8",
                np.dtype(np.int32): "i32"}


def check_arguments(graph: StepGraph, inputs: Mapping[str, np.ndarray], weights: Mapping[str, np.ndarray]
                    ) -> dict[str, int]:
    """``nanocompile/interpreter.py:87-106``: names, symbol bindings, dtypes, shapes."""
    names = set(graph.input_names)
    unknown, missing = sorted(set(inputs) - names), sorted(names - set(inputs))
    if unknown or missing:
        raise InterpreterError(f"inputs: missing {missing}, unexpected {unknown}")
    c = graph.config
    ids, pk, pv = (np.asarray(inputs[n]) for n in graph.input_names)
    bound: dict[str, int] = {}
    for name, array, axes in (("token_ids", ids, {0: "seq"}), ("past_keys", pk, {2: "past"}),
                              ("past_values", pv, {2: "past"})):
        for axis, sym in axes.items():
            if array.ndim <= axis:
                continue
            size = array.shape[axis]
            if bound.setdefault(sym, size) != size:
                raise InterpreterError(f"{name!r} axis {axis} has size {size}, but {sym} is already bound to {bound[sym]}")
    for name, array, dtype, shape in (
            ("token_ids", ids, np.int64, (bound.get("seq", -1),)),
            ("past_keys", pk, np.float32, (c.num_hidden_layers, c.num_key_value_heads, bound.get("past", -1), c.head_dim)),
            ("past_values", pv, np.float32, (c.num_hidden_layers, c.num_key_value_heads, bound.get("past", -1), c.head_dim))):
        if array.dtype != dtype:
            raise InterpreterError(f"input {name!r} is {array.dtype}, expected {_DTYPE_NAMES[np.dtype(dtype)]}")
        if array.shape != shape:
            raise InterpreterError(f"input {name!r} has shape {array.shape}, expected {shape}")
    missing_w = sorted(set(graph.weights) - set(weights))
    if missing_w:
        raise InterpreterError(f"missing weights: {', '.join(missing_w[:5])}")
    for name, (dtype, shape) in graph.weights.items():
        array = weights[name]
        if array.dtype != dtype or tuple(array.shape) != shape:
            raise InterpreterError(f"weight {name!r} is {array.dtype}{list(array.shape)}, "
                                   f"expected {_DTYPE_NAMES[dtype]}{list(shape)}")
    return bound


def _kernel_error(message: str, ids: np.ndarray, vocab: int) -> KernelError:
    bad = ids[(ids < 0) | (ids >= vocab)]
    if bad.size:
        return KernelError(f"gather index {bad.flat[0]} is outside 0..{vocab - 1}")
    return KernelError(message)


# -- the compiled step and the backend ----------------------------------------------------------


FUSED_GROUPS = (
    "gather", "row: rms_norm + block quantize", "matmul_i8_vnni + bias (q, k, v)",
    "rope + kv append + attention", "block quantize", "matmul_i8_vnni + residual (o)",
    "row: rms_norm + block quantize", "matmul_i8_vnni + silu*up (gate, up)", "block quantize",
    "matmul_i8_vnni + residual (down)", "row: final rms_norm", "matmul (tied lm head) + argmax",
)


class CompiledStep:
    """A step graph made resident on the device: call it like ``interpreter.run``.

    The twin of ``CompiledGraph`` (``nanocompile/runtime.py:167-318``). ``program``
    names the fused groups each step launches; ``compile_seconds`` is the time to
    create the arena and upload the weights.
    """

    def __init__(self, graph: StepGraph, weights: Mapping[str, np.ndarray], device: int = 0, max_rows: int = 512,
                 slots: int = 1, capacity: int = 2048):
        started = time.perf_counter()
        self.graph = graph
        self.library_path = LIBRARY_PATH
        self.cached = True
        per_layer = FUSED_GROUPS[1:10]
        self.program = [FUSED_GROUPS[0]] + list(per_layer) * graph.config.num_hidden_layers + list(FUSED_GROUPS[10:])
        self.model = DeviceModel(graph.config, weights, graph.activations, max_rows=max_rows, slots=slots,
                                 capacity=capacity, device=device)
        self.weights = weights
        self.compile_seconds = time.perf_counter() - started

    def __call__(self, inputs: Mapping[str, np.ndarray], weights: Mapping[str, np.ndarray],
                 bindings: Mapping[str, int] | None = None, profile: dict[str, float] | None = None,
                 graph: StepGraph | None = None) -> dict[str, np.ndarray]:
        """One stateless step: the past KV comes from ``inputs`` (host) and the new KV goes back.

        ``graph`` (default: the compiled one) picks ``last_only``; both variants of a
        step share one compiled model."""
        graph = graph or self.graph
        bound = check_arguments(graph, inputs, weights)
        ids = np.ascontiguousarray(inputs["token_ids"], np.int64)
        seq, past = bound["seq"], bound["past"]
        started = time.perf_counter()
        if seq == 0:
            raise InterpreterError("a step needs at least one token")
        if past + seq > self.model.capacity:
            raise InterpreterError(f"past {past} + seq {seq} exceeds the device cache capacity {self.model.capacity}")
        if past:
            self.model.kv_write(0, 0, inputs["past_keys"], inputs["past_values"])
        logits = self._run(ids, slot=0, start=past, last_only=graph.last_only)
        keys, values = self.model.kv_read(0, past, seq)
        if profile is not None:
            profile["step"] = profile.get("step", 0.0) + time.perf_counter() - started
        return {"logits": logits, "keys": keys, "values": values}

    def _run(self, ids: np.ndarray, slot: int, start: int, last_only: bool, want_logits: bool = True):
        """Run ``ids`` at positions start.. of ``slot``, in chunks of ``max_rows``."""
        out = []
        tokens = None
        n = ids.size
        for lo in range(0, n, self.model.max_rows):
            chunk = ids[lo: lo + self.model.max_rows]
            rows = chunk.size
            if last_only:
                logit_rows = [rows - 1] if lo + rows == n else []
            else:
                logit_rows = list(range(rows))
            try:
                lg, tokens_c = self.model.step(chunk, [slot] * rows, np.arange(start + lo, start + lo + rows),
                                               logit_rows, want_logits)
            except KernelError as error:
                raise _kernel_error(str(error), ids, self.graph.config.vocab_size) from None
            if logit_rows:
                out.append(lg)
                tokens = tokens_c
        self.last_tokens = tokens
        return np.concatenate(out) if want_logits else None


class DeviceKVCache:
    """One sequence's keys and values in the device arena (a slot of the step's model)."""

    def __init__(self, compiled: CompiledStep, slot: int, capacity: int):
        self.compiled = compiled
        self.slot = slot
        self.length = 0
        self._capacity = capacity

    @property
    def capacity(self) -> int:
        return self._capacity

    def past(self) -> tuple[np.ndarray, np.ndarray]:
        """Host copies of the filled region, ``[layers, kv_heads, length, head_dim]``."""
        return self.compiled.model.kv_read(self.slot, 0, self.length)

    def _check_room(self, n: int) -> None:
        if self.length + n > self.compiled.model.capacity:
            raise InterpreterError(f"the device cache holds {self.compiled.model.capacity} positions; "
                                   f"{self.length} + {n} do not fit")

    def forward(self, graph: StepGraph, token_ids: np.ndarray, weights) -> np.ndarray:
        self._check_room(token_ids.size)
        logits = self.compiled._run(token_ids, self.slot, self.length, graph.last_only)
        self.length += token_ids.size
        return logits

    def greedy(self, graph: StepGraph, prompt: Sequence[int], max_new_tokens: int, weights) -> list[int]:
        """Prompt step, then ``max_new_tokens - 1`` replays of the captured decode graph."""
        if max_new_tokens <= 0:
            return []
        ids = np.asarray(prompt, np.int64)
        self._check_room(ids.size + max_new_tokens - 1)
        self.compiled._run(ids, self.slot, self.length, last_only=True, want_logits=False)
        self.length += ids.size
        first = int(self.compiled.last_tokens[0])
        generated = [first]
        if max_new_tokens > 1:
            tokens, _ = self.compiled.model.decode([first], [self.slot], [self.length], max_new_tokens - 1)
            generated += [int(t) for t in tokens[:, 0]]
            self.length += max_new_tokens - 1
        return generated


class CUDABackend:
    """A ``Runner`` for ``Qwen2``: the step graph compiled once per weights, on first use.

    ``nanocompile/runtime.py:321-337`` ``CBackend``, for the GPU. ``slots`` bounds how
    many device caches one model serves at once, ``capacity`` their length.
    """

    def __init__(self, device: int = 0, capacity: int = 2048, slots: int = 4, max_rows: int = 512):
        self.device, self.capacity, self.slots, self.max_rows = device, capacity, slots, max_rows
        self._compiled: dict[tuple, CompiledStep] = {}
        self._next_slot: dict[tuple, int] = {}

    def _key(self, graph: StepGraph, weights) -> tuple:
        return (graph.config, graph.activations, id(weights))

    def compiled(self, graph: StepGraph, weights: Mapping[str, np.ndarray]) -> CompiledStep:
        key = self._key(graph, weights)
        entry = self._compiled.get(key)
        if entry is None or entry.weights is not weights:
            entry = CompiledStep(graph, weights, self.device, self.max_rows, self.slots, self.capacity)
            self._compiled[key] = entry
            self._next_slot[key] = 1          # slot 0 serves stateless calls
        return entry

    def __call__(self, graph: StepGraph, inputs, weights) -> dict[str, np.ndarray]:
        return self.compiled(graph, weights)(inputs, weights, graph=graph)

    def new_cache(self, graph: StepGraph, weights, capacity: int) -> DeviceKVCache:
        compiled = self.compiled(graph, weights)
        key = self._key(graph, weights)
        slot = self._next_slot[key]
        if slot >= compiled.model.slots:
            slot = 1 if compiled.model.slots > 1 else 0
        self._next_slot[key] = slot + 1
        if capacity > compiled.model.capacity:
            raise InterpreterError(f"a cache of {capacity} positions exceeds the backend's capacity "
                                   f"{compiled.model.capacity}")
        return DeviceKVCache(compiled, slot, capacity)


def batched_greedy(model: Qwen2, first: Sequence[int], past_keys: Sequence[np.ndarray],
                   past_values: Sequence[np.ndarray], steps: int) -> np.ndarray:
    """Greedy decode of independent sequences together, one token each per step.

    Sequence ``b`` starts from ``first[b]`` after its history ``past_keys[b]`` /
    ``past_values[b]`` (``[layers, kv_heads, past, head_dim]``). Returns the tokens,
    ``[batch, steps]``. Each step is one replay of a captured graph over the batch.
    """
    backend = model.run
    if not isinstance(backend, CUDABackend):
        raise TypeError("batched_greedy needs a CUDABackend runner")
    batch = len(first)
    if batch > backend.slots or batch > backend.max_rows:
        raise InterpreterError(f"{batch} sequences need a backend with at least that many slots and rows")
    compiled = backend.compiled(model.graph_last, model.weights)
    starts = []
    for b in range(batch):
        compiled.model.kv_write(b, 0, past_keys[b], past_values[b])
        starts.append(past_keys[b].shape[2])
    tokens, _ = compiled.model.decode(first, list(range(batch)), starts, steps)
    return tokens.T.copy()
