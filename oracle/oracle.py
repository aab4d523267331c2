"""ctypes front of the CPU oracle (TEST INFRASTRUCTURE: tests/, smoke() and bench.py's
cpu_baseline leg only; the product never imports this module).

``libnc_oracle.so`` restates the arithmetic of nanocompile's generated C for a Qwen2
step (see ``nc_oracle.c``); it is pinned bit for bit against golden vectors that
the reference itself produced (``tests/golden``).
"""

from __future__ import annotations

import ctypes
import subprocess
from collections.abc import Mapping, Sequence
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libnc_oracle.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)


class OrcConfig(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_int64), ("hidden", ctypes.c_int64), ("inter", ctypes.c_int64),
                ("layers", ctypes.c_int64), ("heads", ctypes.c_int64), ("kv_heads", ctypes.c_int64),
                ("head_dim", ctypes.c_int64), ("eps", ctypes.c_float), ("attn_scale", ctypes.c_float),
                ("quant", ctypes.c_int32), ("threads", ctypes.c_int32)]


_LAYER_F32 = ("in_norm", "post_norm", "bq", "bk", "bv", "wq", "wk", "wv", "wo", "wg", "wu", "wd")
_LAYER_I8 = ("qq", "qk", "qv", "qo", "qg", "qu", "qd")
_LAYER_S = ("sq", "sk", "sv", "so", "sg", "su", "sd")


class OrcLayer(ctypes.Structure):
    _fields_ = ([(n, _f32p) for n in _LAYER_F32] + [(n, _i8p) for n in _LAYER_I8]
                + [(n, _f32p) for n in _LAYER_S])


_LIB: ctypes.CDLL | None = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "libnc_oracle.so"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.orc_qwen2_step.restype = ctypes.c_int32
        L.orc_qwen2_step.argtypes = [ctypes.POINTER(OrcConfig), _f32p, _f32p, ctypes.POINTER(OrcLayer), _f32p,
                                     _i64p, ctypes.c_int64, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int32, _f32p, _f32p, _f32p, _i64p]
        L.orc_quantize_blocks.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, _i8p, _f32p, _f32p, _i32p]
        L.orc_matmul_i8_vnni.argtypes = [_i8p, _f32p, _f32p, _i8p, _f32p, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, _f32p, _i32p]
        L.orc_matmul_i8.argtypes = [_f32p, _i8p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.orc_rms_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, _f32p]
        L.orc_lm_head.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.orc_argmax.restype = ctypes.c_int64
        L.orc_argmax.argtypes = [_f32p, ctypes.c_int64]
        for name in ("orc_expf_libm", "orc_expf_restated", "orc_cosf_libm", "orc_sinf_libm"):
            getattr(L, name).restype = ctypes.c_float
            getattr(L, name).argtypes = [ctypes.c_float]
        L.orc_map.argtypes = [ctypes.c_int32, _f32p, ctypes.c_int64, _f32p]
        L.orc_swiglu.argtypes = [_f32p, _f32p, ctypes.c_int64, _f32p]
        L.orc_attention_decode.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int64, ctypes.c_float, _f32p, _f32p]
        _LIB = L
    return _LIB


def _ptr(a: np.ndarray | None, kind=_f32p):
    if a is None:
        return ctypes.cast(None, kind)
    return a.ctypes.data_as(kind)


# -- primitives ----------------------------------------------------------------------


def quantize_blocks(x: np.ndarray):
    """``(xq, xs, offset, block_sums)`` of ``x: f32[rows, k]`` (quantize.py:102-124)."""
    x = np.ascontiguousarray(x, np.float32)
    rows, k = x.shape
    xq = np.empty((rows, k), np.int8)
    xs = np.empty((rows, k // 32), np.float32)
    off = np.empty((rows, 1), np.float32)
    sums = np.empty((rows, k // 32), np.int32)
    lib().orc_quantize_blocks(_ptr(x), rows, k, _ptr(xq, _i8p), _ptr(xs), _ptr(off), _ptr(sums, _i32p))
    return xq, xs, off, sums


def matmul_i8_vnni(xq, xs, offset, q, scales, lanes: bool = False):
    """``out [rows, n]`` (and optionally the int32 Dp4 lanes ``[rows, n, k/4]``)."""
    xq = np.ascontiguousarray(xq, np.int8)
    rows, k = xq.shape
    n = q.shape[0]
    out = np.empty((rows, n), np.float32)
    lane_arr = np.empty((rows, n, k // 4), np.int32) if lanes else None
    lib().orc_matmul_i8_vnni(_ptr(xq, _i8p), _ptr(np.ascontiguousarray(xs, np.float32)),
                             _ptr(np.ascontiguousarray(offset, np.float32)), _ptr(np.ascontiguousarray(q, np.int8), _i8p),
                             _ptr(np.ascontiguousarray(scales, np.float32)), rows, n, k, _ptr(out),
                             _ptr(lane_arr, _i32p))
    return (out, lane_arr) if lanes else out


def matmul_i8(x, q, scales):
    """``out [rows, n]`` of int8 weights and float32 activations (``lower.py:320-356``)."""
    x = np.ascontiguousarray(x, np.float32)
    rows, k = x.shape
    n = q.shape[0]
    out = np.empty((rows, n), np.float32)
    lib().orc_matmul_i8(_ptr(x), _ptr(np.ascontiguousarray(q, np.int8), _i8p), _ptr(np.ascontiguousarray(scales, np.float32)),
                        rows, n, k, _ptr(out))
    return out


def rms_norm(x, w, eps: float, residual=None):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    res = None if residual is None else np.ascontiguousarray(residual, np.float32)
    lib().orc_rms_norm(_ptr(x), _ptr(res), _ptr(np.ascontiguousarray(w, np.float32)), x.shape[0], x.shape[1],
                       np.float32(eps), _ptr(out))
    return out


def lm_head(x, embed):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(embed.shape[0], np.float32)
    lib().orc_lm_head(_ptr(x), _ptr(np.ascontiguousarray(embed, np.float32)), embed.shape[0], embed.shape[1],
                      _ptr(out))
    return out


def argmax(v) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().orc_argmax(_ptr(v), v.size))


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    out = np.empty_like(g)
    lib().orc_swiglu(_ptr(g), _ptr(u), g.size, _ptr(out))
    return out


def _map(which: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_map(which, _ptr(x), x.size, _ptr(out))
    return out


def expf_libm(x: np.ndarray) -> np.ndarray:
    """glibc's expf, element-wise."""
    return _map(0, x)


def expf_restated(x: np.ndarray) -> np.ndarray:
    """The table-driven restatement of glibc's expf that the CUDA kernels use."""
    return _map(1, x)


def cosf_libm(x: np.ndarray) -> np.ndarray:
    return _map(2, x)


def sinf_libm(x: np.ndarray) -> np.ndarray:
    return _map(3, x)


def attention_decode(q, keys, values, heads: int, kv_heads: int, length: int, scale: float):
    """q ``[heads, d]``; keys/values ``[kv, cap, d]`` holding ``length`` positions."""
    q = np.ascontiguousarray(q, np.float32)
    keys = np.ascontiguousarray(keys, np.float32)
    values = np.ascontiguousarray(values, np.float32)
    d = q.shape[-1]
    out = np.empty((heads, d), np.float32)
    probs = np.empty((heads, length), np.float32)
    lib().orc_attention_decode(_ptr(q), _ptr(keys), _ptr(values), heads, kv_heads, length, d, keys.shape[1],
                               np.float32(scale), _ptr(out), _ptr(probs))
    return out, probs


# -- the whole step ------------------------------------------------------------------


class OracleModel:
    """The reference's step on the CPU, holding pointers into ``weights`` (kept alive here).

    ``weights`` are by checkpoint name, quantized ones as ``W@int8`` / ``W@scales``
    (``activations="int8"``) or float32 (``activations=None``).
    """

    def __init__(self, shape, weights: Mapping[str, np.ndarray], activations: str | None, threads: int = 0,
                 inv_freq: np.ndarray | None = None):
        if activations not in (None, "int8", "f32"):
            raise ValueError("the oracle implements float32, int8-vnni and int8 (float activations) projections")
        c = shape
        self.shape = c
        self.quant = {None: 0, "int8": 1, "f32": 2}[activations]
        self._keep: list[np.ndarray] = []
        self.cfg = OrcConfig(c.vocab, c.hidden, c.inter, c.layers, c.heads, c.kv_heads, c.head_dim,
                             np.float32(c.eps), c.attention_scale, self.quant, threads)

        def arr(name: str, dtype=np.float32) -> np.ndarray:
            a = np.ascontiguousarray(weights[name], dtype)
            self._keep.append(a)
            return a

        self.embed = arr("model.embed_tokens.weight")
        self.final_norm = arr("model.norm.weight")
        self.inv_freq = np.ascontiguousarray(c.rope_rates() if inv_freq is None else inv_freq, np.float32)
        layers = (OrcLayer * c.layers)()
        short = {"q_proj": "q", "k_proj": "k", "v_proj": "v", "o_proj": "o", "gate_proj": "g", "up_proj": "u",
                 "down_proj": "d"}
        for i in range(c.layers):
            p = f"model.layers.{i}"
            L = layers[i]
            L.in_norm = _ptr(arr(f"{p}.input_layernorm.weight"))
            L.post_norm = _ptr(arr(f"{p}.post_attention_layernorm.weight"))
            for b in ("q", "k", "v"):
                setattr(L, "b" + b, _ptr(arr(f"{p}.self_attn.{b}_proj.bias")))
            for full, s in short.items():
                base = f"{p}.{'mlp' if full in ('gate_proj', 'up_proj', 'down_proj') else 'self_attn'}.{full}.weight"
                if self.quant:
                    setattr(L, "q" + s, _ptr(arr(base + "@int8", np.int8), _i8p))
                    setattr(L, "s" + s, _ptr(arr(base + "@scales")))
                else:
                    setattr(L, "w" + s, _ptr(arr(base)))
        self.layers = layers

    def step(self, ids: Sequence[int], past_keys: np.ndarray, past_values: np.ndarray, last_only: bool = True):
        """``(logits, keys, values)`` for ``ids`` after the cached ``past_*`` ``[L, kv, cap, d]``."""
        c = self.shape
        ids = np.ascontiguousarray(np.asarray(ids, np.int64))
        seq = ids.size
        past = past_keys.shape[2] if past_keys is not None else 0
        pk = np.ascontiguousarray(past_keys, np.float32)
        pv = np.ascontiguousarray(past_values, np.float32)
        rows = 1 if last_only else seq
        logits = np.empty((rows, c.vocab), np.float32)
        shape = (c.layers, c.kv_heads, seq, c.head_dim)
        keys = np.empty(shape, np.float32)
        values = np.empty(shape, np.float32)
        bad = ctypes.c_int64(0)
        status = lib().orc_qwen2_step(ctypes.byref(self.cfg), _ptr(self.embed), _ptr(self.final_norm), self.layers,
                                      _ptr(self.inv_freq), _ptr(ids, _i64p), seq, _ptr(pk), _ptr(pv), past, past,
                                      1 if last_only else 0, _ptr(logits), _ptr(keys), _ptr(values),
                                      ctypes.byref(bad))
        if status != 0:
            raise IndexError(f"gather index {bad.value} is outside 0..{c.vocab - 1}")
        return logits, keys, values

    def greedy(self, prompt: Sequence[int], steps: int, past_keys=None, past_values=None,
               return_logits: bool = False):
        """Greedy decode: the reference's driver loop with a growing host cache."""
        c = self.shape
        shape = (c.layers, c.kv_heads, 0, c.head_dim)
        pk = np.zeros(shape, np.float32) if past_keys is None else past_keys
        pv = np.zeros(shape, np.float32) if past_values is None else past_values
        pending = list(prompt)
        tokens, all_logits = [], []
        for _ in range(steps):
            logits, k, v = self.step(pending, pk, pv, last_only=True)
            pk = np.concatenate([pk, k], axis=2)
            pv = np.concatenate([pv, v], axis=2)
            tok = argmax(logits[0])
            tokens.append(tok)
            if return_logits:
                all_logits.append(logits[0].copy())
            pending = [tok]
        return (tokens, np.array(all_logits)) if return_logits else tokens
