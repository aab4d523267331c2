"""Per-row int8 weights and the activation scheme of nanocompile's ``int8-vnni`` mode.

Host side, once per model: the projection weights are quantized here in NumPy,
exactly as nanocompile's ``quantize.quantize_int8`` does it
(``nanocompile/quantize.py:55-70``): one float32 scale per output row,
``max(|row|) / 127`` with an all-zero row getting scale 1, and the row divided
by it and rounded half away from zero as ``sign(x) * floor(|x| + 0.5)`` in
float32. The device never sees float32 projection weights in this mode.

The activations are quantized on the device, per 32-value block, by the fused
kernels (``nanocompile/quantize.py:102-124``); ``BLOCK`` is that block.
"""

from __future__ import annotations

from collections.abc import Iterable, Mapping

import numpy as np

INT8_MAX = 127
BLOCK = 32                     # nanocompile/quantize.py:43 DEFAULT_BLOCK
ACTIVATIONS = ("f32", "int8")  # nanocompile/quantize.py:42


def int8_name(name: str) -> str:
    """``nanocompile/quantize.py:47``: the int8 values of weight ``name``."""
    return f"{name}@int8"


def scales_name(name: str) -> str:
    """``nanocompile/quantize.py:51``: the per-row float32 scales of weight ``name``."""
    return f"{name}@scales"


def quantize_int8(weights: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``[out, in]`` float32 to per-row int8 values and float32 scales.

    The same NumPy operations in the same order as ``nanocompile/quantize.py:55-70``,
    so the bytes and scales are identical.
    """
    if weights.ndim != 2:
        raise ValueError(f"expected a 2-D weight matrix, got shape {weights.shape}")
    weights = weights.astype(np.float32, copy=False)
    scales = np.max(np.abs(weights), axis=1) / INT8_MAX
    scales[scales == 0] = 1.0
    scaled = weights / scales[:, None]
    rounded = np.sign(scaled) * np.floor(np.abs(scaled) + 0.5)
    values = np.clip(rounded, -INT8_MAX, INT8_MAX).astype(np.int8)
    return values, scales.astype(np.float32)


def quantized_weights(graph, weights: Mapping[str, np.ndarray]) -> dict[str, np.ndarray]:
    """The arrays ``graph`` reads, quantizing the int8 ones it names from ``weights``.

    ``nanocompile/quantize.py:167-180``: a name already in ``weights`` is passed
    through; ``W@int8`` / ``W@scales`` are made from ``weights[W]``; anything
    else is a ``KeyError``.
    """
    out: dict[str, np.ndarray] = {}
    for name in graph.weights:
        if name in weights:
            out[name] = weights[name]
            continue
        if name.endswith("@int8") or name.endswith("@scales"):
            source = name.rsplit("@", 1)[0]
            if int8_name(source) not in out:
                out[int8_name(source)], out[scales_name(source)] = quantize_int8(weights[source])
            continue
        raise KeyError(f"no weight {name!r}")
    return out


def projection_names(layers: int, keep: Iterable[str] = ()) -> list[str]:
    """The weights a Qwen2 step reads only as ``x @ W.T`` (``nanocompile/quantize.py:86-99``).

    The tied embedding is also the LM head, and a gather table, so it is never
    among them; ``keep`` removes more.
    """
    kept = set(keep)
    names = []
    for i in range(layers):
        p = f"model.layers.{i}"
        for n in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                  "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
            name = f"{p}.{n}.weight"
            if name not in kept:
                names.append(name)
    return names
