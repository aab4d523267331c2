"""Per-row int8 weights and the activation scheme of nanocompile's ``int8-vnni`` mode.

One float32 scale per output row, ``max(|row|) / 127`` with an all-zero row getting scale 1,
and the row divided by it and rounded half away from zero as ``sign(x) * floor(|x| + 0.5)``
in float32, clipped to +-127 (``nanocompile/quantize.py:55-70``). The projections are quantized
once per model: on the host here (:func:`quantize_int8`), or on the device from the float32
weights by ``nc_quantize_int8_rows`` with the same bytes. The device never reads float32
projection weights in this mode.

The activations are quantized on the device, per 32-value block, by the fused kernels
(``nanocompile/quantize.py:102-124``); ``BLOCK`` is that block.
"""

from __future__ import annotations

from collections.abc import Mapping

import numpy as np

from nanocompile_b200.model import ModelShape, projection_shapes

INT8_MAX = 127
BLOCK = 32                     # nanocompile/quantize.py:43 DEFAULT_BLOCK


def int8_name(name: str) -> str:
    """The int8 values of projection ``name`` (``nanocompile/quantize.py:47``)."""
    return f"{name}@int8"


def scales_name(name: str) -> str:
    """The per-row float32 scales of projection ``name`` (``nanocompile/quantize.py:51``)."""
    return f"{name}@scales"


def quantize_int8(weights: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``[out, in]`` float32 to per-row int8 values and float32 scales.

    The NumPy operations of ``nanocompile/quantize.py:55-70`` in the same order -- the scheme's
    bytes are only the reference's if every rounding is the same one.
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


def int8_projection_weights(weights: Mapping[str, np.ndarray], shape: ModelShape) -> dict[str, np.ndarray]:
    """``weights`` with every layer's seven projections replaced by their ``@int8`` / ``@scales`` pair.

    Arrays already given in quantized form are kept as they are; the tied embedding (also the LM
    head and a gather table) and the norms and biases stay float32.
    """
    out: dict[str, np.ndarray] = {}
    projections = {name for layer in range(shape.layers) for name in projection_shapes(shape, layer)}
    for name, array in weights.items():
        if name not in projections:
            out[name] = array
    for name in sorted(projections):
        if int8_name(name) in weights and scales_name(name) in weights:
            continue
        if name not in weights:
            raise KeyError(f"no weight {name!r} to quantize")
        out[int8_name(name)], out[scales_name(name)] = quantize_int8(np.asarray(weights[name]))
    return out
