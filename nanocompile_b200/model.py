"""What a Qwen2 step on the device is sized by, and the seeded synthetic inputs of the workloads.

The reference describes a model by its ``Qwen2Config`` (``nanocompile/models/qwen2.py:45-96``)
and its step by an IR graph. The device step needs only the numbers its arena and kernels are
sized by, :class:`ModelShape`; the CUDA target (``nanocompile_b200.target``) reads them off the
reference's graph, and :meth:`ModelShape.of` takes them from any object with the config's fields.

Weights are named as in the HuggingFace checkpoint the reference binds them by
(``model.layers.N.self_attn.q_proj.weight`` ...; ``W@int8`` / ``W@scales`` for a quantized
projection, ``nanocompile/quantize.py:47-52``): that naming is the interface both sides share.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ModelShape:
    """The sizes and constants of one Qwen2 step with tied embeddings.

    ``eps`` is the RMSNorm epsilon as the step's float32 constant; ``theta`` the RoPE base,
    used only when the caller has no rotation rates of its own (a reference graph carries
    them as a constant, and those are used as they are).
    """

    vocab: int
    hidden: int
    inter: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    eps: float = 1e-6
    theta: float = 1e6

    def __post_init__(self) -> None:
        object.__setattr__(self, "eps", float(np.float32(self.eps)))      # the step's float32 constant
        if min(self.vocab, self.hidden, self.inter, self.layers, self.heads, self.kv_heads, self.head_dim) <= 0:
            raise ValueError(f"every size of {self} must be positive")
        if self.heads % self.kv_heads:
            raise ValueError(f"{self.heads} query heads do not share {self.kv_heads} KV heads evenly")
        if self.head_dim % 2:
            raise ValueError("RoPE rotates pairs: head_dim must be even")

    @classmethod
    def of(cls, config) -> "ModelShape":
        """From an object with ``Qwen2Config``'s fields (the reference's, or a dict-like record)."""
        get = (lambda k: config[k]) if isinstance(config, dict) else (lambda k: getattr(config, k))
        hidden, heads = int(get("hidden_size")), int(get("num_attention_heads"))
        if not bool(get("tie_word_embeddings")):
            raise NotImplementedError("the CUDA step implements Qwen2's tied LM head (tie_word_embeddings=True)")
        return cls(int(get("vocab_size")), hidden, int(get("intermediate_size")), int(get("num_hidden_layers")),
                   heads, int(get("num_key_value_heads")), hidden // heads, float(get("rms_norm_eps")),
                   float(get("rope_theta")))

    def config_fields(self) -> dict:
        """The reference ``Qwen2Config``'s keyword arguments for this shape."""
        return {"vocab_size": self.vocab, "hidden_size": self.hidden, "intermediate_size": self.inter,
                "num_hidden_layers": self.layers, "num_attention_heads": self.heads,
                "num_key_value_heads": self.kv_heads, "rms_norm_eps": self.eps, "rope_theta": self.theta,
                "tie_word_embeddings": True}

    @property
    def q_rows(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_rows(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def kv_shape_per_position(self) -> tuple[int, int, int]:
        return (self.layers, self.kv_heads, self.head_dim)

    def rope_rates(self) -> np.ndarray:
        """The per-plane rotation rates ``1 / theta^(2j/d)`` as float32.

        The float32 NumPy expression of ``nanocompile/nn.py:69-75``: NumPy's float32 ``power``
        rounds differently from libm's ``powf`` at theta = 1e6, so only this expression gives
        the reference's bits.
        """
        exponent = np.arange(0, self.head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(self.head_dim)
        return (np.float32(1.0) / (np.float32(self.theta) ** exponent)).astype(np.float32)

    @property
    def attention_scale(self) -> np.float32:
        """``np.float32(d ** -0.5)``, the score scale (``nanocompile/models/qwen2.py:149``)."""
        return np.float32(self.head_dim ** -0.5)

    def weight_shapes(self, quantized: bool) -> dict[str, tuple[str, tuple[int, ...]]]:
        """Name -> (dtype, shape) of every array the step reads (``W@int8`` / ``W@scales`` when quantized)."""
        h, i = self.hidden, self.inter
        out: dict[str, tuple[str, tuple[int, ...]]] = {"model.embed_tokens.weight": ("float32", (self.vocab, h))}
        for layer in range(self.layers):
            p = f"model.layers.{layer}"
            out[f"{p}.input_layernorm.weight"] = ("float32", (h,))
            out[f"{p}.post_attention_layernorm.weight"] = ("float32", (h,))
            for name, rows in (("q_proj", self.q_rows), ("k_proj", self.kv_rows), ("v_proj", self.kv_rows)):
                out[f"{p}.self_attn.{name}.bias"] = ("float32", (rows,))
            for name, shape in projection_shapes(self, layer).items():
                if quantized:
                    out[f"{name}@int8"] = ("int8", shape)
                    out[f"{name}@scales"] = ("float32", shape[:1])
                else:
                    out[name] = ("float32", shape)
        out["model.norm.weight"] = ("float32", (h,))
        return out


def projection_shapes(shape: ModelShape, layer: int) -> dict[str, tuple[int, int]]:
    """The seven ``x @ W.T`` weights of one layer, ``[out, in]``, in the order a step reads them."""
    p = f"model.layers.{layer}"
    h, i = shape.hidden, shape.inter
    return {f"{p}.self_attn.q_proj.weight": (shape.q_rows, h), f"{p}.self_attn.k_proj.weight": (shape.kv_rows, h),
            f"{p}.self_attn.v_proj.weight": (shape.kv_rows, h), f"{p}.self_attn.o_proj.weight": (h, shape.q_rows),
            f"{p}.mlp.gate_proj.weight": (i, h), f"{p}.mlp.up_proj.weight": (i, h),
            f"{p}.mlp.down_proj.weight": (h, i)}


# The workloads' model shapes.
TINY = ModelShape(256, 64, 128, 2, 4, 2, 16)                  # configuration 1
QWEN2_0_5B = ModelShape(151936, 896, 4864, 24, 14, 2, 64)     # configurations 2-5
# The smallest shape of the 0.5B model's kind (head dim 64, widths of whole 128-byte chunks): its
# few-row decode takes the persistent step and the int8-prefiltered LM head, as 0.5B does.
SMALL = ModelShape(512, 128, 256, 2, 2, 1, 64)


# -- seeded synthetic inputs ----------------------------------------------------------------


def synthetic_weights(shape: ModelShape, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Random-init float32 weights by checkpoint name: ``N(0, std)``, norm gains 1.

    Drawn from one ``np.random.default_rng(seed)`` in checkpoint order -- the embedding, then per
    layer q/k/v weight and bias, o, gate, up, down -- so every engine handed the same seed gets
    the same arrays. Norm gains draw nothing.
    """
    rng = np.random.default_rng(seed)
    scale = np.float32(std)
    h = shape.hidden

    def normal(*dims: int) -> np.ndarray:
        return rng.standard_normal(dims, dtype=np.float32) * scale

    w: dict[str, np.ndarray] = {"model.embed_tokens.weight": normal(shape.vocab, h)}
    for layer in range(shape.layers):
        p = f"model.layers.{layer}"
        w[f"{p}.input_layernorm.weight"] = np.ones(h, np.float32)
        for name, rows in (("q_proj", shape.q_rows), ("k_proj", shape.kv_rows), ("v_proj", shape.kv_rows)):
            w[f"{p}.self_attn.{name}.weight"] = normal(rows, h)
            w[f"{p}.self_attn.{name}.bias"] = normal(rows)
        w[f"{p}.self_attn.o_proj.weight"] = normal(h, shape.q_rows)
        w[f"{p}.post_attention_layernorm.weight"] = np.ones(h, np.float32)
        w[f"{p}.mlp.gate_proj.weight"] = normal(shape.inter, h)
        w[f"{p}.mlp.up_proj.weight"] = normal(shape.inter, h)
        w[f"{p}.mlp.down_proj.weight"] = normal(h, shape.inter)
    w["model.norm.weight"] = np.ones(h, np.float32)
    return w


def synthetic_prompt(vocab: int, n: int, seed: int = 1) -> list[int]:
    """``n`` uniform random token ids in ``[0, vocab)`` from ``np.random.default_rng(seed)``."""
    return [int(x) for x in np.random.default_rng(seed).integers(0, vocab, n)]


def synthetic_cache(shape: ModelShape, sequence: int, past: int) -> tuple[np.ndarray, np.ndarray, int]:
    """Sequence ``sequence`` of the batched-decode workload: its keys and values ``N(0, 1)``
    float32 ``[layers, kv_heads, past, head_dim]`` and its first token, all from
    ``np.random.default_rng(1000 + sequence)``, so any subset can be regenerated alone."""
    rng = np.random.default_rng(1000 + sequence)
    dims = (shape.layers, shape.kv_heads, past, shape.head_dim)
    keys = rng.standard_normal(dims, dtype=np.float32)
    values = rng.standard_normal(dims, dtype=np.float32)
    return keys, values, int(rng.integers(0, shape.vocab))
