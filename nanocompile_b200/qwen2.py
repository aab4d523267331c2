"""Qwen2 on the CUDA backend: the config, the step description, the driver.

This mirrors nanocompile's ``nanocompile/models/qwen2.py`` for the one path this
package accelerates -- a Qwen2 step: embedding, decoder blocks, final norm, tied
LM head -- so code written against the reference's driver runs unchanged:

    model = Qwen2(config, weights, run=CUDABackend(), quantization="int8-vnni")
    greedy(model, prompt_ids, max_new_tokens=24)

What differs is where the work happens. ``build_qwen2`` returns a
:class:`StepGraph`, the description of one step that the CUDA target compiles
(the reference builds an IR graph of the same computation; the kernels here
reproduce the fused C that graph compiles to, operation for operation). The
``Runner`` protocol is the reference's: ``run(graph, inputs, weights) -> dict``
with inputs ``token_ids`` / ``past_keys`` / ``past_values`` and outputs
``logits`` / ``keys`` / ``values``. A runner that also offers a device-resident
cache (``CUDABackend`` does) is used through it, so cached decode never moves
the KV history between host and device.
"""

from __future__ import annotations

import json
from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from nanocompile_b200 import quantize as q


@dataclass(frozen=True)
class Qwen2Config:
    """The hyperparameters the step's shapes depend on (``nanocompile/models/qwen2.py:45-96``)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    rms_norm_eps: float
    rope_theta: float
    tie_word_embeddings: bool

    def __post_init__(self) -> None:
        if self.hidden_size % self.num_attention_heads:
            raise ValueError("hidden_size must divide evenly into attention heads")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("attention heads must divide evenly into KV heads")
        if self.head_dim % 2:
            raise ValueError("RoPE needs an even head_dim")

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def kv_group_size(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    @classmethod
    def from_dict(cls, data: Mapping) -> "Qwen2Config":
        if data.get("architectures") != ["Qwen2ForCausalLM"]:
            raise ValueError(f"not a Qwen2 config: {data.get('architectures')}")
        if data.get("hidden_act", "silu") != "silu":
            raise ValueError(f"hidden_act {data['hidden_act']!r} is not implemented")
        return cls(
            vocab_size=int(data["vocab_size"]),
            hidden_size=int(data["hidden_size"]),
            intermediate_size=int(data["intermediate_size"]),
            num_hidden_layers=int(data["num_hidden_layers"]),
            num_attention_heads=int(data["num_attention_heads"]),
            num_key_value_heads=int(data.get("num_key_value_heads", data["num_attention_heads"])),
            rms_norm_eps=float(data["rms_norm_eps"]),
            rope_theta=float(data.get("rope_theta", 10000.0)),
            tie_word_embeddings=bool(data.get("tie_word_embeddings", False)),
        )

    @classmethod
    def from_model_dir(cls, model_dir: str | Path) -> "Qwen2Config":
        path = Path(model_dir) / "config.json"
        return cls.from_dict(json.loads(path.read_text(encoding="utf-8")))


# The configurations the benchmark and the tests use.
TINY = Qwen2Config(256, 64, 128, 2, 4, 2, 1e-6, 1e6, True)
QWEN2_0_5B = Qwen2Config(151936, 896, 4864, 24, 14, 2, 1e-6, 1e6, True)
# The smallest shape of the 0.5B model's kind (head dim 64, widths of whole 128-byte chunks): the
# few-row decode runs through the persistent step and the int8-prefiltered LM head, as 0.5B does.
SMALL = Qwen2Config(512, 128, 256, 2, 2, 1, 1e-6, 1e6, True)


def inverse_frequencies(head_dim: int, theta: float) -> np.ndarray:
    """RoPE's per-plane rates, the same float32 NumPy expression as ``nanocompile/nn.py:69-75``."""
    exponent = np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim)
    return (np.float32(1.0) / (np.float32(theta) ** exponent)).astype(np.float32)


def attention_scale(head_dim: int) -> np.float32:
    """``np.float32(d ** -0.5)``, the score scale of ``nanocompile/models/qwen2.py:149``."""
    return np.float32(head_dim ** -0.5)


# -- the step ------------------------------------------------------------------

QUANTIZATIONS = {"int8": "f32", "int8-vnni": "int8"}   # nanocompile/models/qwen2.py:275


@dataclass(frozen=True)
class StepGraph:
    """One forward step of Qwen2, as ``build_qwen2`` (``nanocompile/models/qwen2.py:167-224``) builds it.

    ``activations`` is ``None`` for float32 projections, ``"int8"`` for the
    int8-vnni scheme (``matmul_i8_vnni``), ``"f32"`` for int8 weights with float
    activations (``matmul_i8``). ``weights`` lists every array the step reads,
    by checkpoint name, in the reference's naming (``W@int8`` / ``W@scales``
    for quantized projections).
    """

    config: Qwen2Config
    last_only: bool = False
    activations: str | None = None
    keep: tuple[str, ...] = ()

    @property
    def name(self) -> str:
        return "qwen2_last" if self.last_only else "qwen2"

    @property
    def input_names(self) -> tuple[str, ...]:
        return ("token_ids", "past_keys", "past_values")

    @property
    def output_names(self) -> tuple[str, ...]:
        return ("logits", "keys", "values")

    @property
    def quantized(self) -> frozenset[str]:
        if self.activations is None:
            return frozenset()
        return frozenset(q.projection_names(self.config.num_hidden_layers, self.keep))

    @property
    def weights(self) -> dict[str, tuple[np.dtype, tuple[int, ...]]]:
        """Name -> (dtype, shape) of every weight, in the order the reference graph reads them."""
        c = self.config
        h, i, d = c.hidden_size, c.intermediate_size, c.head_dim
        out: dict[str, tuple[np.dtype, tuple[int, ...]]] = {}
        f32, i8 = np.dtype(np.float32), np.dtype(np.int8)
        quantized = self.quantized

        def weight(name: str, shape: tuple[int, ...]) -> None:
            if name in quantized:
                out[q.int8_name(name)] = (i8, shape)
                out[q.scales_name(name)] = (f32, shape[:1])
            else:
                out[name] = (f32, shape)

        weight("model.embed_tokens.weight", (c.vocab_size, h))
        for layer in range(c.num_hidden_layers):
            p = f"model.layers.{layer}"
            weight(f"{p}.input_layernorm.weight", (h,))
            for proj, n in (("q_proj", c.num_attention_heads * d), ("k_proj", c.num_key_value_heads * d),
                            ("v_proj", c.num_key_value_heads * d)):
                weight(f"{p}.self_attn.{proj}.weight", (n, h))
                weight(f"{p}.self_attn.{proj}.bias", (n,))
            weight(f"{p}.self_attn.o_proj.weight", (h, c.num_attention_heads * d))
            weight(f"{p}.post_attention_layernorm.weight", (h,))
            weight(f"{p}.mlp.gate_proj.weight", (i, h))
            weight(f"{p}.mlp.up_proj.weight", (i, h))
            weight(f"{p}.mlp.down_proj.weight", (h, i))
        weight("model.norm.weight", (h,))
        if not c.tie_word_embeddings:
            weight("lm_head.weight", (c.vocab_size, h))
        return out


def build_qwen2(config: Qwen2Config, last_only: bool = False) -> StepGraph:
    """The forward pass for one step (``nanocompile/models/qwen2.py:167``)."""
    return StepGraph(config, last_only)


def quantize(graph: StepGraph, activations: str = "f32", block: int = q.BLOCK,
             keep: Sequence[str] = ()) -> StepGraph:
    """``graph`` with its projections reading per-row int8 weights (``nanocompile/quantize.py:127-164``)."""
    if activations not in q.ACTIVATIONS:
        raise ValueError(f"activations must be one of {q.ACTIVATIONS}, got {activations!r}")
    if block != q.BLOCK:
        raise ValueError(f"the CUDA kernels implement block {q.BLOCK} activation scales, got {block}")
    return StepGraph(graph.config, graph.last_only, activations, tuple(keep))


# -- synthetic weights -----------------------------------------------------------


def synthetic_weights(config: Qwen2Config, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Random-init weights by checkpoint name: ``N(0, std)`` float32, norm gains 1.

    Drawn from ``np.random.default_rng(seed)`` in checkpoint order (embedding;
    per layer q/k/v weight and bias, o, gate, up, down), so every engine given
    the same seed gets the same arrays.
    """
    rng = np.random.default_rng(seed)
    c = config
    h, i, d = c.hidden_size, c.intermediate_size, c.head_dim
    scale = np.float32(std)

    def normal(*shape: int) -> np.ndarray:
        return rng.standard_normal(shape, dtype=np.float32) * scale

    w: dict[str, np.ndarray] = {"model.embed_tokens.weight": normal(c.vocab_size, h)}
    for layer in range(c.num_hidden_layers):
        p = f"model.layers.{layer}"
        w[f"{p}.input_layernorm.weight"] = np.ones(h, np.float32)
        for proj, n in (("q_proj", c.num_attention_heads * d), ("k_proj", c.num_key_value_heads * d),
                        ("v_proj", c.num_key_value_heads * d)):
            w[f"{p}.self_attn.{proj}.weight"] = normal(n, h)
            w[f"{p}.self_attn.{proj}.bias"] = normal(n)
        w[f"{p}.self_attn.o_proj.weight"] = normal(h, c.num_attention_heads * d)
        w[f"{p}.post_attention_layernorm.weight"] = np.ones(h, np.float32)
        w[f"{p}.mlp.gate_proj.weight"] = normal(i, h)
        w[f"{p}.mlp.up_proj.weight"] = normal(i, h)
        w[f"{p}.mlp.down_proj.weight"] = normal(h, i)
    w["model.norm.weight"] = np.ones(h, np.float32)
    if not c.tie_word_embeddings:
        w["lm_head.weight"] = normal(c.vocab_size, h)
    return w


def synthetic_prompt(vocab: int, n: int, seed: int = 1) -> list[int]:
    """``n`` uniform random token ids from ``np.random.default_rng(seed)``."""
    return [int(x) for x in np.random.default_rng(seed).integers(0, vocab, n)]


def synthetic_cache(config: Qwen2Config, sequence: int, past: int) -> tuple[np.ndarray, np.ndarray, int]:
    """Sequence ``sequence`` of the batched-decode workload: keys and values ``N(0, 1)``
    float32 ``[layers, kv_heads, past, head_dim]`` and a first token, all from
    ``np.random.default_rng(1000 + sequence)``, so any subset can be regenerated alone."""
    rng = np.random.default_rng(1000 + sequence)
    shape = (config.num_hidden_layers, config.num_key_value_heads, past, config.head_dim)
    keys = rng.standard_normal(shape, dtype=np.float32)
    values = rng.standard_normal(shape, dtype=np.float32)
    return keys, values, int(rng.integers(0, config.vocab_size))


# -- running it --------------------------------------------------------------------

Runner = Callable[[StepGraph, Mapping[str, np.ndarray], Mapping[str, np.ndarray]], dict[str, np.ndarray]]


class KVCache:
    """Host keys and values for one sequence, grown by doubling (``nanocompile/models/qwen2.py:232-271``).

    This is the cache a plain ``Runner`` gets: a view of the filled region,
    ``[layers, kv_heads, length, head_dim]``, passed in each step. The CUDA
    backend's own cache (``DeviceKVCache``) keeps the history in HBM instead.
    """

    def __init__(self, config: Qwen2Config, capacity: int = 256) -> None:
        if capacity <= 0:
            raise ValueError(f"capacity must be positive, got {capacity}")
        self.config = config
        self.length = 0
        self._keys = self._allocate(capacity)
        self._values = self._allocate(capacity)

    def _allocate(self, capacity: int) -> np.ndarray:
        c = self.config
        return np.zeros((c.num_hidden_layers, c.num_key_value_heads, capacity, c.head_dim), dtype=np.float32)

    @property
    def capacity(self) -> int:
        return self._keys.shape[2]

    def past(self) -> tuple[np.ndarray, np.ndarray]:
        return self._keys[:, :, : self.length], self._values[:, :, : self.length]

    def append(self, keys: np.ndarray, values: np.ndarray) -> None:
        n = keys.shape[2]
        if self.length + n > self.capacity:
            capacity = max(self.length + n, 2 * self.capacity)
            for name in ("_keys", "_values"):
                grown = self._allocate(capacity)
                grown[:, :, : self.length] = getattr(self, name)[:, :, : self.length]
                setattr(self, name, grown)
        self._keys[:, :, self.length : self.length + n] = keys
        self._values[:, :, self.length : self.length + n] = values
        self.length += n


class Qwen2:
    """The model's front door: token IDs in, logits out (``nanocompile/models/qwen2.py:278-345``).

    ``quantization`` is ``None`` (float32), ``"int8"`` or ``"int8-vnni"``; the
    LM head stays float32 either way. The int8 weights are made from
    ``weights`` once, here, on the host.
    """

    def __init__(self, config: Qwen2Config, weights: Mapping[str, np.ndarray], run: Runner,
                 quantization: str | None = None) -> None:
        self.config = config
        self.run = run
        self.quantization = quantization
        self.graph = build_qwen2(config)
        self.graph_last = build_qwen2(config, last_only=True)
        if quantization is not None:
            if quantization not in QUANTIZATIONS:
                raise ValueError(f"quantization must be one of {sorted(QUANTIZATIONS)} or None")
            mode = QUANTIZATIONS[quantization]
            keep = ("lm_head.weight",)
            self.graph = quantize(self.graph, mode, keep=keep)
            self.graph_last = quantize(self.graph_last, mode, keep=keep)
            weights = q.quantized_weights(self.graph, weights)
        self.weights = weights

    def new_cache(self, capacity: int = 256):
        """A cache for one sequence: on the device when the runner keeps one there."""
        factory = getattr(self.run, "new_cache", None)
        if factory is not None:
            return factory(self.graph_last, self.weights, capacity)
        return KVCache(self.config, capacity)

    def forward(self, token_ids: Sequence[int] | np.ndarray, cache=None, last_only: bool = False) -> np.ndarray:
        """Logits for ``token_ids``, the tokens not already in ``cache``."""
        token_ids = np.asarray(token_ids, dtype=np.int64)
        if token_ids.ndim != 1 or token_ids.size == 0:
            raise ValueError(f"expected a non-empty 1-D sequence of token IDs, got {token_ids.shape}")
        graph = self.graph_last if last_only else self.graph
        if cache is not None and hasattr(cache, "forward"):
            return cache.forward(graph, token_ids, self.weights)
        if cache is None:
            c = self.config
            empty = np.zeros((c.num_hidden_layers, c.num_key_value_heads, 0, c.head_dim), np.float32)
            past_keys = past_values = empty
        else:
            past_keys, past_values = cache.past()
        out = self.run(graph, {"token_ids": token_ids, "past_keys": past_keys, "past_values": past_values},
                       self.weights)
        if cache is not None:
            cache.append(out["keys"], out["values"])
        return out["logits"]


def greedy(model: Qwen2, prompt_ids: Sequence[int], max_new_tokens: int, use_cache: bool = True) -> list[int]:
    """Argmax decoding (``nanocompile/models/qwen2.py:348-368``): the first maximum wins.

    With a device cache the argmax is computed on the device, fused into the LM
    head, and the whole decode loop runs as replays of one captured step.
    """
    if not prompt_ids:
        raise ValueError("cannot generate from an empty prompt")
    ids = list(prompt_ids)
    cache = model.new_cache(len(ids) + max_new_tokens) if use_cache else None
    if cache is not None and hasattr(cache, "greedy"):
        return cache.greedy(model.graph_last, ids, max_new_tokens, model.weights)
    pending = ids
    generated: list[int] = []
    for _ in range(max_new_tokens):
        logits = model.forward(pending, cache=cache, last_only=True)
        token = int(np.argmax(logits[0]))
        generated.append(token)
        ids.append(token)
        pending = [token] if use_cache else ids
    return generated
