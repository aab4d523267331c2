"""The CUDA target: a reference Qwen2 step graph, fused by the reference, bound to this library.

The reference compiles a graph as ``fuse(optimize(graph))`` into a ``Program`` of kernel calls
(``nanocompile/runtime.py:182-199``, ``nanocompile/fusion.py:734-742``, ``Program`` and ``Call``
at ``nanocompile/lower.py:101-139``) and renders every call's kernel as C. This target takes the
same program and maps its calls, by fused-group kind, onto the hand-written sm_100a kernels of
``libnc_cuda.so``:

=======================================  ==========================================================
reference calls (``Call.primitive``)     CUDA group (kernels)
=======================================  ==========================================================
``gather`` (embedding)                   ``gather``  (``gather_kernel``)
``row`` reading a norm gain              ``rms_norm`` (``norm_quant_kernel`` or the projection's
                                         ``PRO_NORM`` prologue)
``reduce`` / ``elementwise`` chains      ``block_quantize`` (fused into the norm, attention and
  feeding a ``matmul_i8_vnni``           SwiGLU epilogues)
``matmul_i8_vnni`` / ``matmul_i8`` /     ``qkv_projection`` / ``o_projection`` /
  ``matmul`` (``+epilogue``) reading     ``gate_up_projection`` / ``down_projection``
  layer weights                          (``gemv_i8_fused_kernel``, ``gemm_i8_kernel``,
                                         ``gemm_i8_tc_kernel``, ``gemv_f32_kernel`` ...)
``elementwise`` cos / sin / bias+rotate  ``rope`` (tables at model creation; the rotation in the
                                         attention kernel)
``matmul`` over ``past_keys``, ``row``   ``attention`` (``attention_*_kernel``; the KV history
  softmax, ``matmul`` over ``past_values``  lives in the device cache)
``matmul`` reading the embedding         ``lm_head`` (``gemv_f32_kernel`` / ``gemm_f32_kernel``
  into ``logits``                        with the argmax)
``copy`` concat into ``keys``/``values``  ``kv_output`` (the cache append, read back by copy)
=======================================  ==========================================================

Which step this is, exactly, is decided by rebuilding it: the target reads the shape off the
graph (:class:`~nanocompile_b200.model.ModelShape`), asks the reference's own ``build_qwen2`` and
``quantize`` for that shape's step and requires the two printed graphs (``nanocompile/printer.py``)
to be identical, line for line. Every operation, shape, axis and scalar constant is therefore
the one the kernels implement; the only array constant, RoPE's rates, is taken from the graph
as it is. Anything else -- another model, another quantization block, an untied head -- is
refused with the first line that differs.
"""

from __future__ import annotations

import re
from collections.abc import Iterable
from dataclasses import dataclass, field

import numpy as np

from nanocompile_b200.model import ModelShape

# What each group runs on, for the program listing (``CompiledGraph.source``).
ENTRY_POINTS = {
    "gather": "gather_kernel (nc_gather_rows)",
    "rms_norm": "norm_quant_kernel | PRO_NORM prologue (nc_rms_norm_quantize)",
    "block_quantize": "quantizing epilogues / quantize_blocks (nc_quantize_blocks)",
    "qkv_projection": "gemv_i8_fused_kernel | gemm_i8_kernel | gemm_i8_tc_kernel | gemv_f32_kernel (nc_matmul_*)",
    "rope": "RoPE tables at model creation; rotation + cache append in the attention kernel",
    "attention": "attention_split_tma / attention_batched / attention kernels (nc_attention_cache)",
    "o_projection": "gemv_i8_fused_kernel | gemm_i8_kernel | gemm_i8_tc_kernel | gemv_f32_kernel (nc_matmul_*)",
    "gate_up_projection": "gemv_i8_fused_kernel | gemm_i8_kernel | gemm_i8_tc_kernel | gemv_f32_kernel (nc_matmul_*)",
    "down_projection": "gemv_i8_fused_kernel | gemm_i8_kernel | gemm_i8_tc_kernel | gemv_f32_kernel (nc_matmul_*)",
    "persistent_layers": "decode_mk_kernel (steps of 1-4 rows)",
    "lm_head": "gemv_f32_kernel | gemm_f32_kernel + argmax; lm_head_q8 / lm_head_tc + exact pick (nc_lm_head_*)",
    "kv_output": "cache append (in the attention kernel) + nc_qwen2_kv_read",
}

_LAYER = re.compile(r"^model\.layers\.(\d+)\.(.+)$")
_PROJECTION_GROUP = {"self_attn.q_proj": "qkv_projection", "self_attn.k_proj": "qkv_projection",
                     "self_attn.v_proj": "qkv_projection", "self_attn.o_proj": "o_projection",
                     "mlp.gate_proj": "gate_up_projection", "mlp.up_proj": "gate_up_projection",
                     "mlp.down_proj": "down_projection"}
_ACTIVATIONS = {"matmul_i8_vnni": "int8", "matmul_i8": "f32"}
_MODES = {None: None, "int8": "int8", "f32": "f32"}


class TargetError(NotImplementedError):
    """The graph is not a step the CUDA target implements."""


@dataclass(frozen=True)
class Group:
    """One fused group of the CUDA step: the reference calls it covers and what runs them."""

    kind: str
    layer: int | None
    calls: tuple[int, ...]

    @property
    def entry(self) -> str:
        return ENTRY_POINTS[self.kind]


@dataclass
class CudaProgram:
    """A reference step graph lowered for the CUDA library."""

    graph: object                  # the reference's Graph
    program: object                # the reference's Program, fuse(optimize(graph))
    shape: ModelShape
    activations: str | None        # None: float32 projections; "int8": int8-vnni; "f32": int8 weights, f32 activations
    last_only: bool
    rope_rates: np.ndarray
    groups: list[Group] = field(default_factory=list)

    @property
    def calls(self) -> int:
        return len(self.program.calls)

    def source(self) -> str:
        """The program as text: every reference call, the group it belongs to and what runs it."""
        by_call = {c: g for g in self.groups for c in g.calls}
        lines = [f"// {self.graph.name}: {self.shape}, activations={self.activations}, "
                 f"{len(self.groups)} fused groups over {self.calls} reference calls"]
        for i, call in enumerate(self.program.calls):
            g = by_call[i]
            names = [v.buffer.name for v in call.operands if v.buffer.kind in ("weight", "input")]
            where = "" if g.layer is None else f"[{g.layer}]"
            lines.append(f"call {i:4d} {call.primitive:<26s} -> {g.kind}{where:<6s} {g.entry}"
                         + (f"   reads {', '.join(names)}" if names else ""))
        return "\n".join(lines) + "\n"


# -- reading the shape off the graph ------------------------------------------------------------


def _dim(value) -> int:
    if isinstance(value, int):
        return value
    raise TargetError(f"expected a fixed size, got the symbolic {value}")


def _shape_of(graph) -> tuple[ModelShape, str | None, bool]:
    inputs = {n.attrs["name"]: n for n in graph.inputs}
    if set(inputs) != {"token_ids", "past_keys", "past_values"}:
        raise TargetError(f"a Qwen2 step takes token_ids, past_keys and past_values; this graph takes {sorted(inputs)}")
    if set(graph.outputs) != {"logits", "keys", "values"}:
        raise TargetError(f"a Qwen2 step returns logits, keys and values; this graph returns {sorted(graph.outputs)}")
    pk = inputs["past_keys"].shape
    if len(pk) != 4:
        raise TargetError(f"past_keys is {pk}, expected [layers, kv_heads, past, head_dim]")
    layers, kv_heads, head_dim = _dim(pk[0]), _dim(pk[1]), _dim(pk[3])
    weights = graph.weights
    if "lm_head.weight" in weights:
        raise TargetError("the CUDA step implements the tied LM head; this graph reads lm_head.weight")
    if "model.embed_tokens.weight" not in weights:
        raise TargetError("no model.embed_tokens.weight: not a Qwen2 step")
    vocab, hidden = (_dim(d) for d in weights["model.embed_tokens.weight"].shape)

    def rows(name: str) -> int:
        for key in (name, f"{name}@int8"):
            if key in weights:
                return _dim(weights[key].shape[0])
        raise TargetError(f"no weight {name}: not a Qwen2 step")

    heads = rows("model.layers.0.self_attn.q_proj.weight") // head_dim
    inter = rows("model.layers.0.mlp.gate_proj.weight")
    kinds = {n.op for n in graph.nodes} & set(_ACTIVATIONS)
    if len(kinds) > 1:
        raise TargetError(f"mixed int8 projection kinds {sorted(kinds)}")
    activations = _ACTIVATIONS[kinds.pop()] if kinds else None
    eps = None
    for node in graph.nodes:
        if node.op == "sqrt":
            eps = _scalar_operand(node.inputs[0])
            break
    if eps is None:
        raise TargetError("no RMSNorm epsilon found (no sqrt in the graph)")
    logits = graph.outputs["logits"].shape
    last_only = isinstance(logits[0], int) and logits[0] == 1
    shape = ModelShape(vocab, hidden, inter, layers, heads, kv_heads, head_dim, float(np.float32(eps)), 1e6)
    return shape, activations, last_only


def _scalar_operand(node) -> float | None:
    """The scalar constant of ``add(x, broadcast(reshape(const)))`` (the epsilon under the root)."""
    if node.op != "add":
        return None
    for operand in node.inputs:
        while operand.op in ("broadcast", "reshape"):
            operand = operand.inputs[0]
        if operand.op == "const" and np.asarray(operand.attrs["value"]).size == 1:
            return float(np.asarray(operand.attrs["value"]).reshape(()))
    return None


def _rope_rates(graph, head_dim: int) -> np.ndarray:
    """The rotation rates: the one array constant, of ``head_dim / 2`` float32 values, under the cosine."""
    found = []
    for node in graph.nodes:
        if node.op == "const":
            value = np.asarray(node.attrs["value"])
            if value.size > 1:
                found.append(value)
    if len(found) != 1 or found[0].size != head_dim // 2 or found[0].dtype != np.float32:
        raise TargetError(f"expected one array constant of {head_dim // 2} float32 RoPE rates, found "
                          f"{[(a.dtype.name, a.shape) for a in found]}")
    return np.ascontiguousarray(found[0].reshape(-1))


# -- the identity check ---------------------------------------------------------------------------


def _expected_graph(graph, shape: ModelShape, activations: str | None, last_only: bool):
    from nanocompile import quantize as rq
    from nanocompile.models.qwen2 import Qwen2Config, build_qwen2

    config = Qwen2Config(**shape.config_fields())
    expected = build_qwen2(config, last_only=last_only)
    if activations is not None:
        expected = rq.quantize(expected, activations, keep=("lm_head.weight",))
    return expected


def _first_difference(a: Iterable[str], b: Iterable[str]) -> str | None:
    a, b = list(a), list(b)
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return f"line {i + 1}: {x.strip()!r}, the Qwen2 step has {y.strip()!r}"
    if len(a) != len(b):
        return f"{len(a)} lines, the Qwen2 step has {len(b)}"
    return None


# -- mapping the fused program's calls onto groups --------------------------------------------------


def _classify(program) -> list[Group]:
    groups: list[Group] = []
    layer: int | None = None
    pending: list[int] = []            # calls of a quantize chain, attached to the next projection

    def add(kind: str, at: int | None, calls: list[int]) -> None:
        if groups and groups[-1].kind == kind and groups[-1].layer == at and kind != "rms_norm":
            last = groups.pop()
            calls = list(last.calls) + calls
        groups.append(Group(kind, at, tuple(calls)))

    for i, call in enumerate(program.calls):
        views = call.operands
        weights = [v.buffer.name for v in views if v.buffer.kind == "weight"]
        inputs = {v.buffer.name for v in views if v.buffer.kind == "input"}
        consts = [v for v in views if v.buffer.kind == "const"]
        prim, out = call.primitive, call.output
        layered = [m for m in (_LAYER.match(w) for w in weights) if m]
        if layered:
            layer = int(layered[0].group(1))
        if prim == "gather" and "model.embed_tokens.weight" in weights:
            add("gather", None, [i])
        elif prim == "row" and any(w.endswith("layernorm.weight") or w == "model.norm.weight" for w in weights):
            at = None if "model.norm.weight" in weights else layer
            add("rms_norm", at, [i])
        elif prim.startswith("matmul") and layered:
            parts = {m.group(2).rsplit(".weight", 1)[0] for m in layered if ".weight" in m.group(2)}
            kinds = {_PROJECTION_GROUP.get(p) for p in parts}
            if len(kinds) != 1 or None in kinds:
                raise TargetError(f"call {i} ({prim}) reads {weights}: not one of the step's projections")
            if pending:
                add("block_quantize", layer, pending)
                pending = []
            add(kinds.pop(), layer, [i])
        elif prim.startswith("matmul") and "past_keys" in inputs:
            add("attention", layer, [i])
        elif prim.startswith("matmul") and "past_values" in inputs:
            add("attention", layer, [i])
        elif prim == "row" and not weights and groups and groups[-1].kind == "attention":
            add("attention", layer, [i])                                   # the softmax between them
        elif prim.startswith("matmul") and weights == ["model.embed_tokens.weight"] and out.name == "logits":
            add("lm_head", None, [i])
        elif prim == "copy" and out.kind == "output" and out.name in ("keys", "values"):
            add("kv_output", None, [i])
        elif prim == "elementwise" and consts and not weights:
            add("rope", None, [i])                                         # cos / sin of the angles
        elif prim == "elementwise" and any(w.endswith(("q_proj.bias", "k_proj.bias")) for w in weights):
            add("rope", layer, [i])                                        # bias + rotation
        elif prim in ("reduce", "elementwise") and not weights:
            pending.append(i)
        else:
            names = [v.buffer.name for v in views]
            raise TargetError(f"call {i} ({prim}, reading {names}) is not part of the Qwen2 step the CUDA "
                              f"target implements")
    if pending:
        raise TargetError(f"calls {pending} quantize activations no projection reads")
    return groups


def lower_cuda(graph) -> CudaProgram:
    """Lower a reference Qwen2 step graph for the CUDA library, or raise :class:`TargetError`."""
    from nanocompile.fusion import fuse
    from nanocompile.passes import optimize

    shape, activations, last_only = _shape_of(graph)
    rates = _rope_rates(graph, shape.head_dim)
    expected = _expected_graph(graph, shape, activations, last_only)
    difference = _first_difference(str(graph).splitlines(), str(expected).splitlines())
    if difference is not None:
        raise TargetError(f"graph {graph.name!r} is not the Qwen2 step of {shape} "
                          f"(activations={activations}, last_only={last_only}) the CUDA target implements: "
                          f"{difference}")
    program = fuse(optimize(graph))
    cuda = CudaProgram(graph, program, shape, activations, last_only, rates)
    cuda.groups = _classify(program)
    required = {"qkv_projection", "attention", "o_projection", "gate_up_projection", "down_projection", "rope"}
    for layer in range(shape.layers):
        have = {g.kind for g in cuda.groups if g.layer == layer}
        if not required <= have:
            raise TargetError(f"layer {layer} lacks {sorted(required - have)}")
    return cuda
