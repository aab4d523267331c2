"""Golden vectors from the reference itself (run in a container that has nanocompile).

    python tests/golden/make_golden.py [--reference PATH] [tiny proj quant fp32 batch prefill int8 int8_05b]

Every fixture here is an output of nanocompile's own ``CBackend`` (its generated C,
compiled by gcc) -- never of this repository's code -- on seeded synthetic inputs:
weights from ``nanocompile_b200.model.synthetic_weights`` (``N(0, 0.02)`` in
checkpoint order, norm gains 1), prompts from ``np.random.default_rng``. The GPU
parity tests and the CPU oracle are both held to these files; nothing at test
time reads the reference.

Large logits are stored as a SHA-1 per step (bit-exact check), a strided sample
and the top two entries (tolerance checks), so the files stay small.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from nanocompile_b200.model import (QWEN2_0_5B, TINY, ModelShape, synthetic_cache,  # noqa: E402
                                    synthetic_prompt, synthetic_weights)

SAMPLE_STRIDE = 1009
WIDTHS = [(896, 72), (4864, 24), (160, 40), (96, 24)]   # tests/test_int8.py:146, whole 32-blocks only
TOKENS = [1, 3, 7]


def sha1(a: np.ndarray) -> np.ndarray:
    return np.frombuffer(hashlib.sha1(np.ascontiguousarray(a).tobytes()).digest(), np.uint8)


def ref_config(shape: ModelShape):
    from nanocompile.models.qwen2 import Qwen2Config as RefConfig
    return RefConfig(**shape.config_fields())


def run_greedy(model, prompt, steps, cache):
    pending, tokens, logits = list(prompt), [], []
    for _ in range(steps):
        lg = model.forward(pending, cache=cache, last_only=True)
        tok = int(np.argmax(lg[0]))
        tokens.append(tok)
        logits.append(lg[0].copy())
        pending = [tok]
    return tokens, np.stack(logits)


def summarize(logits: np.ndarray) -> dict[str, np.ndarray]:
    top = np.argsort(-logits, axis=1, kind="stable")[:, :2]
    return {
        "sha1": np.stack([sha1(row) for row in logits]),
        "samples": logits[:, ::SAMPLE_STRIDE].copy(),
        "top_index": top.astype(np.int64),
        "top_value": np.take_along_axis(logits, top, axis=1),
    }


# -- fixtures ---------------------------------------------------------------------


def make_tiny() -> None:
    """Config 1 (tiny), float32 and int8-vnni: 8-token prompt, 16 greedy steps, full logits."""
    from nanocompile.models.qwen2 import Qwen2
    from nanocompile.nn import inverse_frequencies
    from nanocompile.runtime import CBackend

    w = synthetic_weights(TINY, seed=0)
    prompt = synthetic_prompt(TINY.vocab, 8)
    out: dict[str, np.ndarray] = {"prompt": np.array(prompt, np.int64),
                                  "inv_freq": TINY.rope_rates()}
    for tag, quant in (("fp32", None), ("vnni", "int8-vnni")):
        model = Qwen2(ref_config(TINY), w, run=CBackend(), quantization=quant)
        tokens, logits = run_greedy(model, prompt, 16, model.new_cache(4))   # capacity 4: forces growth
        out[f"{tag}_tokens"] = np.array(tokens, np.int64)
        out[f"{tag}_logits"] = logits
        out[f"{tag}_full_logits"] = model.forward(prompt)                   # uncached, every position
        cache = model.new_cache(64)
        rows = [model.forward(prompt[:5], cache=cache)] + [model.forward([t], cache=cache) for t in prompt[5:]]
        out[f"{tag}_chunked_logits"] = np.concatenate(rows)
        keys, values = cache.past()
        out[f"{tag}_keys"] = np.ascontiguousarray(keys)
        out[f"{tag}_values"] = np.ascontiguousarray(values)
    np.savez_compressed(HERE / "tiny.npz", **out)


def make_proj() -> None:
    """One int8-vnni projection per width of tests/test_int8.py, tokens 1/3/7: quantized
    activations, the reference's int8 weights, and the output, from its generated C."""
    from nanocompile import dtypes, quantize
    from nanocompile.frontend import GraphBuilder
    from nanocompile.ir import Graph
    from nanocompile.nn import linear
    from nanocompile.runtime import CompiledGraph

    out: dict[str, np.ndarray] = {}
    for k, n in WIDTHS:
        b = GraphBuilder("projection")
        x = b.input("x", dtypes.f32, (b.symbol("seq"), k))
        graph = quantize.quantize(b.build({"y": linear(x, b.weight("w", (n, k)))}), "int8")
        mm = next(node for node in graph.nodes if node.op == "matmul_i8_vnni")
        graph = Graph(graph.inputs, {"y": graph.outputs["y"], "xq": mm.inputs[0], "xs": mm.inputs[1],
                                     "offset": mm.inputs[2]}, name="projection_parts")
        compiled = CompiledGraph(graph)
        for tokens in TOKENS:
            rng = np.random.default_rng(k + tokens)                       # tests/test_int8.py:150-155
            w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
            xin = (rng.standard_normal((tokens, k)) * 2).astype(np.float32)
            xin[:, ::13] *= 40.0
            weights = quantize.quantized_weights(graph, {"w": w})
            res = compiled({"x": xin}, weights)
            tag = f"k{k}_n{n}_t{tokens}"
            out[f"{tag}_x"] = xin
            out[f"{tag}_q"] = weights["w@int8"]
            out[f"{tag}_scales"] = weights["w@scales"]
            for name in ("y", "xq", "xs", "offset"):
                out[f"{tag}_{name}"] = res[name]
    # nanocompile/quantize.py:55-70 on the edge cases of tests/test_int8.py:66-78
    rng = np.random.default_rng(0)
    wq = (rng.standard_normal((37, 70)) * 0.04).astype(np.float32)
    wq[3] = 0.0
    wq[5, :4] = [0.5, -0.5, 1.5, -2.5]
    wq[5, 4] = 127.0 / 64
    values, scales = quantize.quantize_int8(wq)
    out["qi8_w"], out["qi8_values"], out["qi8_scales"] = wq, values, scales
    np.savez_compressed(HERE / "proj.npz", **out)


WIDTHS_I8 = [(896, 72), (4864, 24), (160, 40), (96, 24), (136, 16), (100, 8)]   # + 8-groups and a short tail


def make_int8_f32() -> None:
    """The int8 mode with float32 activations (matmul_i8, nanocompile/lower.py:320-356): one
    projection per width (widths with 8-element groups and a tail past them included), tokens
    1/3/7; and configuration 1's greedy run with quantization="int8"."""
    from nanocompile import dtypes, quantize
    from nanocompile.frontend import GraphBuilder
    from nanocompile.models.qwen2 import Qwen2
    from nanocompile.nn import linear
    from nanocompile.runtime import CBackend, CompiledGraph

    out: dict[str, np.ndarray] = {}
    for k, n in WIDTHS_I8:
        b = GraphBuilder("projection_i8")
        x = b.input("x", dtypes.f32, (b.symbol("seq"), k))
        graph = quantize.quantize(b.build({"y": linear(x, b.weight("w", (n, k)))}), "f32")
        compiled = CompiledGraph(graph)
        for tokens in TOKENS:
            rng = np.random.default_rng(3 * k + tokens)
            w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
            xin = (rng.standard_normal((tokens, k)) * 2).astype(np.float32)
            weights = quantize.quantized_weights(graph, {"w": w})
            tag = f"k{k}_n{n}_t{tokens}"
            out[f"{tag}_x"] = xin
            out[f"{tag}_q"] = weights["w@int8"]
            out[f"{tag}_scales"] = weights["w@scales"]
            out[f"{tag}_y"] = compiled({"x": xin}, weights)["y"]
    w = synthetic_weights(TINY, seed=0)
    prompt = synthetic_prompt(TINY.vocab, 8)
    model = Qwen2(ref_config(TINY), w, run=CBackend(), quantization="int8")
    tokens, logits = run_greedy(model, prompt, 16, model.new_cache(4))
    out["tiny_prompt"] = np.array(prompt, np.int64)
    out["tiny_tokens"] = np.array(tokens, np.int64)
    out["tiny_logits"] = logits
    out["tiny_full_logits"] = model.forward(prompt)
    np.savez_compressed(HERE / "int8_f32.npz", **out)


def make_05b(quant: str | None, steps: int, name: str) -> None:
    """Configs 2/3: the 0.5B model, 32-token prompt, greedy decode."""
    from nanocompile.models.qwen2 import Qwen2
    from nanocompile.nn import inverse_frequencies
    from nanocompile.runtime import CBackend

    w = synthetic_weights(QWEN2_0_5B, seed=0)
    prompt = synthetic_prompt(QWEN2_0_5B.vocab, 32)
    model = Qwen2(ref_config(QWEN2_0_5B), w, run=CBackend(), quantization=quant)
    cache = model.new_cache(32 + steps)
    started = time.perf_counter()
    tokens, logits = run_greedy(model, prompt, steps, cache)
    print(f"{name}: {steps} steps in {time.perf_counter() - started:.1f} s")
    keys, values = cache.past()
    out = {"prompt": np.array(prompt, np.int64), "tokens": np.array(tokens, np.int64),
           "inv_freq": QWEN2_0_5B.rope_rates(),
           "first_logits": logits[:2].copy(),
           "keys_sha1": np.stack([sha1(np.ascontiguousarray(keys[l])) for l in range(keys.shape[0])]),
           "values_sha1": np.stack([sha1(np.ascontiguousarray(values[l])) for l in range(values.shape[0])]),
           "prompt_keys_layer0": np.ascontiguousarray(keys[0, :, :32]),
           **summarize(logits)}
    np.savez_compressed(HERE / f"{name}.npz", **out)


def make_batch(sequences: int, steps: int, past: int = 2048) -> None:
    """Config 5: independent sequences from N(0,1) caches of 2048 positions, greedy steps each."""
    from nanocompile.models.qwen2 import KVCache, Qwen2
    from nanocompile.runtime import CBackend

    cfg = QWEN2_0_5B
    w = synthetic_weights(cfg, seed=0)
    model = Qwen2(ref_config(cfg), w, run=CBackend(), quantization="int8-vnni")
    all_tokens, shas, samples = [], [], []
    started = time.perf_counter()
    for b in range(sequences):
        keys, values, first = synthetic_cache(cfg, b, past)
        cache = KVCache(model.config, past + steps)
        cache.append(keys, values)
        tokens, logits = run_greedy(model, [first], steps, cache)
        all_tokens.append([first] + tokens)
        s = summarize(logits)
        shas.append(s["sha1"])
        samples.append(s["samples"])
        print(f"batch sequence {b}: {time.perf_counter() - started:.0f} s")
    np.savez_compressed(HERE / "batch.npz", tokens=np.array(all_tokens, np.int64), sha1=np.stack(shas),
                        samples=np.stack(samples[:4]), past=np.int64(past))


def make_prefill(seq: int = 512) -> None:
    """Config 4: one int8-vnni step over a 512-token prompt at past 0, every position's logits."""
    from nanocompile.models.qwen2 import Qwen2
    from nanocompile.runtime import CBackend

    cfg = QWEN2_0_5B
    w = synthetic_weights(cfg, seed=0)
    ids = synthetic_prompt(cfg.vocab, seq, seed=4)
    model = Qwen2(ref_config(cfg), w, run=CBackend(), quantization="int8-vnni")
    cache = model.new_cache(seq)
    started = time.perf_counter()
    last = model.forward(ids, cache=cache, last_only=True)
    print(f"prefill {seq}: {time.perf_counter() - started:.1f} s")
    keys, values = cache.past()
    np.savez_compressed(HERE / "prefill.npz", ids=np.array(ids, np.int64), logits=last[0],
                        keys_sha1=np.stack([sha1(np.ascontiguousarray(keys[l])) for l in range(cfg.layers)]),
                        values_sha1=np.stack([sha1(np.ascontiguousarray(values[l])) for l in range(cfg.layers)]),
                        keys_layer23_head1=np.ascontiguousarray(keys[23, 1, ::37]))


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", default=None,
                        help="the nanocompile checkout (default: NANOCOMPILE_REFERENCE, else BASELINE.json's)")
    parser.add_argument("parts", nargs="*", default=["tiny", "proj", "quant", "fp32", "prefill", "batch"])
    args = parser.parse_args()
    from oracle.build_ref import reference_checkout

    reference = args.reference or reference_checkout()
    if reference is None:
        parser.error("no nanocompile checkout: pass --reference or set NANOCOMPILE_REFERENCE")
    sys.path.insert(1, str(reference))
    os.environ.setdefault("NANOCOMPILE_CACHE", "/tmp/nanocompile-cache")
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
    for part in args.parts:
        started = time.perf_counter()
        {"tiny": make_tiny, "proj": make_proj,
         "quant": lambda: make_05b("int8-vnni", 993, "qwen05b_vnni"),
         "int8": make_int8_f32, "int8_05b": lambda: make_05b("int8", 48, "qwen05b_int8"),
         "fp32": lambda: make_05b(None, 128, "qwen05b_fp32"),
         "prefill": make_prefill,
         "batch": lambda: make_batch(64, 64)}[part]()
        print(f"{part}: {time.perf_counter() - started:.1f} s")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
