"""Benchmark: int8 Qwen2.5-0.5B-architecture decode on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-bs1]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

One JSON line on rank 0. The workload is the batched-decode configuration: 64 independent
sequences per GPU, each from a 2048-position KV cache of N(0, 1) float32 values, one greedy
decode step for all of them per timed step (one replay of the captured step graph). Sequences
are sharded across ranks with no data-path collective ("weak" scaling: per-GPU work fixed);
torch.distributed (NCCL) is used only for the barrier and the max-over-ranks of the timing.

``value`` is device-timed (CUDA events on the model's stream) with every input resident in
HBM; ``e2e`` is the same workload through the public decode call with host buffers: each step
copies that step's input tokens host->device from pinned memory and the step's argmax tokens
device->host, then synchronizes. At N = 1 a ``bs1`` object adds the batch-1 decode of the
same model (32-token prompt, then greedy decode up to 1024 positions).

Weights are synthetic (random init, N(0, 0.02), seed 0), int8-quantized on the host by the
reference's scheme; token ids and caches are seeded. The weights (0.9 GB) and the KV caches
(3.3 GB per GPU) are larger than L2 (126 MB), so no flush is needed between steps.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from nanocompile_b200.model import QWEN2_0_5B, synthetic_cache, synthetic_prompt, synthetic_weights  # noqa: E402
from nanocompile_b200.shard import rank_sequences  # noqa: E402

METRIC = "int8 Qwen2-0.5B decode tok/s (bs1; bs64×1/2/4/8 GPU); % of HBM roofline"
BATCH = 64            # sequences per GPU (configuration 5)
PAST = 2048           # cached positions per sequence at the first step
BS1_PROMPT, BS1_END = 32, 1024
FALLBACK_HBM_GBS = 6650.0


# -- plumbing ---------------------------------------------------------------------------------


class RankGroup:
    """Rank and world from the torchrun environment, and the host-side collectives the timing
    needs: a barrier, the max over ranks, a gather of small records. torch.distributed (NCCL on
    GPUs, gloo on the host) is used here only, never on the data path."""

    def __init__(self, backend: str | None = None, timeout_s: float = 120.0):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dist = None
        self.device = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
            kwargs = {}
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                self.device = torch.device("cuda", self.local)
                kwargs["device_id"] = self.device
            # the communicators are made here, with the process's stdout pointed at stderr: the
            # library may print a version banner, and rank 0's stdout must carry one JSON line
            sys.stdout.flush()
            saved = os.dup(1)
            os.dup2(2, 1)
            try:
                dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
                dist.barrier()
            finally:
                sys.stdout.flush()
                os.dup2(saved, 1)
                os.close(saved)
            self.dist = dist
            self.torch = torch

    def barrier(self) -> None:
        if self.dist is not None:
            self.dist.barrier()

    def max(self, value: float) -> float:
        """The largest ``value`` over the ranks (every rank gets it)."""
        if self.dist is None:
            return value
        t = self.torch.tensor([value], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, obj) -> list:
        """Every rank's ``obj``, in rank order (every rank gets the list)."""
        if self.dist is None:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out

    def close(self) -> None:
        if self.dist is not None:
            self.dist.destroy_process_group()
            self.dist = None


def measured_peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def dram_traffic(kind: str, workload: str) -> float | None:
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/traffic.txt)."""
    path = ROOT / "profiles" / "traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and not line.startswith("#") and parts[0] == workload and parts[1] == kind:
            return float(parts[2])
    return None


class ClockSampler:
    """nvidia-smi samples of the GPU's clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sms, maxes, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxes.append(float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(sms)}


# -- the model ------------------------------------------------------------------------------


def build_model(dev: int, slots: int, capacity: int, max_rows: int | None = None):
    """The 0.5B model on GPU ``dev``: float32 weights uploaded and quantized on the device. The
    host copy of the int8 weights (the CPU baseline's) comes from the host quantizer."""
    from nanocompile_b200 import quantize as q
    from nanocompile_b200 import runtime

    cfg = QWEN2_0_5B
    weights = synthetic_weights(cfg, seed=0)
    model = runtime.DeviceModel(cfg, weights, "int8", max_rows=max_rows or BATCH, slots=slots, capacity=capacity,
                                device=dev)
    return cfg, weights, model


def host_int8_weights(weights):
    from nanocompile_b200 import quantize as q

    return q.int8_projection_weights(weights, QWEN2_0_5B)


def layer_bytes(cfg, rows: int, past: int) -> float:
    """One decoder layer's int8 weights, scales, bias and gains, and its KV rows read for `rows` rows."""
    H, I, d = cfg.hidden, cfg.inter, cfg.head_dim
    heads, kv = cfg.heads, cfg.kv_heads
    nqkv, hq = (heads + 2 * kv) * d, heads * d
    weights = nqkv * H + H * hq + 2 * I * H + H * I
    scales = 4 * (nqkv + H + 2 * I + H) + 4 * nqkv + 2 * 4 * H
    return weights + scales + rows * 2 * kv * (past + 1) * d * 4


def algorithmic_bytes(kind: str, cfg, rows: int, past: int) -> float:
    """Bytes a launch of `kind` must move at least (weights / cache / activations, once each)."""
    H, I, d, V = cfg.hidden, cfg.inter, cfg.head_dim, cfg.vocab
    heads, kv = cfg.heads, cfg.kv_heads
    nqkv = (heads + 2 * kv) * d
    if kind == "lm_head_argmax":
        if rows <= 16:        # int8 prefilter: the int8 copy, its row scales, approximations out and back
            return V * H + V * 4 + rows * (H * 4 + 2 * V * 4)
        return V * H * 4 + rows * H * 4 + rows * V * 4
    if kind == "persistent_layers":
        return cfg.layers * layer_bytes(cfg, rows, past)
    if kind == "attention":
        return rows * (2 * kv * (past + 1) * d * 4 + nqkv * 4 + heads * d * 1.25)
    if kind == "down_projection":
        return H * I + H * 4 + rows * (I * 1.25 + H * 8)
    if kind == "gate_up_projection":
        return 2 * I * H + 2 * I * 4 + rows * (H * 4 + I * 1.25)
    if kind == "qkv_projection":
        return nqkv * H + nqkv * 8 + rows * (H * 4 + nqkv * 4)
    if kind == "o_projection":
        return H * heads * d + H * 4 + rows * (heads * d * 1.25 + H * 8)
    return 0.0


def roofline(profile: dict, cfg, rows: int, past: int, workload: str) -> dict:
    peak, source = measured_peaks()
    kind = max(profile, key=lambda k: profile[k][0])
    total_ms = sum(v[0] for v in profile.values())
    ms, launches = profile[kind]
    per_launch_s = ms / 1000.0 / launches
    alg = algorithmic_bytes(kind, cfg, rows, past)
    achieved = alg / per_launch_s / 1e9
    out = {"kernel": kind, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
           "frac": round(achieved / peak, 4), "peak_source": source, "algorithmic_bytes_per_launch": alg,
           "avg_launch_us": round(per_launch_s * 1e6, 2), "share_of_step": round(ms / total_ms, 3),
           "traffic": dram_traffic(kind, workload),
           "kernel_shares": {k: round(v[0] / total_ms, 3) for k, v in sorted(profile.items(), key=lambda x: -x[1][0])},
           "kernel_us": {k: round(v[0] * 1000.0 / v[1], 2) for k, v in sorted(profile.items(), key=lambda x: -x[1][0])}}
    return out


# -- the CPU baseline (test-infrastructure oracle or the reference's own generated C) ----------


def cpu_model(cfg, wq, threads: int):
    """The reference's own compiled step (oracle/_ref, kind "reference") or the oracle port."""
    ref = ROOT / "oracle" / "_ref"
    if (ref / "plan.json").exists():
        from oracle import ref_runner

        return ref_runner.ReferenceModel(ref, wq, threads=threads), "reference"
    from oracle.oracle import OracleModel

    return OracleModel(cfg, wq, "int8", threads=threads), "port"


def thread_counts() -> list[int]:
    """The reference's NANOCOMPILE_THREADS sweep: 6 (its default), 8, and every host core."""
    cores = os.cpu_count() or 1
    return sorted({min(6, cores), min(8, cores), cores})


def cpu_sample(cfg, wq, steps: int, threads: int | None = None, warmup: int = 1) -> dict:
    """Greedy decode of one sequence of the batched workload on the host cores (``warmup``
    untimed steps first), at each thread count of the sweep; the best is the baseline."""
    keys, values, first = synthetic_cache(cfg, 0, PAST)
    sweep = [threads] if threads else thread_counts()
    model, kind = cpu_model(cfg, wq, sweep[0])
    per_threads = {}
    for n in sweep:
        if hasattr(model, "set_threads"):
            model.set_threads(n)
        elif n != sweep[0]:
            model, kind = cpu_model(cfg, wq, n)
        for _ in range(max(warmup, 1)):                               # warm (first touch, packed weights)
            model.step([first], keys, values, last_only=True)
        started = time.perf_counter()
        model.greedy([first], steps, past_keys=keys, past_values=values)
        per_threads[n] = steps / (time.perf_counter() - started)
    best = max(per_threads, key=per_threads.get)
    return {"value": round(per_threads[best], 3), "unit": "tok/s", "cores": best, "kind": kind,
            "threads_sweep": {str(n): round(v, 3) for n, v in per_threads.items()}, "host_cores": os.cpu_count(),
            "sample": f"{steps} greedy decode steps of one sequence of the batched workload (past {PAST}) per "
                      f"thread count, sequences run one after another as the reference runs them"}


# -- the two arms ------------------------------------------------------------------------------


def run_ours(args, dist: RankGroup) -> dict | None:
    dev = dist.local
    capacity = max(PAST, BS1_END) + args.warmup + args.steps + 16
    cfg, weights, model = build_model(dev, BATCH, capacity)

    first, slots, starts = [], list(range(BATCH)), [PAST] * BATCH
    for b, sequence in enumerate(rank_sequences(dist.rank, dist.world, BATCH)):
        k, v, t = synthetic_cache(cfg, sequence, PAST)
        model.kv_write(b, 0, k, v)
        first.append(t)

    model.decode(first, slots, starts, args.warmup)                 # warm-up: capture + W replays
    dist.barrier()
    with ClockSampler(dev) as clocks:
        ms = model.decode_timed(first, slots, starts, args.steps)   # K replays, CUDA events
    dist.barrier()
    ms_max = dist.max(ms)
    value = BATCH * dist.world * args.steps / (ms_max / 1000.0)

    # e2e: the public decode call with host buffers, host round trip every step
    dist.barrier()
    started = time.perf_counter()
    model.decode(first, slots, starts, args.steps, per_step=True)
    e2e_s = dist.max(time.perf_counter() - started)
    e2e = {"value": round(BATCH * dist.world * args.steps / e2e_s, 1), "unit": "tok/s",
           "h2d_bytes_per_step": BATCH * 8, "d2h_bytes_per_step": BATCH * 8}

    # per-kernel times for the roofline (eager steps with events around every launch)
    profile = model.profile(first, slots, starts, 3)
    launches = sum(n for _, n in profile.values()) // 3 + 1          # + the step-advance kernel
    roof = roofline(profile, cfg, BATCH, PAST, "bs64")
    clock_all = dist.gather(clocks.summary())

    bs1 = prefill = None
    if dist.world == 1 and not args.no_bs1:
        bs1 = run_bs1(cfg, model)
    if dist.world == 1 and not args.no_prefill:
        prefill = run_prefill(cfg, weights, dev, 5)
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = cpu_sample(cfg, host_int8_weights(weights), args.cpu_steps)
    model.close()
    if dist.rank != 0:
        return None
    return {"metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"batched greedy decode: {BATCH} sequences per GPU, each from a {PAST}-position "
                                   f"N(0,1) KV cache (configuration 5), one decode step of all per timed step",
                       "model": "Qwen2.5-0.5B architecture, random init N(0,0.02) seed 0, int8-vnni projections, "
                                "fp32 tied LM head", "global_batch": BATCH * dist.world, "past": PAST,
                       "parallelism": f"dp{dist.world} (independent sequences, no collective)",
                       "l2": "inputs larger than L2 (weights 0.9 GB, KV cache 3.3 GB per GPU); no flush"},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
            "clocks": clock_all[0] | {"per_rank": clock_all if dist.world > 1 else None},
            "gpu_launches": launches * args.steps, "bs1": bs1, "prefill": prefill}


def run_bs1(cfg, model) -> dict:
    """Configuration 3 on slot 0: 32-token prompt, then greedy decode up to 1024 positions."""
    prompt = synthetic_prompt(cfg.vocab, BS1_PROMPT)
    _, tok = model.step(prompt, [0] * BS1_PROMPT, list(range(BS1_PROMPT)), [BS1_PROMPT - 1], want_logits=False)
    first = int(tok[0])
    steps = BS1_END - BS1_PROMPT
    model.decode([first], [0], [BS1_PROMPT], 8)                         # warm-up / capture
    with ClockSampler(model.device) as clocks:
        ms = model.decode_timed([first], [0], [BS1_PROMPT], steps)
    profile = model.profile([first], [0], [512], 4)
    phases = model.phase_times([first], [0], [512], 4)
    # the whole step against HBM: bytes a token must read (the layers' int8 weights and KV rows at
    # the workload's mean position, the LM head as read) over the measured time per token
    peak, source = measured_peaks()
    mean_past = (BS1_PROMPT + BS1_END - 1) // 2
    layers = cfg.layers * layer_bytes(cfg, 1, mean_past)
    head_read = algorithmic_bytes("lm_head_argmax", cfg, 1, mean_past)
    head_fp32 = cfg.vocab * cfg.hidden * 4
    s_per_token = ms / steps / 1000.0
    step = {"bytes_per_token": layers + head_read, "achieved": round((layers + head_read) / s_per_token / 1e9, 1),
            "peak": peak, "unit": "GB/s", "frac": round((layers + head_read) / s_per_token / 1e9 / peak, 4),
            "peak_source": source, "mean_past": mean_past,
            "note": "the LM head reads an int8 copy of the embedding (plus exact rechecks); with the float32 "
                    "embedding read instead the same time would be the frac_fp32_head fraction",
            "bytes_per_token_fp32_head": layers + head_fp32,
            "frac_fp32_head": round((layers + head_fp32) / s_per_token / 1e9 / peak, 4)}
    return {"value": round(steps / (ms / 1000.0), 1), "unit": "tok/s", "ms_per_token": round(ms / steps, 4),
            "workload": f"batch 1: {BS1_PROMPT}-token prompt, then {steps} greedy decode steps (past "
                        f"{BS1_PROMPT}..{BS1_END - 1}) (configuration 3)",
            "roofline": roofline(profile, cfg, 1, 512, "bs1"), "step_roofline": step, "clocks": clocks.summary(),
            "phases_us": {"past": 512, "note": "persistent kernel, per layer: microseconds from the layer's start to "
                          "the last CTA reaching each event (globaltimer), mean over layers and 4 steps", **phases}}


PREFILL = 512          # configuration 4
PREFILL_OPS = 2 * PREFILL * 357_826_560          # int8 multiply-adds of the projections, counted as 2 ops
INT8_DENSE_TOPS = 4500.0                         # nominal dense int8 tensor peak of a B200 (no measured figure)


def run_prefill(cfg, weights, dev: int, iters: int) -> dict:
    """Configuration 4: one step over 512 prompt tokens at past 0 (the last row's token), device-timed."""
    from nanocompile_b200 import runtime

    model = runtime.DeviceModel(cfg, weights, "int8", max_rows=PREFILL, slots=1, capacity=PREFILL + 8, device=dev)
    ids = synthetic_prompt(cfg.vocab, PREFILL, seed=4)
    model.step_timed(ids, 0, 0, 2)                                   # warm-up
    ms = model.step_timed(ids, 0, 0, iters)
    model.probe(True)
    model.step(ids, [0] * PREFILL, list(range(PREFILL)), [PREFILL - 1], want_logits=False)
    kinds = model.probe(False)
    model.close()
    proj_ms = sum(kinds.get(k, (0.0, 0))[0] for k in ("qkv_projection", "o_projection", "gate_up_projection",
                                                       "down_projection"))
    total = sum(v[0] for v in kinds.values())
    tops = PREFILL_OPS / (ms / 1e3) / 1e12
    proj_tops = PREFILL_OPS / (proj_ms / 1e3) / 1e12 if proj_ms else None
    return {"value": round(PREFILL / (ms / 1e3), 1), "unit": "tok/s", "ms": round(ms, 4),
            "workload": f"one {PREFILL}-token prompt step at past 0, int8-vnni (configuration 4), last row's token",
            "int8_tops": round(tops, 2), "projection_ms": round(proj_ms, 4),
            "projection_int8_tops": round(proj_tops, 2) if proj_tops else None,
            "tensor_frac_of_nominal_int8": round(tops / INT8_DENSE_TOPS, 4),
            "projection_tensor_frac_of_nominal_int8": round(proj_tops / INT8_DENSE_TOPS, 4) if proj_tops else None,
            "note": "useful int8 ops 2*512*357.8M over the step time; the projections run on the dp4a kernels "
                    "(the tcgen05 kind::i8 kernel, NC_TC_I8=1, measured slower)",
            "kernel_shares": {k: round(v[0] / total, 3) for k, v in sorted(kinds.items(), key=lambda x: -x[1][0])}}


def run_reference(args) -> dict | None:
    """The reference's CPU implementation of the path, on this arm's metric. Under torchrun only
    rank 0 works and prints; the other ranks exit at once (no process group is made)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    cfg = QWEN2_0_5B
    wq = host_int8_weights(synthetic_weights(cfg, seed=0))
    base = cpu_sample(cfg, wq, max(args.steps, 1), warmup=args.warmup)
    return {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"batched greedy decode from {PAST}-position N(0,1) KV caches (configuration 5), "
                                   f"sequences decoded one after another on the host",
                       "model": "Qwen2.5-0.5B architecture, random init N(0,0.02) seed 0, int8-vnni"},
            "cpu_baseline": base, "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}


def run_phase6(args) -> dict:
    """A/B rounds in one process, the way the reference's bench/phase6.py compares engines: every
    round times one greedy decode step of one sequence of the batched workload (past 2048) on each
    engine, the engine order rotating from round to round; medians and minima per engine, and the
    rounds this backend won (a sign test). Each measurement is appended to ``--records`` as a JSON
    line. Engines: this backend end to end (host ids in, host token out, one graph replay) and the
    reference's compiled step at each thread count of the NANOCOMPILE_THREADS sweep."""
    cfg, weights, model = build_model(0, 1, PAST + 128, max_rows=1)
    keys, values, first = synthetic_cache(cfg, 0, PAST)
    model.kv_write(0, 0, keys, values)
    ref, kind = cpu_model(cfg, host_int8_weights(weights), thread_counts()[0])
    engines = ["b200"] + [f"{kind}@{n}" for n in thread_counts()]
    records, per = [], {e: [] for e in engines}
    pos = PAST
    model.decode([first], [0], [pos], 2, per_step=True)               # warm: capture
    for r in range(args.phase6):
        order = engines[r % len(engines):] + engines[: r % len(engines)]
        for e in order:
            if e == "b200":
                n = 64
                started = time.perf_counter()
                model.decode([first], [0], [pos], n, per_step=True)
                dt = (time.perf_counter() - started) / n
            else:
                n = 2
                ref.set_threads(int(e.split("@")[1])) if hasattr(ref, "set_threads") else None
                ref.step([first], keys, values, last_only=True)     # warm at this thread count
                started = time.perf_counter()
                for _ in range(n):
                    ref.step([first], keys, values, last_only=True)
                dt = (time.perf_counter() - started) / n
            per[e].append(dt)
            rec = {"part": "speed", "round": r, "engine": e, "seconds_per_step": dt, "steps": n, "past": PAST,
                   "order": order}
            records.append(rec)
    model.close()
    Path(args.records).parent.mkdir(parents=True, exist_ok=True)
    with open(args.records, "a") as fh:
        for rec in records:
            fh.write(json.dumps(rec) + "\n")
    best_ref = min((e for e in engines if e != "b200"), key=lambda e: statistics.median(per[e]))
    wins = sum(1 for a, b in zip(per["b200"], per[best_ref]) if a < b)
    return {"phase6": True, "rounds": args.phase6, "records": args.records,
            "median_ms": {e: round(statistics.median(v) * 1e3, 4) for e, v in per.items()},
            "min_ms": {e: round(min(v) * 1e3, 4) for e, v in per.items()},
            "best_reference": best_ref, "b200_wins": wins, "sign_test_p": round(0.5 ** args.phase6, 6) if wins == args.phase6 else None,
            "speedup_median": round(statistics.median(per[best_ref]) / statistics.median(per["b200"]), 1)}


def run_projections(rows: int, iters: int) -> dict:
    """The batched int8 projections alone at the 0.5B model's shapes, each entry point timed with
    CUDA events on the launching stream (after 3 untimed launches): the tensor-core kernel
    (nc_matmul_i8_tc) against the default dp4a one (nc_matmul_i8_vnni; its SwiGLU form without the
    quantized output). Random bytes: the time does not depend on the values."""
    import ctypes

    import torch

    from nanocompile_b200 import runtime as rt

    L = rt.library()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(0)

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    out = {}
    for name, (n, k, epi, pro) in {"qkv_projection": (1152, 896, 1, 0), "o_projection": (896, 896, 2, 2),
                                   "gate_up_projection": (4864, 896, 4, 0), "down_projection": (896, 4864, 2, 2)}.items():
        xq = t(rng.integers(-127, 128, (rows, k), dtype=np.int8))
        xs = t(np.abs(rng.standard_normal((rows, k // 32))).astype(np.float32))
        off = t(rng.standard_normal(rows).astype(np.float32))
        bs = t(rng.integers(-500, 500, (rows, k // 32), dtype=np.int32))
        w, w2 = t(rng.integers(0, 256, (n, k), dtype=np.uint8)), t(rng.integers(0, 256, (n, k), dtype=np.uint8))
        s1, s2 = (t(np.abs(rng.standard_normal(n)).astype(np.float32) * 1e-3) for _ in range(2))
        y = torch.zeros((rows, n), dtype=torch.float32, device=dev)
        extra = {1: t(rng.standard_normal(n).astype(np.float32)), 2: y, 4: w2}[epi]
        qo = torch.zeros((rows, n), dtype=torch.int8, device=dev)
        xo = torch.zeros((rows, n // 32), dtype=torch.float32, device=dev)
        bo = torch.zeros((rows, n // 32), dtype=torch.int32, device=dev)
        ptr = lambda x: x.data_ptr() if x is not None else None                      # noqa: E731
        calls = {"tcgen05": (L.nc_matmul_i8_tc, [y, xq, xs, off, w, s1, extra, s2 if epi == 4 else None,
                                                  bs if pro else None, qo, xo, bo], [rows, n, k, epi, pro, 0])}
        if not pro:                                 # the dp4a entry point takes given offsets
            e2 = 3 if epi == 4 else epi
            calls["dp4a"] = (L.nc_matmul_i8_vnni, [y, xq, xs, off, w, s1, extra, s2 if e2 == 3 else None],
                             [rows, n, k, e2])
        out[name] = {}
        for kind, (fn, p, sz) in calls.items():
            pp = (ctypes.c_void_p * len(p))(*[ptr(x) for x in p])
            ss = (ctypes.c_int64 * len(sz))(*sz)
            st = ctypes.c_void_p(stream.cuda_stream)
            for _ in range(3):
                rt.check(fn(pp, ss, st))
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(iters):
                rt.check(fn(pp, ss, st))
            b.record()
            torch.cuda.synchronize()
            out[name][kind] = round(a.elapsed_time(b) * 1000 / iters, 2)
    rt.device_faults()
    return {"projections_us": out, "rows": rows, "iters": iters}


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=64)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--no-bs1", action="store_true", help="skip the batch-1 measurement")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    parser.add_argument("--no-prefill", action="store_true", help="skip the configuration-4 prefill measurement")
    parser.add_argument("--phase6", type=int, default=0, metavar="ROUNDS",
                        help="alternating-order A/B rounds of one decode step: this backend against the reference "
                             "at each thread count (JSON lines to --records)")
    parser.add_argument("--records", default=str(ROOT / "gpurun_out" / "phase6_results.jsonl"))
    parser.add_argument("--projections", type=int, default=0, metavar="ROWS",
                        help="time the batched int8 projection entry points alone at ROWS rows")
    parser.add_argument("--prefill-only", action="store_true",
                        help="time configuration 4 alone (STEPS timed steps after 2) and print its object")
    parser.add_argument("--cpu-steps", type=int, default=8)
    parser.add_argument("--batch", type=int, default=BATCH, help="sequences per GPU (profiling runs only)")
    parser.add_argument("--past", type=int, default=PAST, help="cached positions at the first step (profiling runs only)")
    args = parser.parse_args()
    globals().update(BATCH=args.batch, PAST=args.past)
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.phase6:
        print(json.dumps(run_phase6(args)), flush=True)
        return 0
    if args.projections:
        print(json.dumps(run_projections(args.projections, max(args.steps, 1))), flush=True)
        return 0
    if args.prefill_only:
        print(json.dumps(run_prefill(QWEN2_0_5B, synthetic_weights(QWEN2_0_5B, seed=0), 0, max(args.steps, 1))), flush=True)
        return 0
    if args.impl == "reference":
        line = run_reference(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    dist = RankGroup("nccl")
    try:
        line = run_ours(args, dist)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
