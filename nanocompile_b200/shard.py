"""Data-parallel decode: one process per GPU, each decoding its own sequences.

The reference has no multi-device path: ``Qwen2.forward`` runs one sequence's step on one
host (``nanocompile/models/qwen2.py:313-346``). Sequences are independent, so the B200 build
scales by giving every rank a disjoint set of them -- sequence ``rank * per_rank + b`` -- with
no collective on the data path. The process group exists only for the barrier around the
timed region, the max of the ranks' device times and gathering small per-rank records.
``backend`` is NCCL on GPUs and gloo on the host (the CPU tests).
"""

from __future__ import annotations

import datetime
import os
from collections.abc import Callable, Sequence


def rank_sequences(rank: int, world: int, per_rank: int) -> range:
    """The sequence indices rank ``rank`` of ``world`` decodes; together they are 0..world*per_rank-1."""
    if not 0 <= rank < world or per_rank < 0:
        raise ValueError(f"rank {rank} of {world} with {per_rank} sequences each")
    return range(rank * per_rank, (rank + 1) * per_rank)


class RankGroup:
    """Rank and world from the torchrun environment, and the three host-side collectives."""

    def __init__(self, backend: str | None = None, timeout_s: float = 120.0):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dist = None
        self.device = None
        if self.world > 1:
            import torch
            import torch.distributed as dist

            backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
            kwargs = {}
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                self.device = torch.device("cuda", self.local)
                kwargs["device_id"] = self.device
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
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


def decode_shard(group: RankGroup, per_rank: int, decode: Callable[[Sequence[int]], list[list[int]]]) -> list[list[int]]:
    """Decode this rank's sequences with ``decode(sequence_indices) -> tokens per sequence`` and
    return every sequence's tokens in global order (gathered; no collective during decoding)."""
    mine = rank_sequences(group.rank, group.world, per_rank)
    tokens = decode(list(mine))
    if len(tokens) != len(mine):
        raise ValueError(f"decode returned {len(tokens)} sequences for {len(mine)}")
    return [t for part in group.gather(tokens) for t in part]
