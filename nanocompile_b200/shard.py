"""Data-parallel decode: one process per GPU, each decoding its own sequences.

The reference has no multi-device path: ``Qwen2.forward`` runs one sequence's step on one
host (``nanocompile/models/qwen2.py:313-346``). Sequences are independent, so the B200 build
scales by giving every rank a disjoint set of them -- sequence ``rank * per_rank + b`` -- with
no collective on the data path. The host-side group (rank, world, a gather of small records)
is supplied by the caller: ``bench.py`` uses ``torch.distributed`` for the barrier and the
max-over-ranks timing; nothing in this package needs it.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from typing import Protocol


class HostGroup(Protocol):
    """What sharding needs from the process group: this rank, the world, a gather of records."""

    rank: int
    world: int

    def gather(self, obj) -> list: ...


def rank_sequences(rank: int, world: int, per_rank: int) -> range:
    """The sequence indices rank ``rank`` of ``world`` decodes; together they are 0..world*per_rank-1."""
    if not 0 <= rank < world or per_rank < 0:
        raise ValueError(f"rank {rank} of {world} with {per_rank} sequences each")
    return range(rank * per_rank, (rank + 1) * per_rank)


def decode_shard(group: HostGroup, per_rank: int, decode: Callable[[Sequence[int]], list[list[int]]]
                 ) -> list[list[int]]:
    """Decode this rank's sequences with ``decode(sequence_indices) -> tokens per sequence`` and
    return every sequence's tokens in global order (gathered once at the end; nothing is exchanged
    while decoding)."""
    mine = rank_sequences(group.rank, group.world, per_rank)
    tokens = decode(list(mine))
    if len(tokens) != len(mine):
        raise ValueError(f"decode returned {len(tokens)} sequences for {len(mine)}")
    return [t for part in group.gather(tokens) for t in part]
