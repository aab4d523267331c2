"""Data-parallel decode host logic on two gloo ranks (CPU): disjoint shards that cover every
sequence, the max over ranks of the timed region, and gathered results that equal one process
decoding all sequences (the sequences are independent, so sharding changes nothing)."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from bench import RankGroup
from nanocompile_b200.shard import decode_shard, rank_sequences

PER_RANK, STEPS, PAST = 3, 4, 16


def test_rank_sequences_partition_the_batch():
    world, per = 4, 5
    seen = [s for r in range(world) for s in rank_sequences(r, world, per)]
    assert seen == list(range(world * per))
    with pytest.raises(ValueError):
        rank_sequences(4, 4, 5)


def test_single_process_group_is_the_identity():
    g = RankGroup()
    assert (g.rank, g.world) == (0, 1)
    assert g.max(2.5) == 2.5 and g.gather("x") == ["x"]
    g.close()


def _tiny_decoder():
    from nanocompile_b200 import quantize as q
    from nanocompile_b200.model import TINY, synthetic_cache, synthetic_weights
    from oracle.oracle import OracleModel

    model = OracleModel(TINY, q.int8_projection_weights(synthetic_weights(TINY, seed=5), TINY), "int8", threads=1)

    def decode(sequences):
        out = []
        for s in sequences:
            keys, values, first = synthetic_cache(TINY, s, PAST)
            out.append(model.greedy([first], STEPS, past_keys=keys, past_values=values))
        return out

    return decode


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    try:
        group = RankGroup("gloo", timeout_s=60)
        tokens = decode_shard(group, PER_RANK, _tiny_decoder())
        slowest = group.max(float(rank + 1) * 1.5)
        group.barrier()
        group.close()
        queue.put((rank, tokens, slowest, None))
    except Exception as e:  # reported to the parent, which fails the test
        queue.put((rank, None, None, repr(e)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_decode_disjoint_shards_equal_to_one_process():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, tokens, slowest, err = queue.get(timeout=240)
            assert err is None, f"rank {rank}: {err}"
            results[rank] = (tokens, slowest)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    expected = _tiny_decoder()(list(range(world * PER_RANK)))
    for rank in range(world):
        tokens, slowest = results[rank]
        assert tokens == expected                       # every rank gathers the whole batch, in order
        assert slowest == 3.0                           # the max over ranks, seen by every rank
    assert len({tuple(t) for t in expected}) > 1        # the sequences really differ


def _killed_rank_main(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import time

    group = RankGroup("gloo", timeout_s=10)
    if rank == 1:
        os._exit(3)                                    # this worker dies between steps, holding nothing
    started = time.monotonic()
    try:
        group.barrier()                                # the next host-side step of the survivors
        queue.put((rank, None, time.monotonic() - started))
    except Exception as e:                             # the failure is seen on the host, as an error
        queue.put((rank, repr(e), time.monotonic() - started))


def test_a_killed_worker_is_detected_by_the_survivors():
    """A rank that exits between steps: the surviving rank's next host collective ends with an
    error within the process group's timeout instead of waiting for ever."""
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_killed_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        rank, err, seconds = queue.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert rank == 0 and err is not None and seconds < 60, (rank, err, seconds)
    assert procs[1].exitcode == 3
