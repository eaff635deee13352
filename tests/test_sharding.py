"""Host logic of the multi-GPU path on the CPU: shard bounds, and the one
collective (all_gather of payload sizes) run by two gloo ranks."""

from __future__ import annotations

import socket
from types import SimpleNamespace

import pytest
import torch
import torch.multiprocessing as mp

from fast_compressai import sharding


@pytest.mark.parametrize("batch,world", [(512, 8), (24, 1), (24, 5), (3, 4), (0, 2), (7, 7)])
def test_shard_bounds_partition_the_batch(batch, world):
    spans = [sharding.shard_bounds(batch, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == batch
    for (a, b), (c, _) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1 and sum(sizes) == batch


def test_shard_bounds_reject_bad_ranks():
    with pytest.raises(ValueError):
        sharding.shard_bounds(8, 2, 2)
    with pytest.raises(ValueError):
        sharding.shard_bounds(8, 0, 0)


def _fake_payload(rank: int):
    # packed bytes, header, rounds and batch differ per rank
    return SimpleNamespace(packed=torch.zeros(1000 + 128 * rank, dtype=torch.uint8), header_bytes=48 + 16 * rank,
                           max_rounds=torch.full((2 + rank, 3), 4 + rank, dtype=torch.int32), batch=2 + rank)


def _worker(rank: int, world: int, port: int, queue) -> None:
    import torch.distributed as dist
    from datetime import timedelta

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        got = sharding.gather_payload_stats(sharding.payload_stats(_fake_payload(rank)))
        queue.put((rank, got))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gather_payload_stats_over_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want_rows = [sharding.payload_stats(_fake_payload(r)) for r in range(world)]
    for rank in range(world):
        got = results[rank]
        assert got["per_rank"] == want_rows
        assert got["packed_bytes"] == sum(r[0] for r in want_rows)
        assert got["rounds"] == sum(r[2] for r in want_rows)
        assert got["images"] == 5


def test_gather_payload_stats_single_process():
    got = sharding.gather_payload_stats(sharding.payload_stats(_fake_payload(1)))
    assert got["per_rank"] == [[1128, 64, 3 * 3 * 5, 3]]
