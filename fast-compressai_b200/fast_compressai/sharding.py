"""Batch sharding over the GPUs of one box.

Images are independent, so a batch splits into contiguous slices, one per
rank, and each rank compresses and decompresses its slice on its own GPU with
its own payload.  No tensor data moves between GPUs.  The only collective is
one ``all_gather`` of each rank's payload sizes at the end, to report the
total compressed size (any process group: NCCL on GPUs, gloo on CPU).
"""

from __future__ import annotations

import torch


def shard_bounds(batch: int, rank: int, world: int) -> tuple[int, int]:
    """Images [start, end) of ``rank`` when ``batch`` images are split over ``world`` ranks.

    The first ``batch % world`` ranks take one image more; every image is in
    exactly one shard.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if batch < 0:
        raise ValueError("batch must be non-negative")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def payload_stats(payload) -> list[int]:
    """[packed_bytes, header_bytes, sum of max_rounds, images] of one WarpDivPayload."""
    return [int(payload.packed.numel()), int(payload.header_bytes), int(payload.max_rounds.sum()),
            int(payload.batch)]


def gather_payload_stats(stats: list[int], device: torch.device | str = "cpu", group=None) -> dict:
    """All-gather every rank's ``payload_stats`` and total them.

    Every rank calls this once, in the same order relative to its other
    collectives.  With world size 1 (or no process group) it returns this
    rank's figures.
    """
    import torch.distributed as dist

    local = torch.tensor(stats, dtype=torch.int64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        parts = [torch.zeros_like(local) for _ in range(dist.get_world_size(group))]
        dist.all_gather(parts, local, group=group)
        rows = [p.tolist() for p in parts]
    else:
        rows = [local.tolist()]
    return {
        "per_rank": rows,
        "packed_bytes": sum(r[0] for r in rows),
        "header_bytes": sum(r[1] for r in rows),
        "rounds": sum(r[2] for r in rows),
        "images": sum(r[3] for r in rows),
    }
