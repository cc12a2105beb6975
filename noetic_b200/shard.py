"""Stream sharding across GPUs.

Decode streams are independent (each has its own LmState, infer.rs:21-23,
and its own sampler Rng), so N GPUs split the streams into N contiguous
shards with the weights replicated on every GPU.  The hot path has no
collective; results are gathered on the host afterwards.
"""

from __future__ import annotations


def shard_range(n_streams: int, world: int, rank: int) -> tuple[int, int]:
    """(first, count) of rank's contiguous shard; the first n % world ranks
    take one extra stream."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(n_streams, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def shard_plan(n_streams: int, world: int) -> list[tuple[int, int]]:
    return [shard_range(n_streams, world, r) for r in range(world)]
