"""Batch sharding across GPUs: independent sequences, no collective.

A batch of n sequences is split into contiguous shards, one per rank; shard r
holds sequences [start, start + size).  Every rank can regenerate its own
sequences' prompts (tie_b200.synth.prompt_ids draws each sequence from its own
seeded stream), so no data moves between ranks; only the timing (and, in tests,
the token ids) are gathered at the end.
"""
from __future__ import annotations


def shard_range(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """(start, size) of rank's contiguous share; shares differ by at most one."""
    if world <= 0 or not 0 <= rank < world or n_items < 0:
        raise ValueError(f"bad shard request n={n_items} rank={rank} world={world}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def dist_env() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment (1 process if unset)."""
    import os
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))
