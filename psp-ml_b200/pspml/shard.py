"""Batch sharding across devices: contiguous slices, replicated weights, no
collective on the hot path (each rank writes its disjoint slice of the
logits; the host gather is a concatenation in rank order)."""
from __future__ import annotations


def slice_for(batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous slice: ceil(batch / world) per rank,
    the last ranks taking what remains (possibly nothing)."""
    if world <= 0 or not 0 <= rank < world or batch < 0:
        raise ValueError("bad shard arguments")
    per = -(-batch // world)
    start = min(batch, rank * per)
    stop = min(batch, start + per)
    return start, stop


def all_slices(batch: int, world: int) -> list[tuple[int, int]]:
    return [slice_for(batch, world, r) for r in range(world)]
