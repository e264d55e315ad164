"""Batch x head slice sharding across GPUs (no collective on the data path).

Slices are independent (reference grid.y = slice, src/flash.zig:51; kernels
offset by slice * stride, src/flash_h64_bn32.zig:51-55), so rank r of N owns
the contiguous range [r*bh//N, (r+1)*bh//N) -- sizes differ by at most one.
"""
from __future__ import annotations


def slice_range(batch_heads: int, world: int, rank: int) -> tuple[int, int]:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    return batch_heads * rank // world, batch_heads * (rank + 1) // world
