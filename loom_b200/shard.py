"""Shard planning for the multi-GPU entries.

A global 1D tensor of n elements is split into `world` contiguous shards in
rank order.  Every shard boundary is a multiple of 4 elements (16 bytes), so
a shard of a 16-byte aligned buffer starts 16-byte aligned and takes the
float4 path of the kernels.  Shard sizes differ by at most 7 elements; a
rank may get an empty shard when n < 4*world (the `_dist` entries accept
n_local = 0 and contribute the reduction identity).
"""

from __future__ import annotations

from typing import List, Tuple


def shard_bounds(n: int, world: int, align: int = 4) -> List[Tuple[int, int]]:
    """[(start, stop)] for ranks 0..world-1, covering [0, n) in order."""
    if n < 0 or world < 1 or align < 1:
        raise ValueError("need n >= 0, world >= 1, align >= 1")
    units = -(-n // align)                 # aligned units, the last may be partial
    base, extra = divmod(units, world)
    bounds, start = [], 0
    for r in range(world):
        stop = min(n, start + (base + (1 if r < extra else 0)) * align)
        bounds.append((start, stop))
        start = stop
    return bounds


def shard(tensor, world: int, rank: int):
    """Rank `rank`'s contiguous view of a 1D tensor (no copy)."""
    start, stop = shard_bounds(int(tensor.shape[0]), world)[rank]
    return tensor[start:stop]
