"""Batch sharding of the DCNv2 layer over several GPUs (one process per GPU).

The layer has no exchange step: image n depends only on x[n], offset[n], mask[n] and the
(replicated) weights. Rank g of G takes the contiguous slice [start, stop) of the global batch
given by `shard_range` and runs its own forward on its own GPU, stream and workspace. No
collective touches the data; results are reassembled only if a caller asks for them.
"""
from __future__ import annotations

from typing import Tuple


def shard_range(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous slice of the batch owned by `rank`: sizes differ by at most one image, the
    first `global_batch % world` ranks take the extra image."""
    if world < 1 or not 0 <= rank < world or global_batch < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_batch(tensors, world: int, rank: int):
    """Slices every batch-major tensor of (x, offset, mask) to this rank's images."""
    n = int(tensors[0].shape[0])
    a, b = shard_range(n, world, rank)
    return [t[a:b].contiguous() for t in tensors], (a, b)
