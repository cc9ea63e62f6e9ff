"""Column sharding of the projections over the GPUs of one node.

Each rank holds a contiguous range of a projection's output rows (the
columns of y) and computes that slice of y from a replicated x; an NCCL
all-gather reassembles y only where the next projection needs all of it.
The fused [gate | up] weight shards both halves with the same row range, so
the SwiGLU epilogue stays local.  Shards are multiples of 16 rows (one MMA
tile) and equal in size, the layout `all_gather_into_tensor` concatenates.

The reference engine is single-device; this module is the host logic of the
multi-GPU extension and carries no arithmetic of its own.
"""
from __future__ import annotations

from typing import Optional

import torch


def shard_rows(total: int, world: int, rank: int, align: int = 16):
    """(first row, rows) of `rank`'s equal shard of `total` output rows."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    per, rem = divmod(total, world)
    if rem or per % align:
        raise ValueError(f"{total} rows do not split into {world} shards of a multiple of {align}")
    return rank * per, per


def gather_rows(local: torch.Tensor, full: Optional[torch.Tensor] = None, group=None) -> torch.Tensor:
    """All-gather the ranks' y slices [m, rows] into y [m, world * rows] in
    rank order.  The collective concatenates the ranks' [m, rows] blocks;
    they are then reordered to [m][world * rows] (for m = 1, the decode case,
    the reorder is free)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    m, rows = local.shape
    cat = torch.empty((world * m, rows), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(cat, local.contiguous(), group=group)
    out = cat.view(world, m, rows).permute(1, 0, 2).reshape(m, world * rows)
    if full is not None:
        full.copy_(out)
        return full
    return out
