"""Batch sharding of the forward pass across the GPUs of one node.

Sequences are independent (attention never crosses a sequence, every other op
is per row), so a batch splits into contiguous slices, one per rank, with no
exchange during compute.  The only communication is the optional final
gather of the outputs to rank 0.  One process per GPU; ranks come from
``torch.distributed``.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def shard_bounds(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of ``rank``'s contiguous slice; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def sharded_forward(
    fn: Callable[[torch.Tensor, Optional[torch.Tensor]], torch.Tensor],
    x: torch.Tensor,
    mask: Optional[torch.Tensor],
    rank: int,
    world: int,
) -> torch.Tensor:
    """Runs ``fn`` on this rank's batch slice of the full batch ``x``/``mask``."""
    s, e = shard_bounds(x.shape[0], world, rank)
    return fn(x[s:e], None if mask is None else mask[s:e])


def gather_to_rank0(local: torch.Tensor, batch: int, rank: int, world: int, group=None) -> Optional[torch.Tensor]:
    """Gathers every rank's output slice into the full [batch, ...] tensor on rank 0.

    Slices may differ in size by one sequence, so they are padded to the
    largest slice for the collective and trimmed afterwards.  Returns None on
    ranks other than 0.
    """
    if world == 1:
        return local
    largest = shard_bounds(batch, world, 0)[1]
    padded = local
    if local.shape[0] < largest:
        pad = torch.zeros((largest - local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        padded = torch.cat([local, pad], dim=0)
    bufs = [torch.empty_like(padded) for _ in range(world)] if rank == 0 else None
    dist.gather(padded.contiguous(), gather_list=bufs, dst=0, group=group)
    if rank != 0:
        return None
    parts = []
    for r in range(world):
        s, e = shard_bounds(batch, world, r)
        parts.append(bufs[r][: e - s])
    return torch.cat(parts, dim=0)
