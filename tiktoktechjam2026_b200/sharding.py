"""Batch sharding of the forward pass across the GPUs of one node.

Sequences are independent (attention never crosses a sequence, every other op
is per row), so a batch splits into contiguous slices, one per rank, with no
exchange during compute.  The only communication is the optional final
gather of the outputs to rank 0.  One process per GPU; ranks come from
``torch.distributed``.
"""

from __future__ import annotations

import ctypes
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib


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


class PeerGatherBuffer:
    """One FP32 output buffer on rank 0's GPU that every rank's batch slice is pushed into.

    Rank 0 allocates ``slots`` buffers shaped ``[batch, *row_shape]`` and exports
    them (``tt_peer_export``); the other ranks map them into their own address
    space (``tt_peer_open``), so ``dst(slot)`` is where this rank's slice goes:
    on rank 0 its own memory (the forward writes there directly), on the
    others rank 0's memory across NVLink, written by the copy engines
    (``tt_model_forward_gather``).  The handles travel through the process
    group's object collectives; nothing is exchanged during compute.
    """

    def __init__(self, batch: int, row_shape: Sequence[int], rank: int, world: int, device: torch.device,
                 slots: int = 1, group=None) -> None:
        self.batch = batch
        self.row_shape = tuple(int(d) for d in row_shape)
        self.rank, self.world = rank, world
        self.start, self.stop = shard_bounds(batch, world, rank)
        row_elems = 1
        for d in self.row_shape:
            row_elems *= d
        self._row_bytes = row_elems * 4
        self.buffers: List[torch.Tensor] = []
        self._opened: List[Tuple[int, int]] = []
        handles = None
        if rank == 0:
            handles = []
            for _ in range(slots):
                buf = torch.empty((batch,) + self.row_shape, dtype=torch.float32, device=device)
                self.buffers.append(buf)
                h = (ctypes.c_char * _lib.TT_PEER_HANDLE_BYTES)()
                off = ctypes.c_size_t()
                with torch.cuda.device(device):
                    _lib.check(_lib.lib().tt_peer_export(buf.data_ptr(), h, ctypes.byref(off)))
                handles.append((bytes(h), int(off.value)))
        if world > 1:
            box = [handles]
            dist.broadcast_object_list(box, src=0, group=group)
            handles = box[0]
        self._bases: List[int] = []
        if rank == 0:
            self._bases = [b.data_ptr() for b in self.buffers]
        else:
            with torch.cuda.device(device):
                for raw, off in handles:
                    ptr = ctypes.c_void_p()
                    h = (ctypes.c_char * _lib.TT_PEER_HANDLE_BYTES).from_buffer_copy(raw)
                    _lib.check(_lib.lib().tt_peer_open(h, off, ctypes.byref(ptr)))
                    self._opened.append((ptr.value, off))
                    self._bases.append(ptr.value)

    def dst(self, slot: int = 0) -> int:
        """Device address of this rank's slice of buffer ``slot`` (rank 0's memory)."""
        return self._bases[slot] + self.start * self._row_bytes

    def local_view(self, slot: int = 0) -> torch.Tensor:
        """Rank 0: buffer ``slot`` as a tensor (the gathered batch once every push has landed)."""
        if self.rank != 0:
            raise RuntimeError("only rank 0 holds the gather buffer")
        return self.buffers[slot]

    def close(self) -> None:
        for ptr, off in self._opened:
            try:
                _lib.lib().tt_peer_close(ptr, off)
            except Exception:  # pragma: no cover - interpreter teardown
                pass
        self._opened = []
