"""Batched serving as independent replicas, one process per GPU.

The fused-kernel path has no exchange step, so a batch of sequences is split
into contiguous blocks, one per rank, and every rank runs its own optimised
model (and CUDA graph) on its block. Nothing here runs inside the forward;
``gather_batch`` is a host-side convenience for callers that want the whole
batch back on one rank.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of the sequences `rank` serves: contiguous blocks, the first
    ``batch % world`` ranks taking one extra sequence."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _rank_world(rank, world):
    if rank is None or world is None:
        if dist.is_available() and dist.is_initialized():
            return dist.get_rank(), dist.get_world_size()
        return 0, 1
    return rank, world


def local_shard(tokens: torch.Tensor, rank: int | None = None, world: int | None = None) -> torch.Tensor:
    """This rank's block of sequences (dim 0) of a full batch."""
    rank, world = _rank_world(rank, world)
    s, e = shard_bounds(tokens.shape[0], world, rank)
    return tokens[s:e]


def gather_batch(local: torch.Tensor, batch: int, dst: int = 0) -> torch.Tensor | None:
    """Collect every rank's block (dim 0) on rank `dst` in batch order; other ranks get None.

    Uses the process group's point-to-point ops; blocks may differ in size by one.
    """
    rank, world = _rank_world(None, None)
    if world == 1:
        return local
    if rank != dst:
        dist.send(local.contiguous(), dst)
        return None
    parts = []
    for r in range(world):
        s, e = shard_bounds(batch, world, r)
        if r == rank:
            parts.append(local)
        else:
            buf = torch.empty((e - s,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
            dist.recv(buf, r)
            parts.append(buf)
    return torch.cat(parts, dim=0)
