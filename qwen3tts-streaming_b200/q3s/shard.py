"""Row sharding of a sampling step across the GPUs of one node.

Rows (streams) are independent, so a step shards by contiguous row blocks with
no collective on the data path: rank r samples rows ``row_range(r, world, B)``
from inputs generated for exactly those rows (the workload generators key
every row by its global index, so the union of the shards is the single-GPU
batch).  ``gather_ids`` brings the sampled ids to rank 0 for verification
only, outside any timed region.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def row_range(rank: int, world: int, total: int) -> tuple[int, int]:
    """Contiguous block of rows for ``rank``; the first ``total % world``
    ranks get one extra row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(int(total), int(world))
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def gather_ids(ids: torch.Tensor, total: int, group: Optional[dist.ProcessGroup] = None) -> Optional[torch.Tensor]:
    """Concatenate every rank's ids (in rank order) on rank 0; other ranks
    get None.  Works with gloo (CPU tensors) and nccl (CUDA tensors)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = [row_range(r, world, total)[1] - row_range(r, world, total)[0] for r in range(world)]
    width = max(sizes)
    pad = torch.full((width,) + tuple(ids.shape[1:]), -1, dtype=ids.dtype, device=ids.device)
    pad[: ids.shape[0]] = ids
    bufs = [torch.empty_like(pad) for _ in range(world)] if rank == 0 else None
    dist.gather(pad, gather_list=bufs, dst=0, group=group)
    if rank != 0:
        return None
    return torch.cat([b[:n] for b, n in zip(bufs, sizes)], dim=0)


def max_over_ranks(value: float, device: torch.device, group: Optional[dist.ProcessGroup] = None) -> float:
    """Max of a per-rank scalar (e.g. a device-timed duration) over ranks."""
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
