"""Pages over GPUs: one process per GPU (launched by torchrun), each detecting its own pages.

Pages are independent (the reference's page pipeline, src/bin/ocr-bench.rs:133-161, runs each
page on its own), so the data path has no collective: a rank only needs to know which pages are
its own.  The process group carries the timing plumbing alone: a barrier around the timed region
and the maximum of the ranks' device times.  Works with the nccl backend (GPU tensors) and with
gloo (CPU tensors).
"""
from __future__ import annotations

from typing import List


def pages_of(rank: int, world: int, n_pages: int) -> List[int]:
    """Global page indices of `rank` when `n_pages` pages are split over `world` ranks: contiguous
    blocks, the first n_pages % world ranks one page larger (strong scaling)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, extra = divmod(n_pages, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def weak_pages_of(rank: int, per_rank: int) -> List[int]:
    """Global page indices of `rank` when every rank detects `per_rank` pages (weak scaling)."""
    return list(range(rank * per_rank, (rank + 1) * per_rank))


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of `value` over the ranks of the default process group (the value itself
    without one).  `device`: where the reduction tensor lives (a CUDA device for nccl, None or
    CPU for gloo)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(device_index=None):
    """A barrier over the default process group, if any (device_ids for nccl)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        if device_index is None:
            dist.barrier()
        else:
            dist.barrier(device_ids=[device_index])
