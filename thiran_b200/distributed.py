"""Leading-axis sharding and the few collectives the hot path needs.

The reference has no distributed execution (its src/distributed only prints a
CPU/GPU partition, src/distributed/PartitionPlanner.cpp:6-32). Here regions
shard along the leading axis with no data-path collective; the full-tensor
sum combines one f64 partial per rank, and MLP data parallelism all-reduces
the weight gradients. The process group is torch.distributed (NCCL on GPUs,
gloo for the CPU tests); kernels never touch peer memory.
"""
from __future__ import annotations


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous leading-axis block of `rank`: (start, count). The first
    total % world ranks take one extra row, so every row is owned once."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank outside world")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Maximum of a per-rank scalar (device time of the slowest rank)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def combine_partial_sums(partial, dist=None):
    """Sums per-rank f64 partials (a 1-element tensor) in place; every rank
    ends with the global total. NCCL's ring/tree order is fixed for a given
    world size, so the combination is reproducible run to run."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(partial)
    return partial


def allreduce_gradients(tensors, dist=None):
    """Sums data-parallel gradients across ranks in place (the caller's loss
    scaling already divides by the global batch)."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        for t in tensors:
            dist.all_reduce(t)
    return tensors
