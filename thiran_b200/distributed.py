"""Leading-axis sharding and the few collectives the hot path needs.

The reference has no distributed execution (its src/distributed only prints a
CPU/GPU partition, src/distributed/PartitionPlanner.cpp:6-32). Here regions
shard along the leading axis with no data-path collective; the full-tensor
sum combines one f64 partial per rank, and MLP data parallelism all-reduces
the weight gradients, either by NCCL all-reduce after the backward pass or
inside the weight-gradient GEMM epilogues through NVLink multicast memory
(MulticastGradients). The process group is torch.distributed (NCCL on GPUs,
gloo for the CPU tests).
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


class MulticastGradients:
    """Weight-gradient buffers in NVLink multicast (NVLS) memory for the fused
    GEMM -> cross-GPU reduction of an MlpSession: every rank maps the same
    buffers, the dW GEMM epilogues add their tiles through the multicast
    address (multimem.red), and each rank reads the summed gradients from its
    own copy. Built on torch symmetric memory; `available` is False when the
    device or fabric has no multicast support (callers then all-reduce)."""

    BARRIER_TIMEOUT_MS = 60000

    def __init__(self, session, dist, group=None):
        import torch
        import torch.distributed._symmetric_memory as symm_mem
        from . import MLP_DW1, MLP_DW2
        self.group = group or dist.group.WORLD
        self.buffers, self.handles = [], []
        shapes = [(MLP_DW1, (session.d_in, session.hidden)), (MLP_DW2, (session.hidden, session.d_out))]
        for which, shape in shapes:
            t = symm_mem.empty(shape, dtype=torch.float32, device="cuda")
            h = symm_mem.rendezvous(t, self.group)
            self.buffers.append((which, t))
            self.handles.append(h)
        self.available = all(h.multicast_ptr for h in self.handles)
        if self.available:
            for (which, t), h in zip(self.buffers, self.handles):
                session.bind(which, t)
                session.bind_reduction(which, h.multicast_ptr)

    def before_step(self):
        """Zero this rank's copies, then wait until every rank has (so no
        rank's reductions land in a buffer another rank is still reading)."""
        for _, t in self.buffers:
            t.zero_()
        self.handles[0].barrier(channel=0, timeout_ms=self.BARRIER_TIMEOUT_MS)

    def after_backward(self):
        """Wait until every rank's reductions have landed."""
        self.handles[0].barrier(channel=1, timeout_ms=self.BARRIER_TIMEOUT_MS)


def allreduce_gradients(tensors, dist=None):
    """Sums data-parallel gradients across ranks in place (the caller's loss
    scaling already divides by the global batch)."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        for t in tensors:
            dist.all_reduce(t)
    return tensors
