"""Leading-axis sharding and the few collectives the hot path needs.

The reference has no distributed execution (its src/distributed only prints a
CPU/GPU partition, src/distributed/PartitionPlanner.cpp:6-32). Here regions
shard along the leading axis with no data-path collective; the full-tensor
sum combines one f64 partial per rank, and MLP data parallelism all-reduces
the weight gradients, either by NCCL all-reduce after the backward pass or
inside the weight-gradient GEMMs over NVLink (FusedGradientAllReduce). The
process group is torch.distributed (NCCL on GPUs, gloo for the CPU tests).
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


def fused_reduction_mode(world: int) -> str:
    """Transport of the fused gradient all-reduce for `world` ranks: plain
    peer loads/stores ("peer") move 2(world-1)/world of the gradients each
    way per GPU, the in-switch reduction ("switch") about 1 + 1/world, so
    peer mode wins at 2 ranks and switch mode from 3 up. Measured on 256 MiB
    of f32 over NVLink 5: 2 ranks 0.41 ms peer vs 0.70 ms switch; 8 ranks
    0.90 ms peer vs 0.62 ms switch."""
    return "peer" if world <= 2 else "switch"


class FusedGradientAllReduce:
    """Weight gradients all-reduced inside the dW GEMMs of an MlpSession: the
    dW buffers and their per-tile signal words live in torch symmetric memory
    that every rank maps; each GEMM stores and announces its tiles, and each
    tile's owner rank sums it over all ranks and writes the total to every
    rank (thb_mlp_bind_reduction), by plain NVLink loads/stores or inside
    NVSwitch (`mode`, default fused_reduction_mode(world)). `available` is
    False when switch mode was asked for and the fabric has no multicast
    (callers then all-reduce with NCCL)."""

    BARRIER_TIMEOUT_MS = 60000

    def __init__(self, session, dist, group=None, mode=None, update=False, compact=False):
        """`update=True` also moves W1, W2 and their bf16 copies into
        symmetric memory (thb_mlp_bind_update), so that a step can run
        session.forward_backward_update(): each tile's owner applies the
        optimizer step in the reduction and writes the new weights to every
        rank. `compact=True` (needs `update`) reduces bf16 gradient tiles
        and keeps each tile's f32 weights on its owner only, broadcasting
        just the bf16 copy (THB_REDUCE_BF16_SHARDED): about a fifth of the
        NVLink bytes; gather_parameters() or close() assembles the f32
        weights."""
        import torch
        import torch.distributed._symmetric_memory as symm_mem
        from . import MLP_DW1, MLP_DW2, MLP_W1, MLP_W2
        self.group = group or dist.group.WORLD
        rank, world = dist.get_rank(self.group), dist.get_world_size(self.group)
        self.mode = mode or fused_reduction_mode(world)
        if self.mode not in ("peer", "switch"):
            raise ValueError(f"unknown fused all-reduce mode {self.mode!r}")
        if compact and not update:
            raise ValueError("the compact reduction applies the optimizer step in the reduction (update=True)")
        self.compact = bool(compact)
        self.buffers, self.handles = [], []
        shapes = [(MLP_DW1, (session.d_in, session.hidden)), (MLP_DW2, (session.hidden, session.d_out))]
        words = [session.reduction_flag_words(which) for which, _ in shapes]
        self.flags = symm_mem.empty((sum(words),), dtype=torch.int32, device="cuda")
        self.flags.zero_()
        self.flag_handle = symm_mem.rendezvous(self.flags, self.group)
        for which, shape in shapes:
            t = symm_mem.empty(shape, dtype=torch.bfloat16 if self.compact else torch.float32, device="cuda")
            h = symm_mem.rendezvous(t, self.group)
            self.buffers.append((which, t))
            self.handles.append(h)
        self.update = bool(update)
        self.param_handles = []
        if self.update:
            for which, shape in ((MLP_W1, (session.d_in, session.hidden)), (MLP_W2, (session.hidden, session.d_out))):
                pair = []
                for dtype in (torch.float32, torch.bfloat16):
                    t = symm_mem.empty(shape, dtype=dtype, device="cuda")
                    pair.append((t, symm_mem.rendezvous(t, self.group)))
                self.param_handles.append((which, pair))
        handles = self.handles + [h for _, pair in self.param_handles for _, h in pair]
        self.available = self.mode == "peer" or all(h.multicast_ptr for h in handles)
        # Every rank's signal words are zero before any rank can announce.
        self.flag_handle.barrier(channel=0, timeout_ms=self.BARRIER_TIMEOUT_MS)
        if self.available:
            offset = 0
            flag_ptrs = [int(p) for p in self.flag_handle.buffer_ptrs]
            switch = self.mode == "switch"
            for ((which, t), h), n in zip(zip(self.buffers, self.handles), words):
                session.bind_reduction(which, [int(p) for p in h.buffer_ptrs], [p + 4 * offset for p in flag_ptrs],
                                       rank, world, h.multicast_ptr if switch else None)
                if self.compact:
                    from . import REDUCE_BF16_SHARDED
                    session.set_reduction_format(which, REDUCE_BF16_SHARDED)
                offset += n
            if self.update:
                # The session's current weights move into the symmetric
                # buffers (set_weights also refreshes the bf16 copies).
                old = [session.buffer(MLP_W1)[0], session.buffer(MLP_W2)[0]]
                for which, ((_, hp), (_, hc)) in self.param_handles:
                    session.bind_update(which, [int(p) for p in hp.buffer_ptrs], [int(p) for p in hc.buffer_ptrs],
                                        hp.multicast_ptr if switch else None, hc.multicast_ptr if switch else None)
                session.set_weight_pointers(old[0], old[1], torch.cuda.current_stream().cuda_stream)
                torch.cuda.current_stream().synchronize()
                self.flag_handle.barrier(channel=0, timeout_ms=self.BARRIER_TIMEOUT_MS)
        self.dist = dist
        self.session = session
        self.bias_grads = bind_bias_gradients(session)

    def close(self):
        """Unbinds the session from the symmetric buffers, so that they can
        be freed while the session lives on: dW returns to the session's own
        buffers, and with `update` the current weights are copied back into
        the session's own W1 and W2. Call it on every rank, between steps.
        With `update` and momentum, each tile's velocity lives on its owner
        rank only, so the velocities are not carried over: set_momentum
        restarts them from zero before a step without the fused update.
        The bias gradients stay bound to `self.bias_grads` (an ordinary
        device tensor), which must outlive the session's later steps."""
        import torch
        from . import MLP_DW1, MLP_DW2, MLP_W1, MLP_W2
        if not self.available or self.session is None:
            return
        weights = [pair[0][0] for _, pair in self.param_handles]
        if self.compact:
            # Each rank holds only its tiles' f32 weights: assemble them all,
            # and let every rank finish reading its peers before any rebinds.
            stream = torch.cuda.current_stream()
            for which, _ in self.param_handles:
                self.session.gather_parameters(which, stream.cuda_stream)
            stream.synchronize()
            self.flag_handle.barrier(channel=0, timeout_ms=self.BARRIER_TIMEOUT_MS)
        for which, _ in self.param_handles:
            self.session.bind_update(which, None, None)
        for which in (MLP_DW1, MLP_DW2):
            self.session.bind_reduction(which, None, None, 0, 1)
        if weights:
            stream = torch.cuda.current_stream()
            self.session.set_weight_pointers(weights[0].data_ptr(), weights[1].data_ptr(), stream.cuda_stream)
            stream.synchronize()
        self.session = None

    def gather_parameters(self):
        """With `compact`: this rank's f32 W1 and W2 (the symmetric buffers)
        assembled from their tile owners; every rank calls it between steps."""
        import torch
        stream = torch.cuda.current_stream()
        for which, _ in self.param_handles:
            self.session.gather_parameters(which, stream.cuda_stream)
        stream.synchronize()
        self.flag_handle.barrier(channel=0, timeout_ms=self.BARRIER_TIMEOUT_MS)
        return [pair[0][0] for _, pair in self.param_handles]

    def after_backward(self):
        """Wait until every rank's owned tiles hold their totals everywhere;
        the bias gradients (hidden + out floats) are summed by NCCL."""
        self.flag_handle.barrier(channel=1, timeout_ms=self.BARRIER_TIMEOUT_MS)
        if self.bias_grads is not None:
            self.dist.all_reduce(self.bias_grads, group=self.group)


def bind_bias_gradients(session):
    """When the session has biases, binds db1 and db2 to one torch tensor
    [hidden + out] (db2 right after db1) so one collective sums both, and
    returns it; otherwise None."""
    import torch
    from . import MLP_B1, MLP_DB1, MLP_DB2
    if session.buffer(MLP_B1)[1] == 0:
        return None
    grads = torch.empty(session.hidden + session.d_out, dtype=torch.float32, device="cuda")
    session.bind(MLP_DB1, grads[:session.hidden])
    session.bind(MLP_DB2, grads[session.hidden:])
    return grads


def allreduce_gradients(tensors, dist=None):
    """Sums data-parallel gradients across ranks in place (the caller's loss
    scaling already divides by the global batch)."""
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        for t in tensors:
            dist.all_reduce(t)
    return tensors
