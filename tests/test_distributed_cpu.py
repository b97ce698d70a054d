"""World-size-2 gloo tests of the multi-GPU host logic on CPU: leading-axis
sharding covers every row once, sharded evaluation of a region equals the
unsharded result, partial sums and gradients combine to the global values,
and the max-over-ranks timing rule."""
import os
import socket

import numpy as np
import pytest

from thiran_b200.distributed import shard_range

torch = pytest.importorskip("torch")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("total,world", [(8192, 2), (8192, 8), (17, 4), (3, 8), (0, 2)])
def test_shards_cover_rows_once(total, world):
    seen = []
    for r in range(world):
        start, count = shard_range(total, r, world)
        seen.extend(range(start, start + count))
    assert seen == list(range(total))


def _worker(rank, world, port, result_path):
    import torch.distributed as dist
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    import oracle_lib
    from thiran_b200 import regions
    from thiran_b200.distributed import (allreduce_gradients, combine_partial_sums, max_over_ranks,
                                         shard_range)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(1)
    a = rng.integers(-1000, 1001, (37, 64), dtype=np.int64)
    b = rng.integers(-1000, 1001, (37, 64), dtype=np.int64)
    start, count = shard_range(a.shape[0], rank, world)
    spec = regions.i64_region()
    mine = oracle_lib.region_eval(spec, [a[start:start + count].copy(), b[start:start + count].copy()])
    gathered = [None] * world
    dist.all_gather_object(gathered, (start, mine))
    x = np.random.default_rng(3).standard_normal(10007).astype(np.float32)
    s0, c0 = shard_range(x.size, rank, world)
    partial = torch.tensor([oracle_lib.sum_all_f64(x[s0:s0 + c0])], dtype=torch.float64)
    combine_partial_sums(partial, dist)
    g = torch.full((4,), float(rank + 1))
    allreduce_gradients([g], dist)
    slowest = max_over_ranks(1.0 + rank, dist)
    if rank == 0:
        full = np.concatenate([m for _, m in sorted(gathered, key=lambda t: t[0])])
        expected = oracle_lib.region_eval(spec, [a, b])
        ok = (np.array_equal(full, expected)
              and abs(partial.item() - oracle_lib.sum_all_f64(x)) <= 1e-9 * max(1.0, abs(partial.item()))
              and torch.equal(g, torch.full((4,), float(sum(range(1, world + 1)))))
              and slowest == float(world))
        with open(result_path, "w") as f:
            f.write("ok" if ok else "mismatch")
    dist.destroy_process_group()


def test_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    result = tmp_path / "result.txt"
    mp.start_processes(_worker, args=(2, free_port(), str(result)), nprocs=2, join=True, start_method="spawn")
    assert result.read_text() == "ok"


def test_compact_reduction_needs_the_fused_update():
    """The bf16 sharded form keeps each tile's f32 weights on its owner, so
    it is refused without the update in the reduction (before any buffer is
    made)."""
    import torch.distributed as dist
    from thiran_b200.distributed import FusedGradientAllReduce
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(free_port()))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        with pytest.raises(ValueError):
            FusedGradientAllReduce(object(), dist, mode="switch", update=False, compact=True)
        with pytest.raises(ValueError):
            FusedGradientAllReduce(object(), dist, mode="ring")
    finally:
        dist.destroy_process_group()
