"""Multi-GPU tests (each skipped with fewer devices than its ranks):
data-parallel MLP steps whose gradient all-reduce is fused into the
weight-gradient GEMMs (peer loads/stores or in-switch reduction over NVLink)
or done by NCCL after the backward pass equal the single-process full-batch
step and follow the oracle's full-batch step (biases, SGD with momentum), at
2, 4 and 8 ranks; unbinding the fused all-reduce (close()) returns the
session to its own buffers. Each test runs spawned ranks over NCCL."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


MOMENTUM = 0.9
LR = 0.05


def problem():
    """Shared synthetic problem: data, weights and (non-zero) biases."""
    batch, d_in, hidden, d_out = 512, 256, 512, 256
    rng = np.random.default_rng(8)
    x = rng.standard_normal((batch, d_in)).astype(np.float32)
    t = rng.standard_normal((batch, d_out)).astype(np.float32)
    w1 = (rng.uniform(-1, 1, (d_in, hidden)) * 0.08).astype(np.float32)
    w2 = (rng.uniform(-1, 1, (hidden, d_out)) * 0.08).astype(np.float32)
    b1 = (rng.standard_normal(hidden) * 0.05).astype(np.float32)
    b2 = (rng.standard_normal(d_out) * 0.05).astype(np.float32)
    return x, t, w1, w2, b1, b2


def session(thb, batch, global_batch, device, w1, w2, b1, b2):
    """A biased, momentum-SGD session whose parameters live in torch tensors."""
    d_in, hidden = w1.shape
    d_out = w2.shape[1]
    s = thb.MlpSession(batch, d_in, hidden, d_out, global_batch=global_batch, device=device)
    cuda = lambda a: torch.from_numpy(a).cuda()
    s.set_weights(cuda(w1), cuda(w2))
    s.set_biases(cuda(b1), cuda(b2))
    s.set_momentum(MOMENTUM)
    params = {"w1": s.bind(thb.MLP_W1, cuda(w1)), "w2": s.bind(thb.MLP_W2, cuda(w2)),
              "b1": s.bind(thb.MLP_B1, cuda(b1)), "b2": s.bind(thb.MLP_B2, cuda(b2))}
    return s, params


def _mlp_rank(rank, world, port, mode, out_path):
    import datetime
    import sys
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import thiran_b200 as thb
    from thiran_b200.distributed import FusedGradientAllReduce, allreduce_gradients, bind_bias_gradients
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    x, t, w1, w2, b1, b2 = problem()
    batch = x.shape[0]
    local = batch // world
    xs = torch.from_numpy(x[rank * local:(rank + 1) * local].copy()).cuda()
    ts = torch.from_numpy(t[rank * local:(rank + 1) * local].copy()).cuda()
    s, params = session(thb, local, batch, rank, w1, w2, b1, b2)
    dw1 = s.bind(thb.MLP_DW1, torch.empty(w1.shape, device="cuda"))
    dw2 = s.bind(thb.MLP_DW2, torch.empty(w2.shape, device="cuda"))
    mc = None
    if mode != "nccl":
        mc = FusedGradientAllReduce(s, dist, mode=mode)
        if not mc.available:
            dist.destroy_process_group()
            if rank == 0:
                open(out_path, "w").write("unavailable")
            return
        dw1, dw2 = mc.buffers[0][1], mc.buffers[1][1]
        dbias = mc.bias_grads
    else:
        dbias = bind_bias_gradients(s)
    for _ in range(3):
        s.forward_backward(xs, ts)
        if mc:
            mc.after_backward()
        else:
            allreduce_gradients([dw1, dw2, dbias], dist)
        s.apply_sgd(LR)
    thb.check_device_status(rank)
    torch.cuda.synchronize()
    results = dict(dw1=dw1.cpu().numpy(), dw2=dw2.cpu().numpy(), dbias=dbias.cpu().numpy(),
                   **{k: v.cpu().numpy() for k, v in params.items()})
    if mc:
        # Unbind between steps: dW returns to the session's own buffers, so a
        # further (local, unreduced) backward pass leaves the symmetric
        # buffers untouched.
        sym = [dw1.clone(), dw2.clone()]
        mc.close()
        own = [s.buffer(thb.MLP_DW1)[0], s.buffer(thb.MLP_DW2)[0]]
        results["unbound"] = np.array(own[0] != dw1.data_ptr() and own[1] != dw2.data_ptr())
        s.forward_backward(xs, ts)
        thb.check_device_status(rank)
        torch.cuda.synchronize()
        results["untouched"] = np.array(torch.equal(sym[0], dw1) and torch.equal(sym[1], dw2))
        dist.barrier()
    if rank == 0:
        np.savez(out_path, **results)
    s.release()
    dist.barrier()
    dist.destroy_process_group()


def single_gpu_reference():
    import thiran_b200 as thb
    from thiran_b200.distributed import bind_bias_gradients
    x, t, w1, w2, b1, b2 = problem()
    s, params = session(thb, x.shape[0], x.shape[0], 0, w1, w2, b1, b2)
    dw1 = s.bind(thb.MLP_DW1, torch.empty(w1.shape, device="cuda"))
    dw2 = s.bind(thb.MLP_DW2, torch.empty(w2.shape, device="cuda"))
    dbias = bind_bias_gradients(s)
    X, T = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
    for _ in range(3):
        s.forward_backward(X, T)
        s.apply_sgd(LR)
    torch.cuda.synchronize()
    return dict(dw1=dw1.cpu().numpy(), dw2=dw2.cpu().numpy(), dbias=dbias.cpu().numpy(),
                **{k: v.cpu().numpy() for k, v in params.items()})


def _device_tensor(ptr, like):
    """A torch view of `like.numel()` f32 values at device address `ptr`
    (through the CUDA array interface; the memory stays the session's)."""
    class _Mem:
        __cuda_array_interface__ = {"shape": tuple(like.shape), "typestr": "<f4", "data": (ptr, False),
                                    "version": 3, "strides": None}
    return torch.as_tensor(_Mem(), device="cuda")


def rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["peer", "switch", "nccl"])
def test_data_parallel_mlp_matches_full_batch(tmp_path, mode, world):
    if gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    out = str(tmp_path / f"{mode}{world}.npz")
    mp.start_processes(_mlp_rank, args=(world, free_port(), mode, out), nprocs=world, join=True,
                       start_method="spawn")
    if os.path.exists(out) and open(out, "rb").read(11) == b"unavailable":
        pytest.skip("no NVLink multicast on this system")
    got = dict(np.load(out))
    ref = single_gpu_reference()
    # Same arithmetic, different batch split of the f32 reductions.
    for k in ("dw1", "dw2", "dbias"):
        assert rel(got[k], ref[k]) <= 1e-2, k
    for k in ("w1", "w2", "b1", "b2"):
        assert rel(got[k], ref[k]) <= 1e-4, k
    # The oracle's full-batch step (the bound of the single-GPU oracle test).
    orc = oracle_steps()
    for k in ("w1", "w2", "b1", "b2"):
        assert rel(got[k], orc[k]) <= 1e-3, k
    if mode != "nccl":
        assert bool(got["unbound"]) and bool(got["untouched"])


def oracle_steps():
    """Three full-batch steps of the oracle (biases, SGD with momentum)."""
    import oracle_lib
    x, t, w1, w2, b1, b2 = problem()
    ws = [w1.copy(), w2.copy(), b1.copy(), b2.copy()]
    vel = [np.zeros_like(a) for a in (w1, b1, w2, b2)]
    for _ in range(3):
        oracle_lib.mlp_step_ex(x, t, ws[0], ws[1], LR, ws[2], ws[3], MOMENTUM, vel)
    return dict(w1=ws[0], w2=ws[1], b1=ws[2], b2=ws[3])


def _update_rank(rank, world, port, mode, out_path):
    """Two data-parallel runs over the same process group: the all-reduce
    fused into the dW GEMMs followed by the separate update pass, and the
    update applied by each tile's owner inside the all-reduce."""
    import datetime
    import sys
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import thiran_b200 as thb
    from thiran_b200.distributed import FusedGradientAllReduce
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    x, t, w1, w2, b1, b2 = problem()
    batch = x.shape[0]
    local = batch // world
    xs = torch.from_numpy(x[rank * local:(rank + 1) * local].copy()).cuda()
    ts = torch.from_numpy(t[rank * local:(rank + 1) * local].copy()).cuda()
    results = {}
    for fused in (False, True):
        s, params = session(thb, local, batch, rank, w1, w2, b1, b2)
        mc = FusedGradientAllReduce(s, dist, mode=mode, update=fused)
        if not mc.available:
            dist.destroy_process_group()
            if rank == 0:
                open(out_path, "w").write("unavailable")
            return
        for _ in range(3):
            if fused:
                s.forward_backward_update(xs, ts, LR)
            else:
                s.forward_backward(xs, ts)
            mc.after_backward()
            s.apply_sgd(LR)
        thb.check_device_status(rank)
        torch.cuda.synchronize()
        weights = [mc.param_handles[0][1][0][0], mc.param_handles[1][1][0][0]] if fused else [params["w1"], params["w2"]]
        copies = [mc.param_handles[0][1][1][0], mc.param_handles[1][1][1][0]] if fused else None
        tag = "fused" if fused else "plain"
        results[f"{tag}_w1"] = weights[0].cpu().numpy()
        results[f"{tag}_w2"] = weights[1].cpu().numpy()
        results[f"{tag}_b1"] = params["b1"].cpu().numpy()
        results[f"{tag}_b2"] = params["b2"].cpu().numpy()
        if copies is not None:
            # Every rank holds the same parameters and bf16 copies.
            for k, (w, c) in enumerate(zip(weights, copies)):
                gathered = [torch.empty_like(w) for _ in range(world)]
                dist.all_gather(gathered, w)
                results[f"ranks_equal_w{k + 1}"] = np.array(all(torch.equal(g, w) for g in gathered))
                results[f"copy_matches_w{k + 1}"] = np.array(torch.equal(c, w.to(torch.bfloat16)))
            # close(): W1 and W2 move back into the session's own buffers
            # with the current values.
            current = [w.clone() for w in weights]
            mc.close()
            own = [s.buffer(thb.MLP_W1)[0], s.buffer(thb.MLP_W2)[0]]
            restored = all(p != w.data_ptr() for p, w in zip(own, weights))
            for p, w in zip(own, current):
                view = torch.empty_like(w)
                view.copy_(_device_tensor(p, w))
                restored = restored and torch.equal(view, w)
            results["closed_restores_weights"] = np.array(restored)
        dist.barrier()
        s.release()
    if rank == 0:
        np.savez(out_path, **results)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["peer", "switch"])
def test_update_fused_into_the_all_reduce(tmp_path, mode, world):
    """The owner-applied update gives the same parameter bits as the separate
    update pass after the fused all-reduce, on every rank, with bf16 copies
    that match, and follows the single-process full-batch step."""
    if gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    out = str(tmp_path / f"update_{mode}{world}.npz")
    mp.start_processes(_update_rank, args=(world, free_port(), mode, out), nprocs=world, join=True,
                       start_method="spawn")
    if os.path.exists(out) and open(out, "rb").read(11) == b"unavailable":
        pytest.skip("no NVLink multicast on this system")
    got = dict(np.load(out))
    for k in ("w1", "w2", "b1", "b2"):
        assert np.array_equal(got[f"fused_{k}"].view(np.uint32), got[f"plain_{k}"].view(np.uint32)), k
    for k in ("1", "2"):
        assert bool(got[f"ranks_equal_w{k}"]) and bool(got[f"copy_matches_w{k}"]), k
    assert bool(got["closed_restores_weights"])
    ref = single_gpu_reference()
    for k in ("w1", "w2", "b1", "b2"):
        assert rel(got[f"fused_{k}"], ref[k]) <= 1e-4, k


def _compact_rank(rank, world, port, mode, out_path):
    """Three data-parallel steps with the bf16 sharded reduction: bf16
    gradient tiles summed by their owners in f32, the owner's f32 weights
    updated, the bf16 copy broadcast; then the f32 weights gathered."""
    import datetime
    import sys
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import thiran_b200 as thb
    from thiran_b200.distributed import FusedGradientAllReduce
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    x, t, w1, w2, b1, b2 = problem()
    batch = x.shape[0]
    local = batch // world
    xs = torch.from_numpy(x[rank * local:(rank + 1) * local].copy()).cuda()
    ts = torch.from_numpy(t[rank * local:(rank + 1) * local].copy()).cuda()
    s, params = session(thb, local, batch, rank, w1, w2, b1, b2)
    mc = FusedGradientAllReduce(s, dist, mode=mode, update=True, compact=True)
    if not mc.available:
        dist.destroy_process_group()
        if rank == 0:
            open(out_path, "w").write("unavailable")
        return
    for _ in range(3):
        s.forward_backward_update(xs, ts, LR)
        mc.after_backward()
        s.apply_sgd(LR)
    thb.check_device_status(rank)
    torch.cuda.synchronize()
    copies = [mc.param_handles[0][1][1][0].clone(), mc.param_handles[1][1][1][0].clone()]
    weights = [w.clone() for w in mc.gather_parameters()]
    results = {"w1": weights[0].cpu().numpy(), "w2": weights[1].cpu().numpy(),
               "b1": params["b1"].cpu().numpy(), "b2": params["b2"].cpu().numpy()}
    for k, (w, c) in enumerate(zip(weights, copies)):
        gathered = [torch.empty_like(w) for _ in range(world)]
        dist.all_gather(gathered, w)
        results[f"ranks_equal_w{k + 1}"] = np.array(all(torch.equal(g, w) for g in gathered))
        results[f"copy_matches_w{k + 1}"] = np.array(torch.equal(c, w.to(torch.bfloat16)))
    mc.close()
    own = [s.buffer(thb.MLP_W1)[0], s.buffer(thb.MLP_W2)[0]]
    results["closed_restores_weights"] = np.array(all(torch.equal(_device_tensor(p, w), w)
                                                      for p, w in zip(own, weights)))
    dist.barrier()
    s.release()
    if rank == 0:
        np.savez(out_path, **results)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["peer", "switch"])
def test_compact_sharded_reduction(tmp_path, mode, world):
    """bf16 gradient payload and owner-sharded f32 weights: every rank ends
    with the same gathered weights, bf16 copies equal to their rounding,
    close() restores them into the session, and the trajectory follows the
    single-process full-batch step and the oracle's (the bf16 rounding of
    each rank's gradient tile moves the update by ~2^-8 of itself)."""
    if gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    out = str(tmp_path / f"compact_{mode}{world}.npz")
    mp.start_processes(_compact_rank, args=(world, free_port(), mode, out), nprocs=world, join=True,
                       start_method="spawn")
    if os.path.exists(out) and open(out, "rb").read(11) == b"unavailable":
        pytest.skip("no NVLink multicast on this system")
    got = dict(np.load(out))
    for k in ("1", "2"):
        assert bool(got[f"ranks_equal_w{k}"]) and bool(got[f"copy_matches_w{k}"]), k
    assert bool(got["closed_restores_weights"])
    ref = single_gpu_reference()
    orc = oracle_steps()
    for k in ("w1", "w2", "b1", "b2"):
        assert rel(got[k], ref[k]) <= 1e-3, k
        assert rel(got[k], orc[k]) <= 1e-3, k

