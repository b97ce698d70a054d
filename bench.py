"""Benchmark of the B200 TensorRegion engine (one JSON line on rank 0).

Default workload: the i64 elementwise region out = (a + b) * a - b on
[8192, 8192] i64 per GPU with a, b uniform integers in [-1000, 1000] (seed
1 + 1000 * rank), checked for overflow. N ranks process N such row blocks of
an [8192 N, 8192] region (weak scaling, no collective). A step is one pass of
the fused region kernel over the rank's block.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                    [--workload i64_region|f32_chain|softmax]

value     device-timed aggregate GB/s (algorithmic bytes: 24 B per element,
          a and b read, out written), inputs resident in HBM; max over ranks.
e2e       the same metric through the public host API (thb_region_execute):
          every step copies the inputs host->device from pinned memory, runs
          the region, reads the result back and checks the error word.
roofline  the fused kernel's achieved GB/s vs the measured HBM copy peak.
The working set (1.5 GiB per step at N=1) is far above the 126 MB L2, so no
L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused-region GB/s and % HBM peak (device-timed) at 1/2/4/8 B200; MLP TFLOP/s"
REF_REGION = {"i64_region": os.path.join(ROOT, "oracle", "_ref", "region_i64_region.so"),
              "f32_chain": os.path.join(ROOT, "oracle", "_ref", "region_f32_chain.so")}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", f"{name}.ncu.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    return None


# ---- workloads ---------------------------------------------------------------------

class Workload:
    name = ""
    bytes_per_element = 0
    dtype = ""
    ncu_name = ""

    def config(self, world):
        raise NotImplementedError


class I64Region(Workload):
    name = "i64_region"
    bytes_per_element = 24
    dtype = "int64"
    rows, cols = 8192, 8192
    ncu_name = "i64_region_8192x8192"

    def build(self, torch, rank, world):
        from thiran_b200 import regions
        g = torch.Generator(device="cuda").manual_seed(1 + 1000 * rank)
        a = torch.randint(-1000, 1001, (self.rows, self.cols), dtype=torch.int64, device="cuda", generator=g)
        b = torch.randint(-1000, 1001, (self.rows, self.cols), dtype=torch.int64, device="cuda", generator=g)
        out = torch.empty_like(a)
        return regions.i64_region(), [a, b], out

    def config(self, world):
        return {"workload": "i64 region (a+b)*a-b, [8192,8192] i64 per GPU, uniform ints [-1000,1000] "
                            "seed 1+1000*rank, overflow-checked",
                "global_shape": [self.rows * world, self.cols], "shard": "one [8192,8192] row block per rank",
                "parallelism": f"row-sharded x{world}, no collective",
                "l2": "working set 1.5 GiB/step per GPU >> 126 MB L2 (no flush needed)"}


class F32Chain(Workload):
    name = "f32_chain"
    bytes_per_element = 8
    dtype = "f32"
    n = 1 << 28
    ncu_name = "f32_chain_2p28"

    def build(self, torch, rank, world):
        from thiran_b200 import regions
        g = torch.Generator(device="cuda").manual_seed(2 + 1000 * rank)
        x = torch.rand(self.n, device="cuda", generator=g) * 2 - 1
        return regions.f32_chain(), [x], torch.empty_like(x)

    def config(self, world):
        return {"workload": "f32 chain ((x*1.5+0.25)*x-x)*0.5+x on 2^28 f32 per GPU, uniform[-1,1] seed 2+1000*rank",
                "global_shape": [self.n * world], "shard": "2^28 elements per rank",
                "parallelism": f"sharded x{world}, no collective", "l2": "2 GiB/step per GPU >> L2"}


class Softmax(Workload):
    name = "softmax"
    bytes_per_element = 8
    dtype = "f32"
    rows, cols = 65536, 4096
    ncu_name = "softmax_65536x4096"
    kernel = "rowWarp softmax (one warp per row, row in registers, warp-shuffle max and sum)"

    def build(self, torch, rank, world):
        from thiran_b200 import regions
        g = torch.Generator(device="cuda").manual_seed(3 + 1000 * rank)
        x = torch.randn((self.rows, self.cols), device="cuda", generator=g)
        return regions.softmax_rows(), [x], torch.empty_like(x)

    def config(self, world):
        return {"workload": "row softmax on [65536,4096] f32 per GPU ~ N(0,1) seed 3+1000*rank",
                "global_shape": [self.rows * world, self.cols], "shard": "one [65536,4096] row block per rank",
                "parallelism": f"row-sharded x{world}, no collective", "l2": "2 GiB/step per GPU >> L2"}


class FullSum(Workload):
    """Full-tensor sum of the [65536, 4096] N(0,1) tensor: every rank sums its
    row shard on the device (two-pass f64 reduction), the per-rank partials
    are combined with an NCCL all-reduce."""
    name = "sum"
    bytes_per_element = 4
    dtype = "f32"
    rows, cols = 65536, 4096
    ncu_name = "full_sum_65536x4096"
    combine = True
    kernel = ("two-pass deterministic f64 full sum: sumAllBulk (48 KiB cp.async.bulk tiles, one partial per SM) "
              "+ sumAllPass2")
    launches_per_step = 2

    def build(self, torch, rank, world):
        from thiran_b200 import regions
        g = torch.Generator(device="cuda").manual_seed(3 + 1000 * rank)
        x = torch.randn(self.rows * self.cols, device="cuda", generator=g)
        return regions.full_sum(), [x], torch.empty(1, device="cuda")

    def config(self, world):
        return {"workload": "full-tensor sum of [65536,4096] f32 per GPU ~ N(0,1) seed 3+1000*rank "
                            "(f64 accumulation)",
                "global_shape": [self.rows * world, self.cols], "shard": "one [65536,4096] row block per rank",
                "parallelism": f"row-sharded x{world}, NCCL all-reduce of one f64 partial per rank"
                               if world > 1 else "single GPU",
                "l2": "1 GiB/step >> L2"}


class Mlp(Workload):
    name = "mlp"
    dtype = "bf16"
    batch, d_in, hidden, d_out = 8192, 4096, 16384, 4096
    ncu_name = "gemm_mlp"

    def flops_per_step(self):
        # 2 forward + 3 backward GEMMs of 2*B*4096*16384 each (the reference's
        # AD also emits a dead dX GEMM, Autodiff.cpp:224, not computed here).
        return 5 * 2 * self.batch * self.d_in * self.hidden

    def config(self, world):
        return {"workload": "2-layer MLP fwd+bwd+SGD (examples/mlp.th structure): batch 8192, 4096->16384->4096, "
                            "broadcast biases (zero-initialised, trained), ReLU, MSE vs N(0,1) targets, "
                            "Xavier-uniform weights, seed 4; bf16 GEMM operands, f32 accumulate",
                "global_batch": self.batch, "dims": [self.d_in, self.hidden, self.d_out],
                "parallelism": f"data-parallel x{world}" if world > 1 else "single GPU",
                "l2": "weights 2x128 MiB bf16 + activations >> 126 MB L2"}


WORKLOADS = {w.name: w for w in (I64Region(), F32Chain(), Softmax(), FullSum(), Mlp())}


def run_mlp(args, workload, torch, dist, thb, world, rank, local, barrier, max_over_ranks):
    b = workload.batch // world
    d_in, hidden, d_out = workload.d_in, workload.hidden, workload.d_out
    g = torch.Generator(device="cuda").manual_seed(4)
    bound1 = (6.0 / (d_in + hidden)) ** 0.5
    bound2 = (6.0 / (hidden + d_out)) ** 0.5
    w1 = (torch.rand((d_in, hidden), device="cuda", generator=g) * 2 - 1) * bound1
    w2 = (torch.rand((hidden, d_out), device="cuda", generator=g) * 2 - 1) * bound2
    gx = torch.Generator(device="cuda").manual_seed(4 + 1000 * rank)
    x = torch.randn((b, d_in), device="cuda", generator=gx)
    t = torch.randn((b, d_out), device="cuda", generator=gx)
    stream = torch.cuda.Stream()
    s = stream.cuda_stream
    session = thb.MlpSession(b, d_in, hidden, d_out, global_batch=workload.batch, device=local)
    dw1 = session.bind(thb.MLP_DW1, torch.empty((d_in, hidden), device="cuda"))
    dw2 = session.bind(thb.MLP_DW2, torch.empty((hidden, d_out), device="cuda"))
    loss = session.bind(thb.MLP_LOSS_SUM, torch.zeros(2, dtype=torch.float64, device="cuda"))
    session.set_weights(w1, w2, s)
    session.set_biases(stream=s)
    lr = 1e-3
    fused = None
    if world > 1 and args.dp_collective != "nccl":
        from thiran_b200.distributed import FusedGradientAllReduce
        from thiran_b200.distributed import fused_reduction_mode
        mode = {"fused": None, "fused-peer": "peer", "fused-switch": "switch"}[args.dp_collective]
        # Measured: the owner-applied update wins in switch mode (8 ranks
        # 2.141 vs 2.204 ms per step) and loses in peer mode (2 ranks 2.87
        # vs 2.79 ms).
        switch = (mode or fused_reduction_mode(world)) == "switch"
        # Measured at 2 ranks (peer mode): 2.907 ms per step compact against
        # 2.795 ms for f32 gradients with the separate update pass, so
        # 'auto' keeps the compact form for switch mode, where the step is
        # bound by NVLink bytes.
        compact = args.dp_format == "bf16-sharded" or (args.dp_format == "auto" and switch)
        update = compact or args.dp_update == "fused" or (args.dp_update == "auto" and switch)
        with torch.cuda.stream(stream):
            fused = FusedGradientAllReduce(session, dist, mode=mode, update=update, compact=compact)
        if not fused.available:
            fused = None
    from thiran_b200.distributed import bind_bias_gradients
    bias_grads = fused.bias_grads if fused else bind_bias_gradients(session)
    collective = None
    if fused:
        collective = ("dW all-reduce fused into the dW GEMMs: per-tile announce, owner rank sums "
                      + ("with NVLink peer loads and stores" if fused.mode == "peer"
                         else "in NVSwitch (multimem.ld_reduce + multimem.st)")
                      + ("; bf16 gradient tiles summed by each tile's owner with f32 accumulation, optimizer step "
                         "applied to the owner's f32 weights (sharded by tile owner), bf16 W written to every rank"
                         if fused.compact else
                         "; optimizer step applied by each tile's owner in the reduction, new W and bf16 W "
                         "written to every rank" if fused.update else "; separate optimizer pass")
                      + "; bias gradients (80 KiB) by NCCL all-reduce")
    elif world > 1:
        collective = "NCCL all-reduce of dW1, dW2 and the bias gradients"
    nvlink = nvlink_bytes_per_step(world, d_in * hidden + hidden * d_out, fused)

    def step(xx=x, tt=t):
        if world == 1:  # thb_mlp_step: the weight updates run in the dW GEMMs' read-out
            session.step(xx, tt, lr, s)
            return
        if fused and fused.update:
            session.forward_backward_update(xx, tt, lr, s)
        else:
            session.forward_backward(xx, tt, s)
        if fused:
            with torch.cuda.stream(stream):
                fused.after_backward()
        elif world > 1:
            with torch.cuda.stream(stream):
                dist.all_reduce(dw1)
                dist.all_reduce(dw2)
                dist.all_reduce(bias_grads)
        session.apply_sgd(lr, s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    thb.check_device_status(local, s)
    session.enable_timing(True)
    sampler = ClockSampler(local)
    sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    gemm_ms, gemm_launches = session.read_timing()
    session.enable_timing(False)
    thb.check_device_status(local, s)
    total_ms = max_over_ranks(start.elapsed_time(end))
    flops_rank = workload.flops_per_step() / world
    value = workload.flops_per_step() * args.steps / (total_ms / 1e3) / 1e12
    achieved = (flops_rank / 5) * gemm_launches / (gemm_ms / 1e3) / 1e12

    # End to end: X, T from pinned host memory every step, loss read back
    # every step. A training loop's input pipeline: step i+1's batch crosses
    # PCIe on a copy stream into the second of two device buffers while
    # step i computes; the host reads step i's loss during step i+1.
    hx = x.cpu().pin_memory()
    ht = t.cpu().pin_memory()
    host_loss = [torch.zeros(2, dtype=torch.float64).pin_memory() for _ in range(2)]
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 10))
    copy_stream = torch.cuda.Stream()
    xs, ts = [x, torch.empty_like(x)], [t, torch.empty_like(t)]
    ready = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    loss_read = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]

    def prefetch(i):
        j = i % 2
        if used[j]:
            copy_stream.wait_event(consumed[j])
        with torch.cuda.stream(copy_stream):
            xs[j].copy_(hx, non_blocking=True)
            ts[j].copy_(ht, non_blocking=True)
            ready[j].record(copy_stream)

    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    prefetch(0)
    with torch.cuda.stream(stream):
        for i in range(e2e_steps):
            j = i % 2
            if i + 1 < e2e_steps:
                prefetch(i + 1)
            stream.wait_event(ready[j])
            step(xs[j], ts[j])
            consumed[j].record(stream)
            used[j] = True
            host_loss[j].copy_(loss, non_blocking=True)
            loss_read[j].record(stream)
            if i > 0:
                loss_read[1 - j].synchronize()
        stream.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = workload.flops_per_step() * e2e_steps / e2e_s / 1e12

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tflops, sample = mlp_cpu_sample(lr, 3)
        cpu_baseline = {"value": tflops, "unit": "TFLOP/s", "cores": 1, "kind": "port", "sample": sample}
    if rank == 0:
        peak = 1383.9
        peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
        peak_kind = "fallback 1.4 PFLOP/s sustained"
        if os.path.exists(peaks_path):
            with open(peaks_path) as f:
                peak = float(json.load(f)["bf16_tflops_sustained"])
            peak_kind = "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (torch.Generator on device, seeded)",
            "config": dict(workload.config(world), **({"gradient_reduction": collective} if collective else {}),
                           **({"nvlink_bytes_per_step_per_gpu": nvlink} if nvlink else {}),
                           optimizer=("SGD applied in the dW GEMMs' read-out (thb_mlp_step), biases by a separate "
                                      "pass" if world == 1 else
                                      "SGD applied by each tile's owner inside the fused all-reduce, biases by a "
                                      "separate pass" if fused and fused.update else
                                      "SGD pass after the gradient all-reduce")),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak,
                         # mean DRAM bytes of the step's GEMM launches (1 GPU capture)
                         "traffic": ncu_traffic(workload.ncu_name) if world == 1 else None,
                         "kernel": "tcgen05 GEMM (256x256 tiles on CTA pairs, cta_group::2, TMEM accumulators; "
                                   "dW GEMMs with the fused all-reduce: 128x256 tiles on single CTAs)",
                         "algorithmic_flops_per_launch": flops_rank / 5,
                         "avg_launch_ms": gemm_ms / max(1, gemm_launches), "peak_source": peak_kind},
            "cpu_baseline": cpu_baseline,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": (x.numel() + t.numel()) * 4,
                    "d2h_bytes_per_step": 16, "steps": e2e_steps,
                    "api": "thb_mlp_* (inputs from pinned host, next batch copied during the current step; "
                           "loss read back every step)"},
            # Per step: X cast, 5 GEMMs, loss + dY, loss-partial sum, two
            # bias-gradient column reductions, and the optimizer: the two bias
            # updates, plus the two weight passes unless the weights were
            # updated inside the GEMMs (1 GPU) or the all-reduce.
            "gpu_launches": args.steps * (12 + (2 if world > 1 and not (fused and fused.update) else 0)),
            "clocks": clocks,
            "loss": float(loss[0].item()) / (workload.batch * d_out) if world == 1 else None,
        }
        print(json.dumps(line), flush=True)
    session.release()
    return 0



def nvlink_bytes_per_step(world, elements, fused):
    """Per GPU and direction, bytes of weight-gradient traffic over NVLink in
    one data-parallel step of `elements` weights on `world` ranks (the 80 KiB
    of bias gradients aside). Switch mode counts what crosses each GPU's
    links (NVSwitch reads a rank's tile once per multimem.ld_reduce and
    replicates a multimem.st), peer mode the loads and stores of other
    ranks' memory."""
    if world <= 1:
        return None
    w = float(world)
    if fused is None:  # NCCL ring all-reduce of f32 gradients
        out = inp = 2.0 * (w - 1) / w * 4
        how = "NCCL ring all-reduce of f32 gradients: 2(w-1)/w x 4 B per element each way"
    elif fused.compact:
        if fused.mode == "switch":
            out = inp = 2.0
            how = "bf16 tiles read once by the switch, bf16 weights multicast: 2 B per element each way"
        else:
            out = inp = 4.0 * (w - 1) / w
            how = "owner loads the other ranks' bf16 tiles and stores the bf16 weights to them: 4(w-1)/w B each way"
    elif fused.mode == "switch":
        reply = 6.0 if fused.update else 4.0  # new f32 + bf16 weights, or the f32 sum
        out = 4.0 * (w - 1) / w + reply / w
        inp = 4.0 / w + reply * (w - 1) / w
        how = "f32 tiles read once by the switch, the f32 sum (or f32 and bf16 weights) multicast"
    else:
        reply = 6.0 if fused.update else 4.0
        out = inp = 4.0 * (w - 1) / w + reply * (w - 1) / w
        how = "owner loads the other ranks' f32 tiles and stores the sum (or the weights) to them"
    return {"out": int(out * elements), "in": int(inp * elements), "model": how}


def bind_host_to_gpu(torch, device):
    """Restricts this process to the host cores local to `device` (the PCIe
    root's NUMA node), so that pinned host buffers allocated afterwards are
    placed in that node's memory; returns the core list, or None where the
    topology is not exposed."""
    try:
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        text = open(f"/sys/bus/pci/devices/{bus}/local_cpulist").read().strip()
        cpus = set()
        for part in text.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return text
    except (OSError, ValueError, AttributeError):
        return None


# ---- clocks ------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.1)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.seek(0)
        rows = [r.split(", ") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows if len(r) >= 9 for k in range(4) if r[5 + k].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows), "window": "warm-up + timed region, 50 ms sampling"}


# ---- CPU baseline (reference CPU path) ----------------------------------------------

class RefArg(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("dtype", C.c_uint32), ("rank", C.c_uint32), ("reserved", C.c_uint32),
                ("shape", C.POINTER(C.c_uint64)), ("data", C.c_void_p), ("count", C.c_uint64)]


def reference_entry(workload):
    """The reference's native CPU region (emitted by its NativeCpu emitter and
    compiled like its JIT, built by oracle/Makefile), or None."""
    path = REF_REGION.get(workload.name)
    if not path or not os.path.exists(path):
        return None
    lib = C.CDLL(path)
    fn = lib.thiran_ref_entry
    fn.restype = C.c_int
    fn.argtypes = [C.POINTER(RefArg), C.c_uint64, C.c_void_p, C.c_uint64, C.c_char_p, C.c_uint64]
    return fn


def mlp_cpu_sample(lr, reps):
    """`reps` MLP training steps of the oracle (its f64-accumulated
    restatement: the reference trains only in its interpreter) at batch 256,
    512 -> 1024 -> 512 with biases, on one core; returns (TFLOP/s, sample)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib
    rng = np.random.default_rng(4)
    cb, ci, ch, co = 256, 512, 1024, 512
    xs = rng.standard_normal((cb, ci)).astype(np.float32)
    ts = rng.standard_normal((cb, co)).astype(np.float32)
    w1s = rng.uniform(-0.05, 0.05, (ci, ch)).astype(np.float32)
    w2s = rng.uniform(-0.05, 0.05, (ch, co)).astype(np.float32)
    b1s, b2s = np.zeros(ch, np.float32), np.zeros(co, np.float32)
    c0 = time.perf_counter()
    for _ in range(reps):
        oracle_lib.mlp_step_ex(xs, ts, w1s, w2s, lr, b1s, b2s)
    cpu_s = time.perf_counter() - c0
    flops = 2 * cb * (ci * ch + ch * co) + 2 * 2 * cb * ch * co + 2 * cb * ci * ch  # 2 forward + 3 backward GEMMs
    return (flops * reps / cpu_s / 1e12,
            f"{reps} MLP step(s) at batch {cb}, {ci}->{ch}->{co} (the oracle's f64-accumulated restatement; "
            f"the reference trains only in its interpreter), {cpu_s:.2f} s")


def cpu_inputs(workload, rows):
    rng = np.random.default_rng(1)
    if workload.name == "i64_region":
        a = rng.integers(-1000, 1001, (rows, workload.cols), dtype=np.int64)
        b = rng.integers(-1000, 1001, (rows, workload.cols), dtype=np.int64)
        return [a, b], np.empty_like(a)
    if workload.name == "f32_chain":
        x = rng.uniform(-1, 1, rows * 8192).astype(np.float32)
        return [x], np.empty_like(x)
    x = rng.standard_normal((rows, workload.cols)).astype(np.float32)
    return [x], np.empty_like(x)


def call_reference(fn, inputs, out):
    keep = []
    args = (RefArg * len(inputs))()
    for k, a in enumerate(inputs):
        shape = (C.c_uint64 * a.ndim)(*a.shape)
        keep.append(shape)
        args[k] = RefArg(2, 1 if a.dtype == np.int64 else 2, a.ndim, 0, shape, a.ctypes.data, a.size)
    fail = C.create_string_buffer(256)
    status = fn(args, len(inputs), out.ctypes.data, out.size, fail, 256)
    if status != 0:
        raise RuntimeError(f"reference CPU path failed: {status} {fail.value.decode()}")


def time_cpu(workload, threads, rows_per_thread, repeats):
    """Times the reference CPU path (or the oracle port) over `threads` host
    threads, each on its own `rows_per_thread` rows; returns (GB/s, kind, sample)."""
    fn = reference_entry(workload)
    kind = "reference"
    if fn is None:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import oracle_lib
        from thiran_b200 import regions
        spec = {"i64_region": regions.i64_region, "f32_chain": regions.f32_chain, "softmax": regions.softmax_rows,
                "sum": regions.full_sum}[workload.name]()
        kind = "port"

        def fn_port(inputs, out):
            if workload.name == "sum":  # the full sum of the flattened rows (a scalar result)
                oracle_lib.region_eval(spec, [inputs[0].reshape(-1)])
            else:
                out[...] = oracle_lib.region_eval(spec, inputs)
    work = [cpu_inputs(workload, rows_per_thread) for _ in range(threads)]
    elements = sum(o.size for _, o in work)

    def run(k):
        inputs, out = work[k]
        for _ in range(repeats):
            if kind == "reference":
                call_reference(fn, inputs, out)
            else:
                fn_port(inputs, out)

    start = time.perf_counter()
    pool = [threading.Thread(target=run, args=(k,)) for k in range(threads)]
    for t in pool:
        t.start()
    for t in pool:
        t.join()
    elapsed = time.perf_counter() - start
    gbs = elements * repeats * workload.bytes_per_element / elapsed / 1e9
    sample = (f"{threads} thread(s) x {rows_per_thread} rows x {repeats} call(s) "
              f"({elements * repeats} elements) of the same region, {elapsed:.2f} s")
    return gbs, kind, sample, elapsed


def _reference_worker(name, rows, calls, start, done):
    """One host process of the reference arm: its own inputs, `calls` calls."""
    workload = WORKLOADS[name]
    fn = reference_entry(workload)
    inputs, out = cpu_inputs(workload, rows)
    call_reference(fn, inputs, out)  # warm (page-in, allocator)
    for _ in range(calls):
        start.wait()
        call_reference(fn, inputs, out)
        done.wait()


def reference_arm(args, workload):
    """Times the reference's own CPU path (emitCpp20 output compiled like its
    JIT) on all host cores: one process per core (the reference's per-call
    path is single-threaded and serialises on process-global runtime state),
    each step every process runs the region once on its own sample rows."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import multiprocessing as mp
    procs_n = os.cpu_count() or 1
    rows = 16 if workload.name == "i64_region" else 8
    kind = "reference"
    unit = "GB/s"
    if workload.name == "mlp":
        # The reference trains only in its interpreter: each step is one
        # training step of the oracle's restatement on one core.
        values = []
        for step in range(args.warmup + args.steps):
            tflops, sample = mlp_cpu_sample(0.01, 1)
            if step >= args.warmup:
                values.append(tflops)
        kind, cores, unit = "port", 1, "TFLOP/s"
    elif reference_entry(workload) is None:
        # No native CPU region in the reference (its Evaluator interprets
        # these): the oracle port, 2048 rows per call.
        gbs, kind, sample, _ = time_cpu(workload, 1, 2048, args.steps)
        values = [gbs]
        cores = 1
    else:
        ctx = mp.get_context("spawn")
        calls = args.warmup + args.steps
        start, done = ctx.Barrier(procs_n + 1), ctx.Barrier(procs_n + 1)
        procs = [ctx.Process(target=_reference_worker, args=(workload.name, rows, calls, start, done))
                 for _ in range(procs_n)]
        for p in procs:
            p.start()
        values = []
        for step in range(calls):
            start.wait()
            t0 = time.perf_counter()
            done.wait()
            elapsed = time.perf_counter() - t0
            if step >= args.warmup:
                values.append(procs_n * rows * 8192 * workload.bytes_per_element / elapsed / 1e9)
        for p in procs:
            p.join()
        cores = procs_n
        sample = (f"{procs_n} process(es) x {rows} rows x 8192 of the workload per step, "
                  f"one reference region call each")
    value = statistics.median(values)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": workload.dtype, "data": "synthetic",
            "config": workload.config(1),
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": kind,
                             "sample": f"per step: {sample}"},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---- GPU arm -------------------------------------------------------------------------

def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="engine", choices=["engine", "reference"])
    p.add_argument("--workload", default="i64_region", choices=sorted(WORKLOADS))
    p.add_argument("--e2e-steps", type=int, default=None)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--dp-collective", default="fused", choices=["fused", "fused-peer", "fused-switch", "nccl"],
                   help="MLP data-parallel gradient reduction: fused into the dW GEMMs (peer loads/stores at "
                        "2 ranks, in-switch from 3; or forced), or NCCL all-reduce after the backward pass")
    p.add_argument("--dp-update", default="auto", choices=["auto", "fused", "pass"],
                   help="with a fused all-reduce: apply the optimizer step in the reduction (each tile's owner; "
                        "'auto' does so in switch mode, where it measured faster) or run the separate update pass "
                        "on every rank (faster in peer mode, 2 ranks)")
    p.add_argument("--dp-format", default="auto", choices=["auto", "bf16-sharded", "f32"],
                   help="with a fused all-reduce: bf16 gradient tiles and f32 weights sharded by tile owner (only "
                        "the bf16 weights are broadcast), or f32 gradients and replicated f32 weights; 'auto' "
                        "takes the bf16 form in switch mode (from 3 ranks)")
    p.add_argument("--shrink", type=int, default=1,
                   help="divide the leading extent (small cases for profiler captures; not a bench line)")
    args = p.parse_args()
    workload = WORKLOADS[args.workload]
    if args.shrink > 1:
        for attr in ("rows", "n", "batch"):
            if hasattr(workload, attr):
                setattr(workload, attr, getattr(workload, attr) // args.shrink)
    if args.impl == "reference":
        return reference_arm(args, workload)

    import torch
    import torch.distributed as dist
    import datetime
    import thiran_b200 as thb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    host_affinity = bind_host_to_gpu(torch, local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if workload.name == "mlp":
        rc = run_mlp(args, workload, torch, dist, thb, world, rank, local, barrier, max_over_ranks)
        if world > 1:
            dist.destroy_process_group()
        return rc

    spec, inputs, out = workload.build(torch, rank, world)
    region = spec.compile(local)
    stream = torch.cuda.Stream()
    s = stream.cuda_stream
    elements = max(t.numel() for t in inputs)
    bytes_per_step_rank = elements * workload.bytes_per_element
    combine = getattr(workload, "combine", False)
    total = torch.zeros(1, dtype=torch.float64, device="cuda")
    from thiran_b200.distributed import combine_partial_sums

    def step(start=None, end=None):
        if start is not None:
            start.record(stream)
        region.launch(inputs, out, s)
        if end is not None:
            end.record(stream)
        if combine:  # one f64 partial per rank, all-reduced over NCCL
            total.copy_(out)
            combine_partial_sums(total, dist if world > 1 else None)

    # Warm-up (also JIT/module load and slot allocation).
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    region.check_errors(s)
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        begin.record(stream)
        for k in range(args.steps):
            step(starts[k], ends[k])
        finish.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    region.check_errors(s)
    per_launch_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    total_ms = begin.elapsed_time(finish)
    total_ms = max_over_ranks(total_ms)
    ms_per_step = total_ms / args.steps
    value = bytes_per_step_rank * world * args.steps / (total_ms / 1e3) / 1e9

    # Roofline of the dominant (only) kernel.
    peak, peak_kind = measured_peaks()
    launch_ms = statistics.mean(per_launch_ms)
    achieved = bytes_per_step_rank / (launch_ms / 1e3) / 1e9
    traffic = ncu_traffic(workload.ncu_name) if world == 1 else None

    # End to end through the public host API, pinned host buffers.
    host_inputs = [t.cpu().pin_memory() for t in inputs]
    host_np = [t.numpy() for t in host_inputs]
    host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    host_out_np = host_out.numpy()
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 20))
    region_host = spec.compile(local)
    region_host.execute(host_np, out=host_out_np)  # warm
    barrier()
    step_s = []
    for _ in range(e2e_steps):
        t0 = time.perf_counter()
        partial = region_host.execute(host_np, out=host_out_np)
        if combine:
            combined = torch.tensor([float(partial)], dtype=torch.float64, device="cuda")
            combine_partial_sums(combined, dist if world > 1 else None)
            combined.item()
        step_s.append(time.perf_counter() - t0)
    # Each step's time is the slowest rank's; the value is taken at the
    # median step (the reference's qualification method, TH-023), the mean
    # is reported beside it.
    if world > 1:
        st = torch.tensor(step_s, dtype=torch.float64, device="cuda")
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
        step_s = st.cpu().tolist()
    e2e_value = bytes_per_step_rank * world / statistics.median(step_s) / 1e9
    e2e_mean = bytes_per_step_rank * world * len(step_s) / sum(step_s) / 1e9
    h2d = sum(t.numel() * t.element_size() for t in inputs)
    d2h = out.numel() * out.element_size()

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = {"i64_region": 1024, "f32_chain": 128}.get(workload.name, 2048)
        gbs, kind, sample, _ = time_cpu(workload, 1, rows, 2)
        cpu_baseline = {"value": gbs, "unit": "GB/s", "cores": 1, "kind": kind,
                        "sample": f"{sample}; the reference CPU path is single-threaded"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": workload.dtype, "data": "synthetic (torch.Generator on device, seeded)",
            "config": workload.config(world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": getattr(workload, "kernel", "generated fused elementwise group (NVRTC, sm_100a), "
                                                               "bulk-copy entry: cp.async.bulk tile ring + mbarriers"),
                         "algorithmic_bytes_per_launch": bytes_per_step_rank,
                         "avg_launch_ms": launch_ms, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"},
            "cpu_baseline": cpu_baseline,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps, "statistic": "median step (slowest rank)", "mean": e2e_mean,
                    "host_affinity": host_affinity,
                    "api": "thb_region_execute (host buffers, pinned)"},
            "gpu_launches": args.steps * getattr(workload, "launches_per_step", 1),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    del region, region_host
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
