"""The benchmark's reference arm runs on host cores only: its JSON line keeps
the contract (one line, the engine arm's metric and unit, a cpu_baseline and
an e2e record without transfers)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload,unit", [("i64_region", "GB/s"), ("f32_chain", "GB/s"), ("softmax", "GB/s"),
                                           ("sum", "GB/s"), ("mlp", "TFLOP/s")])
def test_reference_arm_line(workload, unit):
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                          "--workload", workload], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[-1])
    assert line["impl"] == "reference" and line["unit"] == unit and line["value"] > 0
    assert line["higher_is_better"] is True and line["n_gpus"] == 1 and line["steps"] == 1
    assert line["cpu_baseline"]["unit"] == unit and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    assert line["e2e"] == {"value": line["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]


def test_reference_arm_under_torchrun_prints_once():
    """Launched like the engine arm at N = 2, rank 0 alone runs and prints;
    the other rank exits 0 without work."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                          "--gpus", "2", "--steps", "1", "--warmup", "0"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2


def test_nvlink_byte_model():
    """The bytes per step the MLP line states for each gradient exchange: the
    compact switch form moves 2 B per weight element each way, a fifth of the
    f32 form with the update at 8 ranks; NCCL's ring 2(w-1)/w x 4 B."""
    sys.path.insert(0, ROOT)
    import bench

    class Fused:
        def __init__(self, mode, update, compact):
            self.mode, self.update, self.compact = mode, update, compact

    e = 2 * 4096 * 16384
    assert bench.nvlink_bytes_per_step(1, e, None) is None
    compact = bench.nvlink_bytes_per_step(8, e, Fused("switch", True, True))
    assert compact["in"] == compact["out"] == 2 * e
    f32 = bench.nvlink_bytes_per_step(8, e, Fused("switch", True, False))
    assert f32["in"] == int((4 / 8 + 6 * 7 / 8) * e) and f32["out"] == int((4 * 7 / 8 + 6 / 8) * e)
    nccl = bench.nvlink_bytes_per_step(8, e, None)
    assert nccl["in"] == int(2 * 7 / 8 * 4 * e)
    peer = bench.nvlink_bytes_per_step(2, e, Fused("peer", True, True))
    assert peer["in"] == 2 * e
