"""V0 programs and helpers shared by the shim tests (tests/test_shim.py on the
CPU, tests/test_gpu_shim.py on the GPU): sources that use the operations the
reference's native extractor rejects (src/backend/v0/TensorRegion.cpp:424-431)
and run them through thiran_b200/shim/_build/shim_driver."""
import json
import os
import struct
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVER = os.path.join(ROOT, "thiran_b200", "shim", "_build", "shim_driver")
REF_DRIVER = os.path.join(ROOT, "oracle", "_ref", "ref_driver")

# sum(A, 1) of a matmul; an i64 matmul; a matmul plus a broadcast bias.
PROGRAM = """fn rowsum(A: Tensor<f32,2>, B: Tensor<f32,2>, C: Tensor<f32,2>) -> Tensor<f32,1> {
let P = A * B
return sum(P .* C, 1)
}
fn imm(A: Tensor<i64,2>, B: Tensor<i64,2>) -> Tensor<i64,2> { return A * B }
fn affine(x: Tensor<f32,2>, w: Tensor<f32,2>, b: Tensor<f32,1>) -> Tensor<f32,2> { return x * w + b }
fn total(A: Tensor<f32,2>) -> f32 { return sum(sum(A, 1), 0) }
fn scaled(x: Tensor<f32,1>) -> Tensor<f32,1> { return research_chain(x) * 2.0 }
fn isum(A: Tensor<i64,2>, B: Tensor<i64,2>) -> Tensor<i64,1> { return sum(A * B, 0) }
"""

# A two-layer loss (matmul, sum, elementwise) and an extension loss; their
# reverse mode adds Transpose, BroadcastToShape, ReduceToShape and the
# extension's gradient recipe.
LOSS = """fn loss(x: Tensor<f32,2>, w1: Tensor<f32,2>, w2: Tensor<f32,2>, t: Tensor<f32,2>) -> f32 {
let h = x * w1
let y = h * w2
let e = y - t
let s = e .* e
return sum(sum(s, 1), 0)
}
fn chain_loss(x: Tensor<f32,1>) -> f32 { return sum(research_chain(x), 0) }
"""

# The strict subset the reference extracts itself (extractStrictGpu).
I64_REGION = "fn f(a: Tensor<i64,2>, b: Tensor<i64,2>) -> Tensor<i64,2> { let s = a + b; let m = s .* a; return m - b }"


def write_thb(path, value):
    value = np.asarray(value)
    dtype = 1 if value.dtype == np.int64 else 2
    with open(path, "wb") as f:
        f.write(b"THB1" + struct.pack("<II", dtype, value.ndim))
        f.write(struct.pack("<" + "Q" * value.ndim, *value.shape))
        f.write(np.ascontiguousarray(value, np.int64 if dtype == 1 else np.float32).tobytes())


def read_thb(path):
    with open(path, "rb") as f:
        data = f.read()
    assert data[:4] == b"THB1"
    dtype, rank = struct.unpack("<II", data[4:12])
    shape = struct.unpack("<" + "Q" * rank, data[12:12 + 8 * rank])
    arr = np.frombuffer(data[12 + 8 * rank:], dtype=np.int64 if dtype == 1 else np.float32)
    return arr.reshape(shape) if rank else arr[0]


def run(args, tmp, program, inputs=()):
    """Runs shim_driver (or ref_driver when args[0] == 'ref') with the program
    and inputs written under `tmp`; returns (JSON status line, stdout)."""
    src = os.path.join(tmp, "program.th")
    with open(src, "w") as f:
        f.write(program)
    paths = []
    for k, v in enumerate(inputs):
        p = os.path.join(tmp, f"in{k}.bin")
        write_thb(p, v)
        paths.append(p)
    binary = REF_DRIVER if args[0] == "ref" else DRIVER
    mode = "eval" if args[0] == "ref" else args[0]
    res = subprocess.run([binary, mode, src] + list(args[1:]) + paths, capture_output=True, text=True, timeout=600)
    lines = [line for line in res.stdout.splitlines() if line.startswith("{")]
    return (json.loads(lines[-1]) if lines else None), res.stdout
