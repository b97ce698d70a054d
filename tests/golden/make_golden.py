"""Generates tests/golden/ fixtures by running the REFERENCE implementation.

Runs only where the reference sources are present: `make -C oracle ref` first
builds oracle/_ref/ref_driver from them. Each fixture records inputs and the
reference's output (its Evaluator, src/semantic/v0/Evaluator.cpp, and its
native CPU path, src/backend/v0/NativeCpu.cpp), plus the reference planner's
fusion groups. The CPU tests check the oracle against these files and the GPU
tests check the engine against them.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
DRIVER = os.path.join(ROOT, "oracle", "_ref", "ref_driver")


def write_thb(path, value):
    arr = np.asarray(value)
    dtype = 1 if arr.dtype == np.int64 else 2
    with open(path, "wb") as f:
        f.write(b"THB1" + struct.pack("<II", dtype, arr.ndim))
        for e in arr.shape:
            f.write(struct.pack("<Q", e))
        f.write(np.ascontiguousarray(arr).tobytes())


def read_thb(path):
    with open(path, "rb") as f:
        data = f.read()
    assert data[:4] == b"THB1"
    dtype, rank = struct.unpack("<II", data[4:12])
    shape = struct.unpack("<" + "Q" * rank, data[12:12 + 8 * rank])
    arr = np.frombuffer(data[12 + 8 * rank:], dtype=np.int64 if dtype == 1 else np.float32)
    return arr.reshape(shape) if rank else arr[0]


def evaluate(program: str, function: str, inputs):
    """Runs semantic::evaluateCall on the reference; returns (status, value)."""
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "p.th")
        with open(src, "w") as f:
            f.write(program)
        paths = []
        for k, v in enumerate(inputs):
            p = os.path.join(tmp, f"in{k}.bin")
            write_thb(p, v)
            paths.append(p)
        out = os.path.join(tmp, "out.bin")
        res = subprocess.run([DRIVER, "eval", src, function, out] + paths, capture_output=True, text=True, check=True)
        status = json.loads(res.stdout.strip().splitlines()[-1])
        if status["status"] != "ok":
            return status.get("error_id", "error"), None
        return "ok", read_thb(out)


def vjp(program: str, function: str, cotangent, inputs, gradients: int):
    """Runs the reference's reverse mode (autodiff::differentiate +
    executeVjpWithPrimal); returns (primal, [gradient per parameter])."""
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "p.th")
        with open(src, "w") as f:
            f.write(program)
        paths = []
        for k, v in enumerate(inputs):
            p = os.path.join(tmp, f"in{k}.bin")
            write_thb(p, v)
            paths.append(p)
        ct = os.path.join(tmp, "ct.bin")
        write_thb(ct, cotangent)
        prefix = os.path.join(tmp, "out_")
        res = subprocess.run([DRIVER, "vjp", src, function, prefix, ct] + paths, capture_output=True, text=True,
                             check=True)
        assert json.loads(res.stdout.strip().splitlines()[-1])["status"] == "ok", res.stdout
        return read_thb(prefix + "primal.bin"), [read_thb(prefix + f"grad{k}.bin") for k in range(gradients)]


def plan(program: str, function: str, fusion=True):
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "p.th")
        with open(src, "w") as f:
            f.write(program)
        args = [DRIVER, "plan", src, function] + ([] if fusion else ["nofusion"])
        return subprocess.run(args, capture_output=True, text=True, check=True).stdout


def groups_of(dump: str):
    out = []
    for line in dump.splitlines():
        line = line.strip()
        if line.startswith("group g"):
            nodes = line.split("nodes=")[1].split()[0]
            out.append([int(v[1:]) for v in nodes.split(",")])
    return out


class RefRegion:
    """The reference's native CPU region object (emitCpp20 + host compile)."""

    class Arg(C.Structure):
        _fields_ = [("kind", C.c_uint32), ("dtype", C.c_uint32), ("rank", C.c_uint32), ("reserved", C.c_uint32),
                    ("shape", C.POINTER(C.c_uint64)), ("data", C.c_void_p), ("count", C.c_uint64)]

    def __init__(self, path):
        self.lib = C.CDLL(path)
        self.fn = self.lib.thiran_ref_entry
        self.fn.restype = C.c_int
        self.fn.argtypes = [C.POINTER(self.Arg), C.c_uint64, C.c_void_p, C.c_uint64, C.c_char_p, C.c_uint64]

    def __call__(self, inputs, out_shape, out_dtype):
        args = (self.Arg * len(inputs))()
        keep = []
        for k, a in enumerate(inputs):
            shape = (C.c_uint64 * a.ndim)(*a.shape)
            keep.append(shape)
            args[k] = self.Arg(2, 1 if a.dtype == np.int64 else 2, a.ndim, 0, shape, a.ctypes.data, a.size)
        out = np.empty(out_shape, dtype=out_dtype)
        fail = C.create_string_buffer(256)
        status = self.fn(args, len(inputs), out.ctypes.data, out.size, fail, 256)
        return status, fail.value.decode(), out


F32_CHAIN_4 = """fn f(A:Tensor<f32,1>,B:Tensor<f32,1>) -> Tensor<f32,1> {
let C=A+B
let D=C.*B
let E=D-A
return E+B
}"""
I64_DYN = """fn f(x: Tensor<i64,1>, y: Tensor<i64,1>) -> Tensor<i64,1> {
let z=x+y
return z.*y
}"""
PICK = "fn pick(x: Tensor<i64,1>, i:i64)->i64{return x[i]}"
CHAIN = open(os.path.join(ROOT, "oracle", "programs", "f32_chain.th")).read()
CHAIN_LITERAL = "fn f(x: Tensor<f32,1>) -> Tensor<f32,1> {\nreturn ((x*1.5+0.25).*x - x)*0.5 + x\n}"
I64_REGION = open(os.path.join(ROOT, "oracle", "programs", "i64_region.th")).read()
SQUARE_LINEAR = "fn f(x: Tensor<f32,1>) -> Tensor<f32,1> {\nreturn research_square_linear(x)\n}"
SUMS_I64 = """fn rows(A: Tensor<i64,2>) -> Tensor<i64,1> { return sum(A, 1) }
fn cols(A: Tensor<i64,2>) -> Tensor<i64,1> { return sum(A, 0) }
fn total(A: Tensor<i64,1>) -> i64 { return sum(A, 0) }
"""
SUMS = """fn rows(A: Tensor<f32,2>) -> Tensor<f32,1> { return sum(A, 1) }
fn cols(A: Tensor<f32,2>) -> Tensor<f32,1> { return sum(A, 0) }
fn total(A: Tensor<f32,2>) -> f32 { return sum(sum(A, 1), 0) }
"""
MATMUL = "fn mm(A: Tensor<f32,2>, B: Tensor<f32,2>) -> Tensor<f32,2> { return A * B }"
MATMUL_I64 = "fn mm(A: Tensor<i64,2>, B: Tensor<i64,2>) -> Tensor<i64,2> { return A * B }"
LINEAR_LOSS = """fn loss(x: Tensor<f32,2>, w1: Tensor<f32,2>, w2: Tensor<f32,2>, t: Tensor<f32,2>) -> f32 {
let h = x * w1
let y = h * w2
let e = y - t
let s = e .* e
return sum(sum(s, 1), 0)
}"""

LINEAR_BIAS_LOSS = """fn loss(x: Tensor<f32,2>, w1: Tensor<f32,2>, b1: Tensor<f32,1>, w2: Tensor<f32,2>, b2: Tensor<f32,1>, t: Tensor<f32,2>) -> f32 {
let h = x * w1 + b1
let y = h * w2 + b2
let e = y - t
let s = e .* e
return sum(sum(s, 1), 0)
}"""


def main():
    if not os.path.exists(DRIVER):
        sys.exit(f"{DRIVER} missing: run `make -C oracle ref` (needs the reference sources)")
    fixtures = {}
    arrays = {}

    # Known-answer vectors of the reference's GPU integration test
    # (tests/backend/v0/NativeGpuIntegrationTests.cpp:72-112, :139-163, :165-189).
    a = np.array([1.0, 2.0, 0.0, 3.5, 7.0], np.float32)
    b = np.array([2.0, 4.0, 3.0, 0.5, 1.0], np.float32)
    status, value = evaluate(F32_CHAIN_4, "f", [a, b])
    arrays["kat_f32_a"], arrays["kat_f32_b"], arrays["kat_f32_out"] = a, b, value
    fixtures["kat_f32_chain"] = {"status": status, "groups_fused": groups_of(plan(F32_CHAIN_4, "f")),
                                 "groups_unfused": groups_of(plan(F32_CHAIN_4, "f", fusion=False))}

    x = np.full(257, 3, np.int64)
    status, value = evaluate(I64_DYN, "f", [x, x])
    arrays["kat_i64_257_out"] = value
    fixtures["kat_i64_257"] = {"status": status, "groups_fused": groups_of(plan(I64_DYN, "f"))}

    lefts, rights, outs = [], [], []
    for case in range(100):
        left = np.array([(case * 37 + e * 19) % 257 - 128 for e in range(17)], np.int64)
        right = np.array([(case * 29 + e * 31) % 129 - 64 for e in range(17)], np.int64)
        status, value = evaluate(I64_DYN, "f", [left, right])
        assert status == "ok"
        lefts.append(left); rights.append(right); outs.append(value)
    arrays["kat_i64_diff_left"] = np.stack(lefts)
    arrays["kat_i64_diff_right"] = np.stack(rights)
    arrays["kat_i64_diff_out"] = np.stack(outs)

    status, _ = evaluate(I64_DYN, "f", [np.array([2**63 - 1], np.int64), np.array([1], np.int64)])
    fixtures["kat_i64_overflow"] = {"status": status}
    for idx in (256, 257, -1):
        status, value = evaluate(PICK, "pick", [x, np.int64(idx)])
        fixtures[f"kat_pick_{idx}"] = {"status": status, "value": None if value is None else int(value)}

    xs = np.array([-2.0, -0.5, 0.0, 1.5, 3.0, 7.25, -9.0], np.float32)
    status, value = evaluate(SQUARE_LINEAR, "f", [xs])
    arrays["kat_square_linear_in"], arrays["kat_square_linear_out"] = xs, value

    # Benchmark-shaped regions at fixture sizes, through the reference
    # Evaluator AND its native CPU path (emitCpp20 + host compile).
    rng = np.random.default_rng(0)
    chain_x = rng.uniform(-1, 1, 1 << 14).astype(np.float32)
    status, value = evaluate(CHAIN, "f", [chain_x])
    arrays["chain_x"], arrays["chain_eval"] = chain_x, value
    ref = RefRegion(os.path.join(ROOT, "oracle", "_ref", "region_f32_chain.so"))
    s, _, out = ref([chain_x], chain_x.shape, np.float32)
    assert s == 0
    arrays["chain_native_cpu"] = out
    fixtures["chain"] = {"groups_fused": groups_of(plan(CHAIN, "f"))}
    status, value = evaluate(CHAIN_LITERAL, "f", [chain_x])
    assert status == "ok"
    arrays["chain_literal_eval"] = value

    rng = np.random.default_rng(1)
    ia = rng.integers(-1000, 1001, (64, 96), dtype=np.int64)
    ib = rng.integers(-1000, 1001, (64, 96), dtype=np.int64)
    status, value = evaluate(I64_REGION, "f", [ia, ib])
    arrays["i64_a"], arrays["i64_b"], arrays["i64_eval"] = ia, ib, value
    ref = RefRegion(os.path.join(ROOT, "oracle", "_ref", "region_i64_region.so"))
    s, _, out = ref([ia, ib], ia.shape, np.int64)
    assert s == 0
    arrays["i64_native_cpu"] = out
    big = np.array([[3037000500, 1]], np.int64)
    s, fail, _ = ref([big, np.zeros_like(big)], big.shape, np.int64)
    fixtures["i64_region"] = {"groups_fused": groups_of(plan(I64_REGION, "f")),
                              "groups_unfused": groups_of(plan(I64_REGION, "f", fusion=False)),
                              "overflow_status": s, "overflow_id": fail}

    # Reductions and matmul (Evaluator only; the reference has no native path).
    rng = np.random.default_rng(3)
    m = rng.standard_normal((64, 128)).astype(np.float32)
    arrays["sum_in"] = m
    for fn in ("rows", "cols", "total"):
        status, value = evaluate(SUMS, fn, [m])
        arrays[f"sum_{fn}"] = np.asarray(value, np.float32)
    # i64 sums (checked adds in order) and a prefix that overflows although
    # the total would fit.
    im = np.random.default_rng(9).integers(-(1 << 40), 1 << 40, (33, 70), dtype=np.int64)
    arrays["sum_i64_in"] = im
    for fn in ("rows", "cols"):
        status, value = evaluate(SUMS_I64, fn, [im])
        arrays[f"sum_i64_{fn}"] = np.asarray(value, np.int64)
    status, value = evaluate(SUMS_I64, "total", [im.reshape(-1)])
    arrays["sum_i64_total"] = np.asarray(value, np.int64)
    edge = np.array([np.iinfo(np.int64).max, 1, -1], np.int64)
    fixtures["sum_i64_prefix_overflow"] = evaluate(SUMS_I64, "total", [edge])[0]
    fixtures["sum_i64_rows_prefix_overflow"] = evaluate(SUMS_I64, "rows", [edge.reshape(1, 3)])[0]
    fixtures["sum_i64_cols_prefix_overflow"] = evaluate(SUMS_I64, "cols", [edge.reshape(3, 1)])[0]
    rng = np.random.default_rng(4)
    ma = rng.standard_normal((16, 32)).astype(np.float32)
    mb = rng.standard_normal((32, 24)).astype(np.float32)
    status, value = evaluate(MATMUL, "mm", [ma, mb])
    arrays["mm_a"], arrays["mm_b"], arrays["mm_out"] = ma, mb, value
    # Shapes whose K and N are not multiples of 8 (examples/transformer.th
    # multiplies [2,4] by [4,4], [4,2] and [2,8]), and the i64 rule with its
    # overflow failure.
    oa = rng.standard_normal((37, 13)).astype(np.float32)
    ob = rng.standard_normal((13, 5)).astype(np.float32)
    status, value = evaluate(MATMUL, "mm", [oa, ob])
    arrays["mm_odd_a"], arrays["mm_odd_b"], arrays["mm_odd_out"] = oa, ob, value
    ia = rng.integers(-1000, 1001, (33, 70), dtype=np.int64)
    ib = rng.integers(-1000, 1001, (70, 19), dtype=np.int64)
    status, value = evaluate(MATMUL_I64, "mm", [ia, ib])
    arrays["mm_i64_a"], arrays["mm_i64_b"], arrays["mm_i64_out"] = ia, ib, value
    half = np.array([[1 << 62, 1 << 62]], np.int64)  # products fit, their sum is 2^63
    status, _ = evaluate(MATMUL_I64, "mm", [half, np.array([[1], [1]], np.int64)])
    fixtures["mm_i64_sum_overflow"] = status
    root = np.array([[3037000500]], np.int64)  # 3037000500^2 > INT64_MAX
    status, _ = evaluate(MATMUL_I64, "mm", [root, root])
    fixtures["mm_i64_product_overflow"] = status

    # Reverse mode (src/autodiff/v0/Autodiff.cpp): extension gradient recipes
    # and the matmul / sum / broadcast rules of a linear two-layer loss.
    rng = np.random.default_rng(6)
    dz = rng.uniform(-2, 2, 7).astype(np.float32)
    _, (g,) = vjp(SQUARE_LINEAR, "f", dz, [xs], 1)
    arrays["ad_square_linear_dz"], arrays["ad_square_linear_grad"] = dz, g
    cx = rng.uniform(-1, 1, 4096).astype(np.float32)
    cdz = rng.uniform(-1, 1, 4096).astype(np.float32)
    _, (g,) = vjp(CHAIN, "f", cdz, [cx], 1)
    arrays["ad_chain_x"], arrays["ad_chain_dz"], arrays["ad_chain_grad"] = cx, cdz, g
    lx = rng.standard_normal((16, 32)).astype(np.float32)
    lw1 = (rng.standard_normal((32, 64)) * 0.2).astype(np.float32)
    lw2 = (rng.standard_normal((64, 32)) * 0.2).astype(np.float32)
    lt = rng.standard_normal((16, 32)).astype(np.float32)
    loss, (gx, gw1, gw2, gt) = vjp(LINEAR_LOSS, "loss", np.float32(1.0), [lx, lw1, lw2, lt], 4)
    arrays.update(ad_lin_x=lx, ad_lin_w1=lw1, ad_lin_w2=lw2, ad_lin_t=lt, ad_lin_loss=np.float32(loss),
                  ad_lin_dx=gx, ad_lin_dw1=gw1, ad_lin_dw2=gw2, ad_lin_dt=gt)
    # The same loss with broadcast biases (the examples/mlp.th structure).
    bx = rng.standard_normal((16, 32)).astype(np.float32)
    bw1 = (rng.standard_normal((32, 64)) * 0.2).astype(np.float32)
    bb1 = (rng.standard_normal(64) * 0.1).astype(np.float32)
    bw2 = (rng.standard_normal((64, 24)) * 0.2).astype(np.float32)
    bb2 = (rng.standard_normal(24) * 0.1).astype(np.float32)
    bt = rng.standard_normal((16, 24)).astype(np.float32)
    loss, grads = vjp(LINEAR_BIAS_LOSS, "loss", np.float32(1.0), [bx, bw1, bb1, bw2, bb2, bt], 6)
    arrays.update(ad_linb_x=bx, ad_linb_w1=bw1, ad_linb_b1=bb1, ad_linb_w2=bw2, ad_linb_b2=bb2, ad_linb_t=bt,
                  ad_linb_loss=np.float32(loss))
    for name, g in zip(("dx", "dw1", "db1", "dw2", "db2", "dt"), grads):
        arrays[f"ad_linb_{name}"] = g

    # The reference's own GPU artifacts (buildGpuAot, NativeArtifacts.cpp:1056-1097):
    # THIRAN16 container, serialized region, generated PTX payload.
    for program, stem in (("f32_chain", "ref_f32_chain"), ("i64_region", "ref_i64_region")):
        for suffix, extra in (("", []), ("_nofusion", ["nofusion"])):
            out = os.path.join(HERE, f"{stem}{suffix}.tha")
            subprocess.run([DRIVER, "tha", os.path.join(ROOT, "oracle", "programs", f"{program}.th"), "f", out] + extra,
                           check=True, capture_output=True)
            os.chmod(out, 0o644)

    # The reference's model bundle (createModelBundle + writeModelBundle,
    # src/model/v0/ModelBundle.cpp:328-360): public x, frozen parameters w, b
    # of fn f(x, w, b) = research_chain(x) .* w + b, one GPU artifact; and the
    # reference Evaluator's result on a second public input.
    rng = np.random.default_rng(13)
    mx = rng.uniform(-1, 1, (96, 200)).astype(np.float32)
    mw = rng.standard_normal((96, 200)).astype(np.float32)
    mb = rng.standard_normal((96, 200)).astype(np.float32)
    mx2 = rng.uniform(-1, 1, (96, 200)).astype(np.float32)
    model_program = os.path.join(ROOT, "oracle", "programs", "research_model.th")
    with tempfile.TemporaryDirectory() as tmp:
        paths = []
        for k, v in enumerate([mx, mw, mb]):
            p = os.path.join(tmp, f"m{k}.bin")
            write_thb(p, v)
            paths.append(p)
        out = os.path.join(HERE, "ref_research_model.thm")
        subprocess.run([DRIVER, "thm", model_program, "f", out, "1"] + paths, check=True, capture_output=True)
        os.chmod(out, 0o644)
    program = open(model_program).read()
    for name, x in (("model_x", mx), ("model_x2", mx2)):
        status, value = evaluate(program, "f", [x, mw, mb])
        assert status == "ok"
        arrays[name], arrays[name + "_eval"] = x, value

    # Software renderer scenes (graphics::render, src/graphics/v0/Graphics.cpp)
    # rendered by the reference: random triangles under a perspective camera
    # (clipping, overlap), equal-depth duplicates (first triangle wins), and
    # an orthographic view cutting the near and far planes.
    for name, scene in graphics_scenes().items():
        with tempfile.TemporaryDirectory() as tmp:
            paths = []
            for key in ("positions", "indices", "colors", "model", "view", "projection"):
                p = os.path.join(tmp, key + ".bin")
                write_thb(p, scene[key])
                paths.append(p)
            res = subprocess.run([DRIVER, "render"] + paths + [str(scene["width"]), str(scene["height"]),
                                                                os.path.join(tmp, "o_")],
                                 check=True, capture_output=True, text=True)
            status = json.loads(res.stdout.strip().splitlines()[-1])
            assert status["status"] == "ok", status
            for key, value in scene.items():
                arrays[f"gfx_{name}_{key}"] = np.asarray(value)
            arrays[f"gfx_{name}_color"] = read_thb(os.path.join(tmp, "o_color.bin"))
            arrays[f"gfx_{name}_depth"] = read_thb(os.path.join(tmp, "o_depth.bin"))
            arrays[f"gfx_{name}_stats"] = np.array(status["stats"], np.uint64)

    np.savez_compressed(os.path.join(HERE, "reference_outputs.npz"), **arrays)
    with open(os.path.join(HERE, "reference_fixtures.json"), "w") as f:
        json.dump(fixtures, f, indent=1, sort_keys=True)
    print("wrote", len(arrays), "arrays and", len(fixtures), "fixtures")


def graphics_scenes():
    """Scene inputs; matrices come from the oracle's restated helpers (the
    cube known answer pins them to the reference's)."""
    sys.path.insert(0, os.path.dirname(HERE))
    sys.path.insert(0, ROOT)
    import oracle_lib as orc
    g = orc.gfx
    scenes = {}
    rng = np.random.default_rng(17)
    n = 240
    scenes["random"] = dict(
        positions=rng.uniform(-1.6, 1.6, (n * 3, 3)).astype(np.float32),
        indices=np.arange(n * 3, dtype=np.int64).reshape(n, 3),
        colors=rng.uniform(0, 1, (n * 3, 4)).astype(np.float32),
        model=g.multiply(g.rotation_y(np.float32(0.3)), g.rotation_x(np.float32(-0.2))).reshape(4, 4),
        view=g.look_at([0.5, 1.0, 3.0], [0, 0, 0], [0, 1, 0]).reshape(4, 4),
        projection=g.perspective(np.float32(1.1), np.float32(160 / 120), np.float32(0.5), np.float32(20)).reshape(4, 4),
        width=160, height=120)
    tri = np.array([[-.8, -.6, .3], [.7, -.5, .3], [0, .8, .3]], np.float32)
    scenes["ties"] = dict(
        positions=np.concatenate([tri, tri, tri * 0.5]).astype(np.float32),
        indices=np.array([[0, 1, 2], [3, 4, 5], [6, 7, 8]], np.int64),
        colors=np.array([[1, 0, 0, 1]] * 3 + [[0, 1, 0, 1]] * 3 + [[0, 0, 1, 1]] * 3, np.float32),
        model=g.identity().reshape(4, 4), view=g.identity().reshape(4, 4), projection=g.identity().reshape(4, 4),
        width=64, height=48)
    m = 120
    scenes["ortho"] = dict(
        positions=rng.uniform(-1.3, 1.3, (m * 3, 3)).astype(np.float32),
        indices=rng.integers(0, m * 3, (m, 3), dtype=np.int64),
        colors=rng.uniform(0, 1, (m * 3, 4)).astype(np.float32),
        model=g.rotation_z(np.float32(0.4)).reshape(4, 4), view=g.identity().reshape(4, 4),
        projection=g.orthographic(-1.2, 1.2, -1, 1, 0, 1).reshape(4, 4),
        width=97, height=81)
    return scenes


if __name__ == "__main__":
    main()
