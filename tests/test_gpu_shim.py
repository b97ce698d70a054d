"""V0 programs through the reference-side binding on the GPU: source ->
reference front end (parse, analyse, verify) -> thiran_b200/shim lowering ->
thb_region_compile / execute, against the reference Evaluator
(src/semantic/v0/Evaluator.cpp) run by ref_driver on the same inputs, and the
reference's own reverse mode (autodiff::differentiate + executeVjpWithPrimal)
against the generated forward and backward functions run on the engine.

Bars: exact-mode matmuls, elementwise chains and i64 bit-exact; results that
pass through a Sum are f64-accumulated on the GPU against the Evaluator's
sequential f32, 1e-5 relative (|ref| + rms); tensor-core matmuls 2e-2.
"""
import os

import numpy as np
import pytest

from shim_programs import DRIVER, I64_REGION, LOSS, PROGRAM, REF_DRIVER, read_thb, run

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def drivers():
    if not (os.path.exists(DRIVER) and os.path.exists(REF_DRIVER)):
        # Both link the reference's library, built only where its sources are.
        pytest.skip("shim_driver / ref_driver are not built (make -C oracle ref; make -C thiran_b200/shim)")


def block_error(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    return float(np.max(np.abs(got - ref) / (np.abs(ref) + rms + 1e-30)))


def gpu_and_reference(tmp_path, program, function, inputs, mode="exact"):
    status, out = run(["run", function, "0", mode, "0", str(tmp_path / "gpu.bin")], str(tmp_path), program, inputs)
    assert status and status["status"] == "ok", out
    ref_status, out = run(["ref", function, str(tmp_path / "ref.bin")], str(tmp_path), program, inputs)
    assert ref_status and ref_status["status"] == "ok", out
    return read_thb(str(tmp_path / "gpu.bin")), read_thb(str(tmp_path / "ref.bin"))


def test_sum_of_matmul(drivers, tmp_path):
    rng = np.random.default_rng(1)
    a = rng.standard_normal((37, 29)).astype(np.float32)
    b = rng.standard_normal((29, 45)).astype(np.float32)
    c = rng.standard_normal((37, 45)).astype(np.float32)
    got, ref = gpu_and_reference(tmp_path, PROGRAM, "rowsum", [a, b, c])
    assert got.shape == ref.shape == (37,)
    assert block_error(got, ref) <= 1e-5
    got, _ = gpu_and_reference(tmp_path, PROGRAM, "rowsum", [a, b, c], mode="tensor")
    assert block_error(got, ref) <= 2e-2


def test_i64_matmul(drivers, tmp_path):
    rng = np.random.default_rng(2)
    a = rng.integers(-1000, 1001, (21, 64), dtype=np.int64)
    b = rng.integers(-1000, 1001, (64, 13), dtype=np.int64)
    got, ref = gpu_and_reference(tmp_path, PROGRAM, "imm", [a, b])
    np.testing.assert_array_equal(got, ref)
    big = np.array([[1 << 62, 1 << 62]], np.int64)
    status, out = run(["run", "imm", "0", "exact", "0", str(tmp_path / "o.bin")], str(tmp_path), PROGRAM,
                      [big, np.ones((2, 1), np.int64)])
    assert status == {"status": "error", "code": "TH-SPEC-I64-OVERFLOW", "category": "SemanticFailure"}, out


def test_i64_column_sum_of_matmul(drivers, tmp_path):
    rng = np.random.default_rng(8)
    a = rng.integers(-(1 << 20), 1 << 20, (40, 17), dtype=np.int64)
    b = rng.integers(-(1 << 20), 1 << 20, (17, 9), dtype=np.int64)
    got, ref = gpu_and_reference(tmp_path, PROGRAM, "isum", [a, b])
    np.testing.assert_array_equal(got, ref)


def test_matmul_with_broadcast_bias_bitwise(drivers, tmp_path):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((16, 12)).astype(np.float32)
    w = rng.standard_normal((12, 7)).astype(np.float32)
    b = rng.standard_normal(7).astype(np.float32)
    got, ref = gpu_and_reference(tmp_path, PROGRAM, "affine", [x, w, b])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_full_sum_and_extension_with_scalar(drivers, tmp_path):
    rng = np.random.default_rng(4)
    a = rng.standard_normal((64, 300)).astype(np.float32)
    got, ref = gpu_and_reference(tmp_path, PROGRAM, "total", [a])
    assert abs(float(got) - float(ref)) <= 1e-5 * float(np.sum(np.abs(a)))
    x = rng.uniform(-1, 1, 1000).astype(np.float32)
    got, ref = gpu_and_reference(tmp_path, PROGRAM, "scaled", [x])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_reference_region_through_execute_native_gpu(drivers, tmp_path):
    """The reference's own extracted region (extractStrictGpu) through the
    binding's executeNativeGpu."""
    rng = np.random.default_rng(5)
    a = rng.integers(-1000, 1001, (33, 70), dtype=np.int64)
    b = rng.integers(-1000, 1001, (33, 70), dtype=np.int64)
    status, out = run(["native", "f", "0", str(tmp_path / "gpu.bin")], str(tmp_path), I64_REGION, [a, b])
    assert status and status["status"] == "ok", out
    np.testing.assert_array_equal(read_thb(str(tmp_path / "gpu.bin")), (a + b) * a - b)
    big = np.array([[3037000500]], np.int64)
    status, _ = run(["native", "f", "0", str(tmp_path / "o.bin")], str(tmp_path), I64_REGION, [big, np.zeros_like(big)])
    assert status["code"] == "TH-SPEC-I64-OVERFLOW" and status["category"] == "SemanticFailure"


@pytest.mark.parametrize("mode,bar", [("exact", 1e-5), ("tensor", 2e-2)])
def test_generated_reverse_mode_on_the_engine(drivers, tmp_path, mode, bar):
    """loss(x, w1, w2, t) = sum((x w1 w2 - t)^2): the generated forward (primal
    and 14 saved values) and backward (4 gradients) run on the engine."""
    rng = np.random.default_rng(6)
    x = rng.standard_normal((24, 16)).astype(np.float32)
    w1 = (rng.standard_normal((16, 32)) * 0.3).astype(np.float32)
    w2 = (rng.standard_normal((32, 8)) * 0.3).astype(np.float32)
    t = rng.standard_normal((24, 8)).astype(np.float32)
    from shim_programs import write_thb
    write_thb(str(tmp_path / "ct.bin"), np.float32(1.0))
    status, out = run(["vjp", "loss", mode, "0", str(tmp_path / "o_"), str(tmp_path / "ct.bin")], str(tmp_path), LOSS,
                      [x, w1, w2, t])
    assert status and status["status"] == "ok" and status["gradients"] == 4, out
    primal, ref_primal = read_thb(str(tmp_path / "o_primal.bin")), read_thb(str(tmp_path / "o_ref_primal.bin"))
    assert abs(float(primal) - float(ref_primal)) <= bar * abs(float(ref_primal))
    for k in range(4):
        got = read_thb(str(tmp_path / f"o_grad{k}.bin"))
        ref = read_thb(str(tmp_path / f"o_ref_grad{k}.bin"))
        assert got.shape == ref.shape
        assert block_error(got, ref) <= bar, k


def test_extension_gradient_recipe_on_the_engine(drivers, tmp_path):
    rng = np.random.default_rng(7)
    x = rng.uniform(-1, 1, 4097).astype(np.float32)
    from shim_programs import write_thb
    write_thb(str(tmp_path / "ct.bin"), np.float32(0.75))
    status, out = run(["vjp", "chain_loss", "exact", "0", str(tmp_path / "o_"), str(tmp_path / "ct.bin")],
                      str(tmp_path), LOSS, [x])
    assert status and status["status"] == "ok", out
    got, ref = read_thb(str(tmp_path / "o_grad0.bin")), read_thb(str(tmp_path / "o_ref_grad0.bin"))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("stem", ["ref_f32_chain", "ref_f32_chain_nofusion", "ref_i64_region",
                                  "ref_i64_region_nofusion"])
def test_reference_artifacts_through_load_and_execute(drivers, tmp_path, stem):
    """The reference's own GPU artifacts (buildGpuAot) through the binding's
    loadAndExecuteArtifact: the reference loader validates them, the region
    runs on the engine, bit-exact against the oracle."""
    import oracle_lib
    from shim_programs import write_thb
    from thiran_b200 import regions
    import subprocess
    rng = np.random.default_rng(9)
    if "f32" in stem:
        inputs = [rng.uniform(-1, 1, 4099).astype(np.float32)]
        spec = regions.f32_chain()
    else:
        inputs = [rng.integers(-1000, 1001, (37, 129), dtype=np.int64) for _ in range(2)]
        spec = regions.i64_region()
    paths = []
    for k, v in enumerate(inputs):
        write_thb(str(tmp_path / f"in{k}.bin"), v)
        paths.append(str(tmp_path / f"in{k}.bin"))
    golden = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", f"{stem}.tha")
    res = subprocess.run([DRIVER, "artifact", golden, "0", str(tmp_path / "o.bin")] + paths, capture_output=True,
                         text=True)
    assert '"status":"ok"' in res.stdout, res.stdout
    got = read_thb(str(tmp_path / "o.bin"))
    want = oracle_lib.region_eval(spec, inputs)
    assert got.dtype == want.dtype and np.array_equal(got.view(np.uint8), want.view(np.uint8))
