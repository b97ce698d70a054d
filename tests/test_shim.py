"""The reference-side binding (thiran_b200/shim) on the CPU: it compiles and
links against the reference's own headers and library, lowers V0 functions
that use Matmul, Sum, a broadcast bias and autodiff's generated forward and
backward functions into regions the engine's verifier and planner accept, and
without a device its execution path fails with GPU-DRIVER-NOT-FOUND (the
reference's BackendUnavailable category) instead of falling back."""
import os
import subprocess

import pytest

from shim_programs import DRIVER, LOSS, PROGRAM, ROOT, I64_REGION, run

REFERENCE = os.environ.get("THIRAN_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")


@pytest.fixture(scope="module")
def driver():
    if os.path.isdir(os.path.join(REFERENCE, "include")) and \
            os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libthiran_ref.a")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "thiran_b200", "shim"), f"REF={REFERENCE}"], check=True,
                       stdout=subprocess.DEVNULL)
    if not os.path.exists(DRIVER):
        pytest.skip("the reference sources are absent (the binding compiles against its headers)")
    return DRIVER


def lowered(tmp_path, program, function, element=0, mode="exact"):
    _, out = run(["lower", function, str(element), mode], str(tmp_path), program)
    nodes = [dict(kv.split("=", 1) for kv in line.split()[2:]) for line in out.splitlines() if line.startswith("node ")]
    return out, nodes


@pytest.mark.parametrize("function,ops", [
    ("rowsum", {"38", "32", "9"}),        # MatMul, Sum, ElementMultiply
    ("imm", {"38"}),
    ("affine", {"38", "39", "7"}),        # MatMul, BroadcastToShape (the rank-1 bias), Add
    ("total", {"32"}),
    ("scaled", {"10", "9"}),              # Extension, scalar Multiply as ElementMultiply
    ("isum", {"38", "32"}),               # i64 MatMul and Sum
])
def test_lowering_admits_what_the_reference_extractor_defers(driver, tmp_path, function, ops):
    out, nodes = lowered(tmp_path, PROGRAM, function)
    assert "plan groups=" in out, out
    assert ops <= {n["op"] for n in nodes}, out


def test_matmul_mode(driver, tmp_path):
    _, exact = lowered(tmp_path, PROGRAM, "rowsum", 0, "exact")
    _, tensor = lowered(tmp_path, PROGRAM, "rowsum", 0, "tensor")
    assert [n["axis"] for n in exact if n["op"] == "38"] == ["1"]
    assert [n["axis"] for n in tensor if n["op"] == "38"] == ["0"]


@pytest.mark.parametrize("element", [0, 1, 2, 3])
def test_generated_backward_functions_lower(driver, tmp_path, element):
    out, nodes = lowered(tmp_path, LOSS, "loss@backward", element)
    assert "plan groups=" in out, out
    ops = {n["op"] for n in nodes}
    assert {"39", "40"} <= ops or {"40"} <= ops, out     # BroadcastToShape / ReduceToShape
    if element < 3:
        assert {"37", "38"} <= ops, out                 # Transpose, MatMul


def test_generated_forward_tuple_elements_lower(driver, tmp_path):
    for element in range(15):
        out, _ = lowered(tmp_path, LOSS, "loss@forward", element)
        assert "plan groups=" in out, (element, out)


def test_no_device_fails_without_fallback(driver, tmp_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    import numpy as np
    a = np.ones((4, 3), np.float32)
    status, _ = run(["run", "rowsum", "0", "exact", "0", str(tmp_path / "o.bin")], str(tmp_path), PROGRAM,
                    [a, a.T.copy(), np.ones((4, 4), np.float32)])
    assert status == {"status": "error", "code": "GPU-DRIVER-NOT-FOUND", "category": "BackendUnavailable"}
    x = np.ones((2, 3), np.int64)
    status, _ = run(["native", "f", "0", str(tmp_path / "o.bin")], str(tmp_path), I64_REGION, [x, x])
    assert status["code"] == "GPU-DRIVER-NOT-FOUND"


def test_unsupported_forms_are_diagnosed(driver, tmp_path):
    program = "fn f(x: Tensor<f32,2>) -> Tensor<f32,2> { return x[0:2, :] }"
    out, _ = lowered(tmp_path, program, "f")
    assert out.startswith("BACKEND-UNSUPPORTED"), out


def test_artifact_path_validates_then_needs_a_device(driver, tmp_path):
    """`thiran run --backend gpu file.tha`: the reference's loader checks the
    container, the region then needs the engine's device."""
    torch = pytest.importorskip("torch")
    import numpy as np
    from shim_programs import write_thb
    x = np.ones(64, np.float32)
    write_thb(str(tmp_path / "x.bin"), x)
    golden = os.path.join(ROOT, "tests", "golden", "ref_f32_chain.tha")
    res = subprocess.run([DRIVER, "artifact", golden, "0", str(tmp_path / "o.bin"), str(tmp_path / "x.bin")],
                         capture_output=True, text=True)
    if not torch.cuda.is_available():
        assert '"code":"GPU-DRIVER-NOT-FOUND"' in res.stdout, res.stdout
    # A corrupted payload is the loader's failure, before any device work.
    data = bytearray(open(golden, "rb").read())
    data[-5] ^= 0xFF
    bad = tmp_path / "bad.tha"
    bad.write_bytes(bytes(data))
    res = subprocess.run([DRIVER, "artifact", str(bad), "0", str(tmp_path / "o.bin"), str(tmp_path / "x.bin")],
                         capture_output=True, text=True)
    assert '"status":"error"' in res.stdout and "ARTIFACT-" in res.stdout, res.stdout
