"""`.tha` artifacts on the GPU: the reference's own GPU artifacts run on this
engine bit-exactly against the reference's CPU path on the same inputs
(its buildGpuAot output, tests/golden/ref_*.tha); this engine's artifacts
load without an NVRTC run and give the same bits as compiling the region."""
import os

import numpy as np
import pytest

import oracle_lib as orc
import thiran_b200 as thb
from thiran_b200 import regions

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("suffix", ["", "_nofusion"])
def test_reference_chain_artifact_matches_reference_cpu(device, golden, suffix):
    region = thb.Artifact.load(os.path.join(GOLDEN, f"ref_f32_chain{suffix}.tha")).compile(device)
    out = region.execute([golden["chain_x"]])
    assert out.view(np.uint32).tolist() == golden["chain_native_cpu"].view(np.uint32).tolist()


@pytest.mark.parametrize("suffix", ["", "_nofusion"])
def test_reference_i64_artifact_matches_reference_cpu(device, golden, suffix):
    region = thb.Artifact.load(os.path.join(GOLDEN, f"ref_i64_region{suffix}.tha")).compile(device)
    out = region.execute([golden["i64_a"], golden["i64_b"]])
    assert np.array_equal(out, golden["i64_native_cpu"])
    assert region.evidence["kernel_launches"] == (1 if suffix == "" else 3)


def test_reference_i64_artifact_reports_overflow(device):
    """The checked i64 arithmetic of the artifact's region: (a+b)*a-b on
    a = 3037000500 overflows (NativeGpuIntegrationTests.cpp:277-283)."""
    region = thb.Artifact.load(os.path.join(GOLDEN, "ref_i64_region.tha")).compile(device)
    a = np.array([[3037000500, 1]], np.int64)
    with pytest.raises(thb.GpuError) as err:
        region.execute([a, np.zeros_like(a)])
    assert err.value.status == thb.STATUS_SEMANTIC and err.value.code == "TH-SPEC-I64-OVERFLOW"


def test_reference_artifact_at_scale(device):
    """2^22 + 5 elements through the reference's chain artifact: equal to
    the oracle (pinned bit-exact to the reference's CPU path)."""
    rng = np.random.default_rng(41)
    x = rng.uniform(-1, 1, (1 << 22) + 5).astype(np.float32)
    region = thb.Artifact.load(os.path.join(GOLDEN, "ref_f32_chain.tha")).compile(device)
    out = region.execute([x])
    assert np.array_equal(out.view(np.uint32), orc.region_eval(regions.f32_chain(), [x]).view(np.uint32))


@pytest.mark.parametrize("builder,inputs", [
    (regions.f32_chain, lambda r: [r.uniform(-1, 1, 100003).astype(np.float32)]),
    (regions.i64_region, lambda r: [r.integers(-1000, 1001, (257, 129), dtype=np.int64) for _ in range(2)]),
    (regions.softmax_rows, lambda r: [r.standard_normal((300, 1000)).astype(np.float32)]),
])
def test_engine_artifact_runs_without_nvrtc(device, builder, inputs):
    spec = builder()
    artifact = thb.Artifact.load(thb.build_artifact(spec))
    region = artifact.compile(device)
    args = inputs(np.random.default_rng(43))
    out = region.execute(args)
    assert region.evidence["driver_jit_loads"] == 0
    direct = spec.compile(device).execute(args)
    assert np.array_equal(np.asarray(out).view(np.uint8), np.asarray(direct).view(np.uint8))
