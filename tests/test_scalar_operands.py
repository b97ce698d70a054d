"""Scalar operands inside elementwise chains (tensor (x) literal, tensor (x)
scalar input). The reference evaluates these only in its Evaluator, which
broadcasts the scalar (src/semantic/v0/Evaluator.cpp:95-124); its native
extractor rejects them. The oracle is pinned to the Evaluator on the chain's
literal source; the engine fuses the whole chain into one kernel."""
import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions
import oracle_lib as orc


def test_literal_chain_oracle_matches_reference_evaluator(golden):
    out = orc.region_eval(regions.f32_chain_literal(), [golden["chain_x"]])
    assert out.view(np.uint32).tolist() == golden["chain_literal_eval"].view(np.uint32).tolist()


def test_literal_chain_is_one_fused_group():
    text, counts = regions.f32_chain_literal().describe(thb.DESCRIBE_PLAN)
    assert counts == [1, 1, 1]
    src, _ = regions.f32_chain_literal().describe(thb.DESCRIBE_SOURCE)
    assert "__int_as_float(0x3fc00000)" in src and "__int_as_float(0x3e800000)" in src
    assert int(regions.f32_chain_literal().describe(thb.DESCRIBE_CUBIN)[0]) > 0


def scalar_input_region():
    b = thb.RegionBuilder("axpy")
    x = b.input(thb.F32, [None])
    s = b.input(thb.F32, [])
    y = b.input(thb.F32, [None])
    return b.build(b.add(b.mul(s, x), y))


def test_scalar_input_becomes_kernel_parameter():
    spec = scalar_input_region()
    text, counts = spec.describe(thb.DESCRIBE_PLAN)
    assert counts == [1, 1, 1]
    src, _ = spec.describe(thb.DESCRIBE_SOURCE)
    assert "float s0" in src
    x = np.arange(10, dtype=np.float32)
    y = np.ones(10, np.float32)
    np.testing.assert_array_equal(orc.region_eval(spec, [x, 2.5, y]), 2.5 * x + 1)


@pytest.mark.gpu
def test_literal_chain_gpu_bit_exact(device, golden):
    spec = regions.f32_chain_literal()
    region = spec.compile(device)
    out = region.execute([golden["chain_x"]])
    assert out.view(np.uint32).tolist() == golden["chain_literal_eval"].view(np.uint32).tolist()
    assert region.evidence["kernel_launches"] == 1
    x = np.random.default_rng(2).uniform(-1, 1, (1 << 22) + 1).astype(np.float32)
    assert np.array_equal(region.execute([x]).view(np.uint32), orc.region_eval(spec, [x]).view(np.uint32))


@pytest.mark.gpu
def test_scalar_input_gpu(device):
    spec = scalar_input_region()
    region = spec.compile(device)
    rng = np.random.default_rng(3)
    x = rng.standard_normal(100003).astype(np.float32)
    y = rng.standard_normal(100003).astype(np.float32)
    for s in (2.5, -0.125, 0.0):
        assert np.array_equal(region.execute([x, s, y]).view(np.uint32),
                              orc.region_eval(spec, [x, s, y]).view(np.uint32))


@pytest.mark.gpu
def test_integer_literal_overflow_checked(device):
    b = thb.RegionBuilder("i")
    a = b.input(thb.I64, [None])
    spec = b.build(b.mul(b.add(a, b.integer(3)), a))
    region = spec.compile(device)
    data = np.arange(-50, 50, dtype=np.int64)
    np.testing.assert_array_equal(region.execute([data]), orc.region_eval(spec, [data]))
    with pytest.raises(thb.GpuError) as err:
        region.execute([np.array([2**62], np.int64)])
    assert err.value.code == "TH-SPEC-I64-OVERFLOW"
