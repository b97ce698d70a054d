"""The generated CUDA source of every region kind compiles for sm_100a
(NVRTC, no device needed): the vector, scalar and bulk-copy entries of each
fusion group, with tensor inputs, literals, runtime scalar parameters,
extension recipes and their gradients, and multi-group backward regions."""
import pytest

import thiran_b200 as thb
from thiran_b200 import regions
from test_scalar_operands import scalar_input_region


def two_scalar_region():
    b = thb.RegionBuilder("two_scalars")
    x = b.input(thb.F32, [None])
    s = b.input(thb.F32, [])
    u = b.input(thb.F32, [])
    y = b.input(thb.F32, [None])
    return b.build(b.add(b.mul(b.add(b.mul(s, x), u), y), x))


CASES = {
    "f32_chain": regions.f32_chain,
    "f32_chain_literal": regions.f32_chain_literal,
    "f32_chain4": regions.f32_chain4,
    "i64_region": regions.i64_region,
    "i64_dynamic": regions.i64_dynamic,
    "scalar_input": scalar_input_region,
    "two_scalars": two_scalar_region,
    "extension_gradient": lambda: regions.extension_gradient(regions.chain_operation()),
    "linear_loss_backward": regions.linear_loss_backward,
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_generated_source_compiles(name):
    spec = CASES[name]()
    src, _ = spec.describe(thb.DESCRIBE_SOURCE)
    # Every elementwise group carries the bulk-copy entry next to the
    # vector and scalar ones.
    assert src.count("_vec(") == src.count("_scalar(") == src.count("_bulk(")
    assert int(spec.describe(thb.DESCRIBE_CUBIN)[0]) > 0
