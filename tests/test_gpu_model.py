"""Model bundles on the GPU: the reference's bundle runs bit-exactly against
its Evaluator; the frozen parameters reach HBM once at compile time and
every call uploads only the public input."""
import os

import numpy as np
import pytest

import thiran_b200 as thb

pytestmark = pytest.mark.gpu
PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_research_model.thm")


def test_reference_model_matches_reference_evaluator(device, golden):
    session = thb.Model.load(PATH).compile(device)
    assert session.compile_evidence["host_to_device_bytes"] == 2 * 96 * 200 * 4
    for name in ("model_x", "model_x2", "model_x"):
        out = session.execute([golden[name]])
        assert out.view(np.uint32).tolist() == golden[name + "_eval"].view(np.uint32).tolist()
        # Only the public input crosses PCIe on each call.
        assert session.evidence["host_to_device_bytes"] == golden[name].nbytes
        assert session.evidence["kernel_launches"] == 1


def test_model_public_abi_checks(device, golden):
    session = thb.Model.load(PATH).compile(device)
    with pytest.raises(thb.GpuError) as err:
        session.execute([])
    assert err.value.code == "MODEL-PUBLIC-INPUT-COUNT"
    with pytest.raises(thb.GpuError) as err:
        session.execute([np.zeros((96, 199), np.float32)], output_shape=[96, 200])
    assert err.value.code == "MODEL-PUBLIC-INPUT-ABI"
    with pytest.raises(thb.GpuError) as err:
        session.execute([np.zeros((96, 200), np.int64)])
    assert err.value.code == "MODEL-PUBLIC-INPUT-ABI"
