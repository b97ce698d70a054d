"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on CPU."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) device")
    # Build the engine and the oracle checker when absent (no-op when current).
    for directory in ("thiran_b200", "oracle"):
        target = os.path.join(ROOT, directory, "libthiran_b200.so" if directory == "thiran_b200" else "liboracle.so")
        if not os.path.exists(target):
            subprocess.run(["make", "-C", os.path.join(ROOT, directory), "-j8"], check=True,
                           stdout=subprocess.DEVNULL)


@pytest.fixture(scope="session")
def golden():
    data = np.load(os.path.join(TESTS, "golden", "reference_outputs.npz"))
    return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def fixtures():
    with open(os.path.join(TESTS, "golden", "reference_fixtures.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def oracle():
    import oracle_lib
    return oracle_lib


@pytest.fixture(scope="session")
def device():
    """The B200 under test; GPU tests fail (not skip) when it is absent."""
    import thiran_b200 as thb
    info = thb.probe(0)
    assert info.device_available, f"no CUDA device: {info.error_code.decode()} {info.name.decode()}"
    assert info.compute_major == 10, f"expected sm_100 (B200), got {info.compute_major}.{info.compute_minor}"
    return 0
