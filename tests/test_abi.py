"""The C-ABI library loads, exports every declared symbol, and refuses to run
without a device (no CPU fallback)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for header in os.listdir(os.path.join(ROOT, "include")):
        if header.endswith(".h"):
            text = open(os.path.join(ROOT, "include", header)).read()
            names |= set(re.findall(r"\b(thb_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(thb.LIBRARY_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    assert len(declared_symbols()) >= 15


def test_binding_covers_every_declared_symbol():
    assert set(declared_symbols()) <= set(thb.SIGNATURES)


def test_abi_version_and_layout():
    assert thb.lib().thb_abi_version() == 1
    assert thb.lib().thb_backend_built() == 1
    # Layouts shared with the reference (ScalarNodeV0, ThiranAbiArg,
    # OperationDescriptorV0 on x86-64).
    assert C.sizeof(thb.ScalarNode) == 20
    assert C.sizeof(thb.AbiArg) == 40
    assert C.sizeof(thb.OperationDesc) == 80
    assert C.sizeof(thb.Evidence) == 33 * 8


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="checks the no-device path")
def test_no_device_no_fallback():
    info = thb.probe(0)
    assert info.backend_built == 1 and info.device_available == 0
    assert info.error_code.decode() == "GPU-DRIVER-NOT-FOUND"
    with pytest.raises(thb.GpuError) as err:
        regions.f32_chain().compile()
    assert err.value.code == "GPU-DRIVER-NOT-FOUND" and err.value.status == thb.STATUS_BACKEND


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(thb, "_lib", None)
    monkeypatch.setattr(thb, "LIBRARY_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(ImportError):
        thb.lib()
