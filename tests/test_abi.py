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


def test_plain_c_caller(tmp_path):
    """The header is C99 and the library links into a plain C program, as a
    reference-side shim would use it: the program describes a region (plan
    counts without a device) and probes the device."""
    import shutil
    import subprocess
    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    src = tmp_path / "caller.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "thiran_b200.h"
int main(void) {
    /* out = (a + b) * a - b over [4] i64 (the i64 region) */
    uint32_t d3[2] = {1, 2}, d4[2] = {3, 1}, d5[2] = {4, 2};
    thb_region_node n[5];
    memset(n, 0, sizeof n);
    for (int k = 0; k < 5; ++k) { n[k].id = k + 1; n[k].dtype = THB_DTYPE_I64; n[k].rank = 1; n[k].extent[0] = 4; }
    n[0].op = THB_OP_INPUT; n[1].op = THB_OP_INPUT;
    n[2].op = THB_OP_ADD; n[2].dependencies = d3; n[2].dependency_count = 2;
    n[3].op = THB_OP_ELEMENT_MULTIPLY; n[3].dependencies = d4; n[3].dependency_count = 2;
    n[4].op = THB_OP_SUBTRACT; n[4].dependencies = d5; n[4].dependency_count = 2;
    uint32_t inputs[2] = {1, 2};
    thb_region_desc desc = {1, "c_caller", n, 5, inputs, 2, 5};
    thb_plan_options options = {1, 1};
    uint64_t needed = 0, counts[3] = {0, 0, 0};
    char failure[256] = {0};
    int s = thb_region_describe(&desc, options, THB_DESCRIBE_PLAN, NULL, 0, &needed, counts, failure, sizeof failure);
    thb_device_info info;
    int p = thb_probe(0, &info);
    printf("%d %llu %llu %llu %u %d %d\n", s, (unsigned long long)counts[0], (unsigned long long)counts[1],
           (unsigned long long)counts[2], thb_abi_version(), info.backend_built, p);
    return 0;
}
''')
    exe = tmp_path / "caller"
    lib_dir = os.path.dirname(thb.LIBRARY_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                    "-L", lib_dir, "-lthiran_b200", f"-Wl,-rpath,{lib_dir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120, check=True).stdout.split()
    status, groups, fused, kernels, version, built, probe = (int(v) for v in out)
    assert (status, groups, fused, kernels, version, built) == (thb.STATUS_OK, 1, 1, 1, 1, 1)
    if not os.path.exists("/dev/nvidia0"):
        assert probe == thb.STATUS_BACKEND
