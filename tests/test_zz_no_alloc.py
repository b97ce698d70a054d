"""The allocation-free full-tensor sum, for callers that cannot allocate
device memory (hosts that own all device memory and forbid cudaMalloc /
cudaFree from components), against the existing region Sum entry point.

Both go through the C ABI. The test allocates its own inputs and outputs with
torch (test plumbing); the entry point under test allocates nothing and keeps
its block partials in the library's static scratch. Two calls in a row must
each agree with the region path within the reductions' 1e-5 relative bound
(they share kernels and grid, so they are expected to agree exactly). This
file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def noalloc_sum(torch, x, stream):
    out32 = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
    out64 = torch.full((1,), float("nan"), dtype=torch.float64, device="cuda")
    fail = C.create_string_buffer(512)
    status = thb.lib().thb_sum_all_f32_noalloc(0, x.data_ptr(), x.numel(), out32.data_ptr(), out64.data_ptr(),
                                                C.c_void_p(stream), fail, len(fail))
    assert status == thb.STATUS_OK, fail.value.decode()
    torch.cuda.synchronize()
    return out32.item(), out64.item()


def region_sum(torch, region, x, stream):
    """The existing entry point: thb_region_execute on a full-sum region."""
    return float(region.execute([x.cpu().numpy()]))


def test_noalloc_sum_matches_region_sum_twice(device):
    torch = pytest.importorskip("torch")
    stream = torch.cuda.current_stream().cuda_stream
    region = regions.full_sum().compile(device)
    g = torch.Generator(device="cuda").manual_seed(3)
    first = torch.randn(1 << 24, device="cuda", generator=g)
    second = torch.rand((1 << 22) + 3, device="cuda", generator=g) * 4 - 1  # ragged, different values
    for x in (first, second):
        check_against_region(torch, region, x, stream)


def check_against_region(torch, region, x, stream):
    got32, got64 = noalloc_sum(torch, x, stream)
    want = region_sum(torch, region, x, stream)
    assert abs(got32 - want) <= RTOL * max(1.0, abs(want))
    assert abs(got64 - want) <= RTOL * max(1.0, abs(want))
    host = float(np.sum(x.cpu().numpy(), dtype=np.float64))
    assert abs(got64 - host) <= RTOL * max(1.0, abs(host))


def test_noalloc_sum_small_empty_and_unaligned(device):
    """The paths below the bulk-tile pass: a small input (pass 1 with 128-bit
    loads writing its partials into the static scratch), an empty input, and
    an input that starts 4 bytes past a 16-byte boundary (scalar loads)."""
    torch = pytest.importorskip("torch")
    stream = torch.cuda.current_stream().cuda_stream
    region = regions.full_sum().compile(device)
    g = torch.Generator(device="cuda").manual_seed(5)
    base = torch.randn((1 << 20) + 9, device="cuda", generator=g)
    small = base[:1000].clone()
    unaligned = base[1:]
    assert unaligned.data_ptr() % 16 == 4
    for x in (small, unaligned, small):
        check_against_region(torch, region, x, stream)
    empty = torch.empty(0, device="cuda")
    got32, got64 = noalloc_sum(torch, empty, stream)
    assert got32 == 0.0 and got64 == 0.0
