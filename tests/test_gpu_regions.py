"""GPU parity of the elementwise TensorRegion path, through the C ABI.

Mirrors tests/backend/v0/NativeGpuIntegrationTests.cpp of the reference:
known-answer chains, fused vs unfused evidence, the 100-case i64
differential, overflow / bounds / divide-by-zero failures, async submission,
zero-size and layout rejection; then the benchmark regions at full size
against the oracle (bit-exact).
"""
import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions
import oracle_lib as orc

pytestmark = pytest.mark.gpu


def test_kat_f32_chain_fused_evidence(device, golden):
    region = regions.f32_chain4().compile(device)
    out = region.execute([golden["kat_f32_a"], golden["kat_f32_b"]])
    assert np.max(np.abs(out - golden["kat_f32_out"])) <= 1e-6
    assert out.view(np.uint32).tolist() == golden["kat_f32_out"].view(np.uint32).tolist()
    ev = region.evidence
    assert ev["kernel_launches"] == 1 and ev["fusion_groups"] == 1 and ev["fused_kernel_groups"] == 1
    assert ev["logical_intermediates"] == 3 and ev["materialized_intermediates"] == 0
    assert ev["planner_owned_allocations"] == 1 and ev["retained_planner_allocations"] == 0
    assert ev["host_to_device_copies"] == 2 and ev["device_to_host_copies"] == 1
    assert ev["synchronizations"] == 1


def test_kat_f32_chain_unfused_evidence(device, golden):
    region = regions.f32_chain4().compile(device, fusion=False)
    out = region.execute([golden["kat_f32_a"], golden["kat_f32_b"]])
    assert out.view(np.uint32).tolist() == golden["kat_f32_out"].view(np.uint32).tolist()
    ev = region.evidence
    assert ev["kernel_launches"] == 4 and ev["fusion_groups"] == 4
    assert ev["planner_owned_allocations"] == 3 and ev["physical_temporary_slots"] == 2
    assert ev["reused_slot_assignments"] == 1


def test_kat_i64_odd_size_single_upload(device, golden):
    region = regions.i64_dynamic().compile(device)
    x = np.full(257, 3, np.int64)
    out = region.execute([x, x])
    np.testing.assert_array_equal(out, golden["kat_i64_257_out"])
    assert region.evidence["input_storage_uploads"] == 1
    assert x[0] == 3  # inputs are never mutated


@pytest.mark.parametrize("fusion", [True, False])
def test_kat_i64_differential(device, golden, fusion):
    region = regions.i64_dynamic().compile(device, fusion=fusion)
    for case in range(100):
        out = region.execute([golden["kat_i64_diff_left"][case], golden["kat_i64_diff_right"][case]])
        np.testing.assert_array_equal(out, golden["kat_i64_diff_out"][case])


def test_overflow_reported(device, fixtures):
    region = regions.i64_dynamic().compile(device)
    with pytest.raises(thb.GpuError) as err:
        region.execute([np.array([2**63 - 1], np.int64), np.array([1], np.int64)])
    assert err.value.code == fixtures["kat_i64_overflow"]["status"] and err.value.status == thb.STATUS_SEMANTIC
    # The region stays usable after a checked failure.
    out = region.execute([np.full(4, 2, np.int64), np.full(4, 3, np.int64)])
    np.testing.assert_array_equal(out, np.full(4, 15, np.int64))


@pytest.mark.parametrize("a,b", [(-(2**63), -1), (2**62, 2), (-(2**63), 1)])
def test_overflow_edges_match_oracle(device, a, b):
    spec = regions.i64_region()
    region = spec.compile(device)
    x = np.array([[a]], np.int64)
    y = np.array([[b]], np.int64)
    try:
        expected = orc.region_eval(spec, [x, y])
    except orc.OracleFailure as failure:
        with pytest.raises(thb.GpuError) as err:
            region.execute([x, y])
        assert err.value.code == failure.code
    else:
        np.testing.assert_array_equal(region.execute([x, y]), expected)


def test_dropped_failure_is_delivered(device):
    region = regions.i64_dynamic().compile(device)
    thb.take_unobserved_errors()
    pending = region.submit([np.array([2**63 - 1], np.int64), np.array([1], np.int64)])
    pending.release()
    assert thb.take_unobserved_errors() == ["TH-SPEC-I64-OVERFLOW"]


def test_divide_by_zero(device):
    op = thb.Operation("ratio", [(thb.SCALAR_INPUT, 0, 0, 0, 0.0), (thb.SCALAR_INPUT, 0, 0, 1, 0.0),
                                 (thb.SCALAR_DIVIDE, 0, 1, 0, 0.0)], root=2, arity=2,
                       effect=thb.EFFECT_MAY_TRAP, fusible=False)
    b = thb.RegionBuilder("d")
    x = b.input(thb.F32, [None])
    y = b.input(thb.F32, [None])
    spec = b.build(b.extension(op, x, y))
    region = spec.compile(device)
    num = np.array([1.0, 3.0, -2.0, 7.0], np.float32)
    den = np.array([4.0, 3.0, 0.5, 3.0], np.float32)
    np.testing.assert_array_equal(region.execute([num, den]), orc.region_eval(spec, [num, den]))
    den[2] = 0.0
    with pytest.raises(thb.GpuError) as err:
        region.execute([num, den])
    assert err.value.code == "TH021-DIVIDE-BY-ZERO"


@pytest.mark.parametrize("index,expect", [(256, 3), (257, "TH-SPEC-BOUNDS"), (-1, "TH-SPEC-BOUNDS")])
def test_index_bounds(device, index, expect):
    b = thb.RegionBuilder("pick")
    x = b.input(thb.I64, [None])
    i = b.input(thb.I64, [])
    region = b.build(b.index(b.alias(x), b.alias(i))).compile(device)
    data = np.full(257, 3, np.int64)
    if isinstance(expect, int):
        assert region.execute([data, index]) == expect
    else:
        with pytest.raises(thb.GpuError) as err:
            region.execute([data, index])
        assert err.value.code == expect
        assert region.evidence["kernel_launches"] == 0


def test_copy_and_alias(device):
    b = thb.RegionBuilder("copied")
    x = b.input(thb.I64, [None])
    y = b.input(thb.I64, [None])
    z = b.copy(b.alias(x))
    region = b.build(b.add(b.alias(z), b.alias(y))).compile(device)
    out = region.execute([np.full(257, 3, np.int64), np.full(257, 4, np.int64)])
    assert out[0] == 7 and region.evidence["device_to_device_copies"] == 1
    b = thb.RegionBuilder("identity")
    x = b.input(thb.I64, [None])
    region = b.build(b.alias(x)).compile(device)
    host = np.arange(257, dtype=np.int64)
    np.testing.assert_array_equal(region.execute([host]), host)


def test_tensor_literal_region(device):
    b = thb.RegionBuilder("lit")
    x = b.input(thb.I64, [2, 2])
    elems = [b.integer(v) for v in (5, 6, 7, 8)]
    lit = b.literal(thb.I64, [2, 2], elems)
    spec = b.build(b.add(b.alias(x), lit))
    region = spec.compile(device)
    out = region.execute([np.array([[1, 2], [3, 4]], np.int64)])
    np.testing.assert_array_equal(out, [[6, 8], [10, 12]])  # NativeCpuTests.cpp:79


def test_zero_size(device):
    region = regions.i64_dynamic().compile(device)
    empty = np.zeros(0, np.int64)
    out = region.execute([empty, empty])
    assert out.size == 0 and region.evidence["kernel_launches"] == 0


def test_layout_rejected(device):
    b = thb.RegionBuilder("f")
    x = b.input(thb.I64, [None, None])
    y = b.input(thb.I64, [None, None])
    region = b.build(b.add(x, y)).compile(device)
    m = np.array([[1, 2], [3, 4]], np.int64).T
    with pytest.raises(thb.GpuError) as err:
        region.execute([m, m])
    assert err.value.code == "GPU-UNSUPPORTED-LAYOUT" and region.evidence["kernel_launches"] == 0


def test_arity_and_type_rejected(device):
    region = regions.i64_dynamic().compile(device)
    with pytest.raises(thb.GpuError) as err:
        region.execute([np.zeros(3, np.int64)])
    assert err.value.code == "GPU-INPUT-ARITY"
    with pytest.raises(thb.GpuError) as err:
        region.execute([np.zeros(3, np.float32), np.zeros(3, np.float32)])
    assert err.value.code == "GPU-INPUT-TYPE"


def test_invalid_device(device):
    count = thb.probe(0).device_count
    with pytest.raises(thb.GpuError) as err:
        regions.f32_chain4().compile(count)
    assert err.value.code == "GPU-INVALID-DEVICE"


def test_async_submit_observe_and_stress(device):
    region = regions.i64_dynamic().compile(device)
    x = np.full(257, 3, np.int64)
    p = region.submit([x, x])
    assert p.submit_evidence["pending_operations"] == 1 and p.submit_evidence["active_write_reservations"] == 1
    np.testing.assert_array_equal(p.observe(), np.full(257, 18, np.int64))
    assert p.evidence["observations"] == 1 and p.evidence["active_read_reservations"] == 0
    np.testing.assert_array_equal(p.observe(), np.full(257, 18, np.int64))  # observe twice
    for _ in range(150):
        q = region.submit([x, x])
        np.testing.assert_array_equal(q.observe(), np.full(257, 18, np.int64))
        q.release()
    a = region.submit([x, x])
    other = x.copy()
    b = region.submit([other, other])
    np.testing.assert_array_equal(b.observe(), np.full(257, 18, np.int64))
    np.testing.assert_array_equal(a.observe(), np.full(257, 18, np.int64))


def test_chain_2p20_bit_exact(device):
    """Config: 2^20 f32, uniform[-1,1] (seed 0), chain as one extension recipe."""
    x = np.random.default_rng(0).uniform(-1, 1, 1 << 20).astype(np.float32)
    spec = regions.f32_chain()
    out = spec.compile(device).execute([x])
    expected = orc.region_eval(spec, [x])
    assert np.array_equal(out.view(np.uint32), expected.view(np.uint32))


@pytest.mark.parametrize("n", [1, 3, 17, 257, 4097, (1 << 16) + 5])
def test_chain_odd_sizes(device, n):
    x = np.random.default_rng(n).uniform(-4, 4, n).astype(np.float32)
    spec = regions.f32_chain4()
    y = np.random.default_rng(n + 1).uniform(-4, 4, n).astype(np.float32)
    out = spec.compile(device).execute([x, y])
    assert np.array_equal(out.view(np.uint32), orc.region_eval(spec, [x, y]).view(np.uint32))


def test_i64_region_8192_exact(device):
    """Config: (a+b)*a-b on [8192,8192] i64, uniform ints in [-1000,1000] (seed 1)."""
    rng = np.random.default_rng(1)
    a = rng.integers(-1000, 1001, (8192, 8192), dtype=np.int64)
    b = rng.integers(-1000, 1001, (8192, 8192), dtype=np.int64)
    spec = regions.i64_region()
    out = spec.compile(device).execute([a, b])
    np.testing.assert_array_equal(out, orc.region_eval(spec, [a, b]))


def pinned(torch, array):
    t = torch.from_numpy(array).pin_memory()
    return t, t.numpy()


def test_pipelined_host_execution(device):
    """Large row-local regions over pinned host buffers run chunk by chunk on
    three streams; results and checked failures are unchanged."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(21)
    spec = regions.i64_region()
    region = spec.compile(device)
    _, a = pinned(torch, rng.integers(-1000, 1001, (2048, 8192), dtype=np.int64))
    _, b = pinned(torch, rng.integers(-1000, 1001, (2048, 8192), dtype=np.int64))
    _, out = pinned(torch, np.empty((2048, 8192), np.int64))
    region.execute([a, b], out=out)
    assert region.evidence["host_to_device_copies"] > 2  # chunked
    np.testing.assert_array_equal(out, orc.region_eval(spec, [a, b]))
    a[-1, -1], b[-1, -1] = 2**62, 2**62  # overflow in the last chunk only
    with pytest.raises(thb.GpuError) as err:
        region.execute([a, b], out=out)
    assert err.value.code == "TH-SPEC-I64-OVERFLOW"
    # Pageable buffers take the unchunked path with the same result.
    a[-1, -1], b[-1, -1] = 1, 1
    np.testing.assert_array_equal(region.execute([a.copy(), b.copy()]), orc.region_eval(spec, [a, b]))


def test_pipelined_softmax_rows(device):
    torch = pytest.importorskip("torch")
    _, x = pinned(torch, np.random.default_rng(22).standard_normal((8192, 4096)).astype(np.float32))
    _, out = pinned(torch, np.empty((8192, 4096), np.float32))
    region = regions.softmax_rows().compile(device)
    region.execute([x], out=out)
    assert region.evidence["host_to_device_copies"] > 1
    ref = orc.softmax_rows(x)
    assert float(np.max(np.abs(out - ref) / ref)) <= 1e-5


def test_device_launch_path(device):
    torch = pytest.importorskip("torch")
    spec = regions.i64_region()
    region = spec.compile(device)
    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.randint(-1000, 1001, (512, 1000), dtype=torch.int64, device="cuda", generator=g)
    b = torch.randint(-1000, 1001, (512, 1000), dtype=torch.int64, device="cuda", generator=g)
    out = torch.empty_like(a)
    region.launch([a, b], out, torch.cuda.current_stream().cuda_stream)
    region.check_errors(torch.cuda.current_stream().cuda_stream)
    np.testing.assert_array_equal(out.cpu().numpy(), orc.region_eval(spec, [a.cpu().numpy(), b.cpu().numpy()]))
    # Unaligned (offset) operands take the scalar kernel.
    a1, b1, o1 = a.view(-1)[1:], b.view(-1)[1:], torch.empty(a.numel() - 1, dtype=torch.int64, device="cuda")
    spec1 = regions.i64_dynamic()
    r1 = spec1.compile(device)
    r1.launch([a1, b1], o1, torch.cuda.current_stream().cuda_stream)
    r1.check_errors(torch.cuda.current_stream().cuda_stream)
    np.testing.assert_array_equal(o1.cpu().numpy(), orc.region_eval(spec1, [a1.cpu().numpy(), b1.cpu().numpy()]))


def test_device_launch_latches_errors(device):
    torch = pytest.importorskip("torch")
    region = regions.i64_dynamic().compile(device)
    a = torch.tensor([2**62, 1], dtype=torch.int64, device="cuda")
    out = torch.empty_like(a)
    s = torch.cuda.current_stream().cuda_stream
    region.launch([a, a], out, s)
    with pytest.raises(thb.GpuError) as err:
        region.check_errors(s)
    assert err.value.code == "TH-SPEC-I64-OVERFLOW"
    region.check_errors(s)  # cleared after being read
