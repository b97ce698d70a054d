"""GPU parity of the reduction regions (row softmax, row max, sums).

Tolerance (north-star contract for reductions): 1e-5 relative per element
against the f64-accumulated CPU restatement.
"""
import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions
import oracle_lib as orc

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def rel_err(actual, expected):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    return float(np.max(np.abs(actual - expected) / np.maximum(np.abs(expected), 1e-30)))


@pytest.mark.parametrize("rows,cols", [(1, 4), (17, 4096), (257, 1024), (64, 8192), (33, 4100), (5, 12000),
                                       (3, 4097), (1000, 64)])
def test_softmax_shapes(device, rows, cols):
    x = np.random.default_rng(rows * 7 + cols).standard_normal((rows, cols)).astype(np.float32)
    out = regions.softmax_rows().compile(device).execute([x])
    assert rel_err(out, orc.softmax_rows(x)) <= RTOL


def test_softmax_65536x4096(device):
    """Config: [65536,4096] f32 ~ N(0,1) (seed 3)."""
    x = np.random.default_rng(3).standard_normal((65536, 4096)).astype(np.float32)
    out = regions.softmax_rows().compile(device).execute([x])
    assert rel_err(out, orc.softmax_rows(x)) <= RTOL
    np.testing.assert_allclose(out.sum(axis=1, dtype=np.float64), 1.0, rtol=1e-5)


def test_softmax_extreme_values(device):
    x = np.array([[1e30, -1e30, 0.0, 5.0], [-50.0, -50.0, -50.0, -50.0], [88.0, 88.0, -88.0, 0.0]], np.float32)
    out = regions.softmax_rows().compile(device).execute([x])
    assert rel_err(out[out > 0], orc.softmax_rows(x)[out > 0]) <= RTOL
    np.testing.assert_array_equal(out == 0, orc.softmax_rows(x) == 0)


@pytest.mark.parametrize("rows,cols", [(1, 1), (17, 4096), (300, 333), (64, 8192),
                                       # warp-per-row kernel: partial last packet column, short rows
                                       (257, 1028), (1000, 64), (5, 2048)])
def test_row_max_and_sum(device, rows, cols):
    x = np.random.default_rng(cols).standard_normal((rows, cols)).astype(np.float32)
    b = thb.RegionBuilder("rm")
    v = b.input(thb.F32, [None, None])
    mx = b.build(b.row_max(v)).compile(device).execute([x])
    np.testing.assert_array_equal(mx, orc.max_rows(x))
    b = thb.RegionBuilder("rs")
    v = b.input(thb.F32, [None, None])
    rs = b.build(b.sum(v, 1)).compile(device).execute([x])
    assert rel_err(rs, orc.sum_rows(x)) <= RTOL or np.max(np.abs(rs - orc.sum_rows(x))) <= 1e-5
    b = thb.RegionBuilder("cs")
    v = b.input(thb.F32, [None, None])
    cs = b.build(b.sum(v, 0)).compile(device).execute([x])
    assert np.max(np.abs(cs - orc.sum_cols(x))) <= RTOL * max(1.0, float(np.max(np.abs(orc.sum_cols(x)))))


@pytest.mark.parametrize("n", [1, 5, 1023, 1 << 20, (1 << 20) + 3])
def test_full_sum_sizes(device, n):
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    total = regions.full_sum().compile(device).execute([x])
    ref = orc.sum_all_f64(x)
    assert abs(total - ref) <= RTOL * max(1.0, abs(ref))


def test_full_sum_65536x4096(device):
    """Config: full-tensor sum of the [65536,4096] N(0,1) (seed 3) tensor."""
    x = np.random.default_rng(3).standard_normal((65536, 4096)).astype(np.float32).reshape(-1)
    total = regions.full_sum().compile(device).execute([x])
    ref = orc.sum_all_f64(x)
    assert abs(total - ref) <= RTOL * max(1.0, abs(ref))


def test_softmax_then_sum_region(device):
    """softmax -> row sums in one region: two kernels, rows sum to 1."""
    b = thb.RegionBuilder("sm")
    v = b.input(thb.F32, [None, None])
    spec = b.build(b.sum(b.softmax(v), 1))
    x = np.random.default_rng(5).standard_normal((128, 4096)).astype(np.float32)
    region = spec.compile(device)
    out = region.execute([x])
    np.testing.assert_allclose(out, 1.0, rtol=1e-5)
    assert region.evidence["kernel_launches"] == 2


def _sum_i64_region(kind):
    b = thb.RegionBuilder("s")
    if kind == "total":
        x = b.input(thb.I64, [None])
        return b.build(b.sum(x, 0))
    x = b.input(thb.I64, [None, None])
    return b.build(b.sum(x, 1 if kind == "rows" else 0))


def test_sum_i64_matches_reference(device, golden):
    m = golden["sum_i64_in"]
    for kind in ("rows", "cols"):
        out = _sum_i64_region(kind).compile(device).execute([m])
        np.testing.assert_array_equal(out, golden[f"sum_i64_{kind}"])
    assert _sum_i64_region("total").compile(device).execute([m.reshape(-1).copy()]) == int(golden["sum_i64_total"])


@pytest.mark.parametrize("shape", [(1, 1), (7, 3), (300, 4099), (4097, 33), (1 << 22,), (1000003,), (5,)])
def test_sum_i64_random_exact(device, shape):
    """Large magnitudes (|v| < 2^50, totals far beyond f64's 53 bits): the
    result is exact; where a partial sum in the reference order overflows,
    the same failure id."""
    rng = np.random.default_rng(sum(shape))
    x = rng.integers(-(1 << 50), 1 << 50, shape, dtype=np.int64)
    kinds = ("total",) if len(shape) == 1 else ("rows", "cols")
    for kind in kinds:
        spec = _sum_i64_region(kind)
        try:
            want = orc.region_eval(spec, [x])
        except orc.OracleFailure as failure:
            with pytest.raises(thb.GpuError) as err:
                spec.compile(device).execute([x])
            assert err.value.code == failure.code
            continue
        got = spec.compile(device).execute([x])
        np.testing.assert_array_equal(got, want)


def test_sum_i64_prefix_overflow(device, fixtures):
    """The reference fails when any partial sum in its order leaves the i64
    range, even if the total would fit ([MAX, 1, -1]); a reordered sum must
    not hide that, and a sum whose partials stay in range must not fail
    ([-1, MAX, 1] overflows only at the end in the reference order too, so
    it fails; [1, -1, MAX] fits)."""
    mx = np.iinfo(np.int64).max
    for kind, shape in (("total", (3,)), ("rows", (1, 3)), ("cols", (3, 1))):
        region = _sum_i64_region(kind).compile(device)
        with pytest.raises(thb.GpuError) as err:
            region.execute([np.array([mx, 1, -1], np.int64).reshape(shape)])
        assert err.value.code == "TH-SPEC-I64-OVERFLOW"
        out = region.execute([np.array([1, -1, mx], np.int64).reshape(shape)])
        assert int(np.asarray(out).reshape(-1)[0]) == mx
    # A long vector whose prefix crosses the edge in the middle of a block.
    x = np.ones(1 << 20, np.int64)
    x[5000] = mx - 4000
    x[5001] = -(1 << 40)
    with pytest.raises(thb.GpuError) as err:
        _sum_i64_region("total").compile(device).execute([x])
    assert err.value.code == fixtures["sum_i64_prefix_overflow"]


def test_sum_i64_empty(device):
    """Sums over empty extents are 0 (the reference's accumulator starts at
    0): zero columns, zero rows, an empty vector."""
    rows = _sum_i64_region("rows").compile(device)
    np.testing.assert_array_equal(rows.execute([np.zeros((3, 0), np.int64)]), np.zeros(3, np.int64))
    cols = _sum_i64_region("cols").compile(device)
    np.testing.assert_array_equal(cols.execute([np.zeros((0, 4), np.int64)]), np.zeros(4, np.int64))
    assert _sum_i64_region("total").compile(device).execute([np.zeros(0, np.int64)]) == 0
