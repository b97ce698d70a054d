"""GPU parity of the reverse-AD region operations against the reference's own
reverse mode (golden fixtures from its autodiff::executeVjpWithPrimal) and
the oracle.

Extension gradients are elementwise f32 recipes: bit-exact. Transpose,
broadcast and zero-like move data: exact. ReduceToShape accumulates in f64:
1e-5 relative. MatMul runs bf16 x bf16 -> f32 on the tensor cores: relative
Frobenius error <= 2e-2 against the reference's f32 result.
"""
import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions
import oracle_lib as orc

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def test_extension_gradients_bit_exact(device, golden):
    spec = regions.extension_gradient(regions.square_linear_operation())
    out = spec.compile(device).execute([golden["kat_square_linear_in"], golden["ad_square_linear_dz"]])
    assert out.view(np.uint32).tolist() == golden["ad_square_linear_grad"].view(np.uint32).tolist()
    spec = regions.extension_gradient(regions.chain_operation())
    region = spec.compile(device)
    out = region.execute([golden["ad_chain_x"], golden["ad_chain_dz"]])
    assert out.view(np.uint32).tolist() == golden["ad_chain_grad"].view(np.uint32).tolist()
    # forward + gradient fuse into one kernel
    assert region.evidence["kernel_launches"] == 1
    rng = np.random.default_rng(31)
    x = rng.uniform(-1, 1, (1 << 20) + 7).astype(np.float32)
    dz = rng.uniform(-1, 1, x.size).astype(np.float32)
    out = region.execute([x, dz])
    assert np.array_equal(out.view(np.uint32), orc.region_eval(spec, [x, dz]).view(np.uint32))


@pytest.mark.parametrize("name", ["dx", "dw1", "dw2", "dt"])
def test_linear_loss_backward_region(device, golden, name):
    args = [golden["ad_lin_x"], golden["ad_lin_w1"], golden["ad_lin_w2"], golden["ad_lin_t"], 1.0]
    out = regions.linear_loss_backward(name).compile(device).execute(args)
    assert rel(out, golden[f"ad_lin_{name}"]) <= 2e-2


@pytest.mark.parametrize("name", ["dx", "dw1", "db1", "dw2", "db2", "dt"])
def test_biased_linear_loss_backward_region(device, golden, name):
    """Broadcast biases: BroadcastToShape in the forward, ReduceToShape onto
    the bias in the backward; bf16 GEMM operands, so 2e-2 against the
    reference's f32 vjp."""
    args = [golden[f"ad_linb_{k}"] for k in ("x", "w1", "b1", "w2", "b2", "t")] + [1.0]
    out = regions.linear_bias_loss_backward(name).compile(device).execute(args)
    assert rel(out, golden[f"ad_linb_{name}"]) <= 2e-2


@pytest.mark.parametrize("rows,cols,dtype", [(1, 1, np.float32), (33, 65, np.float32), (1000, 4096, np.float32),
                                             (257, 129, np.int64)])
def test_transpose(device, rows, cols, dtype):
    b = thb.RegionBuilder("t")
    x = b.input(thb.F32 if dtype == np.float32 else thb.I64, [None, None])
    spec = b.build(b.transpose(x))
    data = np.random.default_rng(rows).standard_normal((rows, cols)).astype(dtype) if dtype == np.float32 else \
        np.arange(rows * cols, dtype=np.int64).reshape(rows, cols)
    np.testing.assert_array_equal(spec.compile(device).execute([data]), data.T)


def test_broadcast_reduce_zero_like(device):
    rng = np.random.default_rng(41)
    m = rng.standard_normal((300, 257)).astype(np.float32)
    for axis, src in ((0, rng.standard_normal(257).astype(np.float32)), (1, rng.standard_normal(300).astype(np.float32))):
        b = thb.RegionBuilder("bc")
        v = b.input(thb.F32, [None])
        r = b.input(thb.F32, [None, None])
        spec = b.build(b.broadcast_to_shape(v, r, axis))
        np.testing.assert_array_equal(spec.compile(device).execute([src, m]), orc.region_eval(spec, [src, m]))
    b = thb.RegionBuilder("bs")
    s = b.input(thb.F32, [])
    r = b.input(thb.F32, [None])
    spec = b.build(b.broadcast_to_shape(s, r, 0))
    np.testing.assert_array_equal(spec.compile(device).execute([2.5, m[0]]), np.full(257, 2.5, np.float32))
    for ref in (np.zeros(257, np.float32), np.zeros((1, 257), np.float32), np.zeros((300, 1), np.float32),
                np.zeros((300, 257), np.float32)):
        b = thb.RegionBuilder("rs")
        v = b.input(thb.F32, [None, None])
        r = b.input(thb.F32, [None] * ref.ndim)
        spec = b.build(b.reduce_to_shape(v, r))
        got = spec.compile(device).execute([m, ref])
        want = orc.region_eval(spec, [m, ref])
        assert np.max(np.abs(got - want)) <= 1e-5 * max(1.0, float(np.max(np.abs(want))))
    b = thb.RegionBuilder("z")
    r = b.input(thb.F32, [None, None])
    spec = b.build(b.zero_like(r))
    np.testing.assert_array_equal(spec.compile(device).execute([m]), np.zeros_like(m))


def test_matmul_region_against_reference(device, golden):
    b = thb.RegionBuilder("mm")
    x = b.input(thb.F32, [None, None])
    y = b.input(thb.F32, [None, None])
    spec = b.build(b.matmul(x, y))
    out = spec.compile(device).execute([golden["mm_a"], golden["mm_b"]])  # 16x32 * 32x24
    assert rel(out, golden["mm_out"]) <= 2e-2
    rng = np.random.default_rng(51)
    a = rng.standard_normal((300, 512)).astype(np.float32)
    bm = rng.standard_normal((512, 264)).astype(np.float32)
    out = spec.compile(device).execute([a, bm])
    assert rel(out, orc.matmul_f64acc(a, bm)) <= 2e-2
    # K % 8 != 0: the operands are zero-padded to 16-byte rows in the bf16 cast.
    a5, b5 = np.ascontiguousarray(a[:, :500]), bm[:500].copy()
    out = spec.compile(device).execute([a5, b5])
    assert rel(out, orc.matmul_f64acc(a5, b5)) <= 2e-2
