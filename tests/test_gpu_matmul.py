"""MatMul region nodes in all three forms, against the reference Evaluator's
rule (src/semantic/v0/Evaluator.cpp:125-154) as recorded from the reference
and restated by the oracle:

* i64: checked multiply and add, bit-exact, TH-SPEC-I64-OVERFLOW when a
  product or a partial sum leaves the i64 range;
* f32 exact mode: sequential, separately rounded f32 sums, bit-exact;
* f32 tensor-core mode (bf16 operands, f32 accumulation) at shapes whose K
  and N are not multiples of 8: the bf16 contract, per element
  |d| <= 2e-2 (|ref| + rms(ref)).

examples/transformer.th (MatMul, Transpose, Softmax, Add) runs as one region
and follows the oracle; the softmax's exp is CUDA's expf against glibc's exp,
so the bound there is 1e-5 relative per element.
"""
import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions
import oracle_lib as orc

pytestmark = pytest.mark.gpu


def block_error(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref)))
    return float(np.max(np.abs(got - ref) / (np.abs(ref) + rms)))


def test_matmul_i64_matches_reference(device, golden):
    region = regions.matmul(thb.I64).compile(device)
    out = region.execute([golden["mm_i64_a"], golden["mm_i64_b"]])
    np.testing.assert_array_equal(out, golden["mm_i64_out"])


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (64, 64, 64), (130, 517, 77), (300, 16, 1000), (5, 3000, 7)])
def test_matmul_i64_random_exact(device, m, k, n):
    rng = np.random.default_rng(m * 7 + k + n)
    a = rng.integers(-(1 << 20), 1 << 20, (m, k), dtype=np.int64)
    b = rng.integers(-(1 << 20), 1 << 20, (k, n), dtype=np.int64)
    spec = regions.matmul(thb.I64)
    np.testing.assert_array_equal(spec.compile(device).execute([a, b]), orc.region_eval(spec, [a, b]))


def test_matmul_i64_overflow(device, fixtures):
    region = regions.matmul(thb.I64).compile(device)
    half = np.array([[1 << 62, 1 << 62]], np.int64)
    root = np.array([[3037000500]], np.int64)
    for key, (a, b) in (("mm_i64_sum_overflow", (half, np.array([[1], [1]], np.int64))),
                        ("mm_i64_product_overflow", (root, root))):
        with pytest.raises(thb.GpuError) as err:
            region.execute([a, b])
        assert err.value.code == fixtures[key] == "TH-SPEC-I64-OVERFLOW"
    # The region is usable again after a failed call.
    a = np.arange(6, dtype=np.int64).reshape(2, 3)
    np.testing.assert_array_equal(region.execute([a, a.T.copy()]), a @ a.T)


def test_matmul_exact_f32_bitwise(device, golden):
    region = regions.matmul(thb.F32, exact=True).compile(device)
    for a, b, want in ((golden["mm_a"], golden["mm_b"], golden["mm_out"]),
                       (golden["mm_odd_a"], golden["mm_odd_b"], golden["mm_odd_out"])):
        out = region.execute([a, b])
        assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("m,k,n", [(2, 4, 4), (2, 4, 2), (2, 2, 8), (257, 1023, 129), (64, 4096, 96)])
def test_matmul_exact_f32_random_bitwise(device, m, k, n):
    rng = np.random.default_rng(m + k + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    spec = regions.matmul(thb.F32, exact=True)
    out = spec.compile(device).execute([a, b])
    want = orc.region_eval(spec, [a, b])
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("m,k,n", [(37, 13, 5), (2, 4, 4), (2, 4, 2), (2, 2, 8), (300, 517, 131), (129, 1001, 3)])
def test_matmul_tensor_cores_any_k_and_n(device, golden, m, k, n):
    """K or N not a multiple of 8: the operands are zero-padded in the bf16
    cast, so the result follows the f32 rule within the bf16 contract."""
    if (m, k, n) == (37, 13, 5):
        a, b, want = golden["mm_odd_a"], golden["mm_odd_b"], golden["mm_odd_out"]
    else:
        rng = np.random.default_rng(m * 3 + k + n)
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        want = orc.matmul_f32(a, b)
    out = regions.matmul(thb.F32).compile(device).execute([a, b])
    assert out.shape == (m, n)
    assert block_error(out, want) <= 2e-2
    # Same bf16 operands summed in f64: only the accumulation order differs.
    exact_bf16 = orc.round_bf16(a).astype(np.float64) @ orc.round_bf16(b).astype(np.float64)
    assert block_error(out, exact_bf16) <= 1e-4


def test_transformer_example_region(device):
    """examples/transformer.th on its own shapes and on a larger block."""
    torch = pytest.importorskip("torch")
    for tokens, d, dv in ((2, 4, 8), (96, 64, 128)):
        rng = np.random.default_rng(tokens)
        x = rng.standard_normal((tokens, d)).astype(np.float32)
        w = lambda rows, cols: (rng.standard_normal((rows, cols)) / np.sqrt(rows)).astype(np.float32)
        wq, wk, wv, wo = w(d, d), w(d, d), w(d, dv), w(dv, d)
        inputs = [x, wq, wk, wv, wo]
        spec = regions.transformer_block(exact=True)
        out = spec.compile(device).execute(inputs)
        want = orc.region_eval(spec, inputs)
        np.testing.assert_allclose(out, want, rtol=1e-5, atol=1e-6)
        # The legacy torch lowering (PythonExecutorEmitter.cpp:87-97), f32 on the CPU.
        tx = [torch.from_numpy(v) for v in inputs]
        q, k = tx[0] @ tx[1], tx[0] @ tx[2]
        ctx = torch.softmax(q @ k.T, dim=-1) @ (tx[0] @ tx[3])
        np.testing.assert_allclose(out, (ctx @ tx[4] + tx[0]).numpy(), rtol=1e-4, atol=1e-5)
        # Tensor-core matmuls: six bf16-operand products composed through a
        # softmax (each product alone holds the per-element contract, tested
        # above), so the block is held to 2e-2 in relative Frobenius norm.
        fast = regions.transformer_block(exact=False).compile(device).execute(inputs)
        assert np.linalg.norm(fast.astype(np.float64) - want) <= 2e-2 * np.linalg.norm(want.astype(np.float64))


@pytest.mark.parametrize("m,k,n", [(0, 5, 3), (4, 0, 3), (4, 5, 0), (0, 0, 0)])
def test_matmul_empty_extents(device, m, k, n):
    """Empty extents: an empty result, or K = 0 giving zeros (the Evaluator's
    accumulators start at 0), in every form."""
    for dtype, exact in ((thb.F32, True), (thb.F32, False), (thb.I64, False)):
        np_type = np.int64 if dtype == thb.I64 else np.float32
        a, b = np.ones((m, k), np_type), np.ones((k, n), np_type)
        spec = regions.matmul(dtype, exact)
        out = spec.compile(device).execute([a, b])
        want = orc.region_eval(spec, [a, b])
        assert out.shape == want.shape == (m, n)
        np.testing.assert_array_equal(out, want)
        assert not out.any()
