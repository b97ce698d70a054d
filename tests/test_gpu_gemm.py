"""tcgen05 GEMM parity against the CPU oracle.

The oracle multiplies the same bf16-rounded operands in f32 with f64
accumulation; the engine accumulates in f32 in tensor memory. Per-element
tolerance: |C - C_ref| <= 1e-3 * (|C_ref| + rms(C_ref)), a bound the f32
accumulation order difference stays well inside. Against the reference's f32
result (operands NOT rounded to bf16) the north-star bf16 tolerance applies:
relative Frobenius error <= 2e-2.
"""
import numpy as np
import pytest

import thiran_b200 as thb
import oracle_lib as orc

pytestmark = pytest.mark.gpu


def close(actual, expected, tol=1e-3):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    scale = np.abs(expected) + np.sqrt(np.mean(expected ** 2)) + 1e-30
    return float(np.max(np.abs(actual - expected) / scale)) <= tol


def run_gemm(torch, a32, b32, a_major, b_major, epilogue=thb.EPI_F32, aux32=None):
    """a32: logical A [M,K], b32: logical B [K,N] (f32 numpy, already bf16-exact)."""
    m, k = a32.shape
    n = b32.shape[1]
    a_store = a32 if a_major == thb.MAJOR_K else a32.T.copy()
    b_store = b32.T.copy() if b_major == thb.MAJOR_K else b32
    A = torch.from_numpy(np.ascontiguousarray(a_store)).cuda().to(torch.bfloat16)
    B = torch.from_numpy(np.ascontiguousarray(b_store)).cuda().to(torch.bfloat16)
    out_dtype = torch.float32 if epilogue == thb.EPI_F32 else torch.bfloat16
    Cm = torch.full((m, n), float("nan"), dtype=out_dtype, device="cuda")
    aux = torch.from_numpy(aux32).cuda().to(torch.bfloat16) if aux32 is not None else None
    s = torch.cuda.current_stream().cuda_stream
    thb.gemm(A, B, Cm, m, n, k, a_major, b_major, epilogue, aux=aux, stream=s)
    thb.check_device_status(0, s)
    return Cm.float().cpu().numpy()


@pytest.mark.parametrize("a_major", [thb.MAJOR_K, thb.MAJOR_MN])
@pytest.mark.parametrize("b_major", [thb.MAJOR_K, thb.MAJOR_MN])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 640), (384, 768, 1024), (200, 296, 136),
                                   # CTA-pair tiles (256 rows): second block partly / wholly past M,
                                   # more tiles than pairs; single CTAs: more tiles than SMs
                                   (136, 512, 128), (296, 256, 64), (4096, 2048, 256), (128, 40960, 192)])
def test_gemm_majors_and_shapes(device, a_major, b_major, m, n, k):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(m * 131 + n * 7 + k)
    a = orc.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    b = orc.round_bf16(rng.standard_normal((k, n)).astype(np.float32))
    c = run_gemm(torch, a, b, a_major, b_major)
    assert close(c, orc.matmul_f64acc(a, b))


@pytest.mark.parametrize("epilogue", [thb.EPI_BF16, thb.EPI_RELU_BF16, thb.EPI_MASK_BF16])
def test_gemm_epilogues(device, epilogue):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(epilogue)
    m, n, k = 256, 512, 512
    a = orc.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    b = orc.round_bf16(rng.standard_normal((k, n)).astype(np.float32))
    aux = orc.round_bf16(rng.standard_normal((m, n)).astype(np.float32)) if epilogue == thb.EPI_MASK_BF16 else None
    c = run_gemm(torch, a, b, thb.MAJOR_K, thb.MAJOR_MN, epilogue, aux)
    ref = orc.matmul_f64acc(a, b)
    if epilogue == thb.EPI_RELU_BF16:
        ref = np.maximum(ref, 0)
    if epilogue == thb.EPI_MASK_BF16:
        ref = np.where(aux > 0, ref, 0)
    ref = orc.round_bf16(ref)
    assert close(c, ref, tol=8e-3)  # one bf16 rounding of the result
    if epilogue != thb.EPI_BF16:
        assert np.array_equal(c == 0, ref == 0)


def test_gemm_against_reference_f32_semantics(device, golden):
    """The reference's own matmul (Evaluator order, f32 operands) at the
    golden fixture's shape, within the bf16 tolerance 2e-2."""
    torch = pytest.importorskip("torch")
    a, b = golden["mm_a"], golden["mm_b"]
    m, k = a.shape
    n = b.shape[1]
    pad = lambda x, r, c: np.pad(x, ((0, r - x.shape[0]), (0, c - x.shape[1])))
    ap, bp = pad(a, 128, 64), pad(b, 64, 256)
    c = run_gemm(torch, orc.round_bf16(ap), orc.round_bf16(bp), thb.MAJOR_K, thb.MAJOR_K)[:m, :n]
    ref = golden["mm_out"]
    assert np.linalg.norm(c - ref) / np.linalg.norm(ref) <= 2e-2


def test_gemm_rejects_bad_arguments(device):
    torch = pytest.importorskip("torch")
    a = torch.zeros((128, 60), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros((256, 60), dtype=torch.bfloat16, device="cuda")
    c = torch.zeros((128, 256), dtype=torch.float32, device="cuda")
    with pytest.raises(thb.GpuError) as err:
        thb.gemm(a, b, c, 128, 256, 60, lda=60, ldb=60)  # 60 is not a multiple of 8
    assert err.value.code == "GPU-GEMM-ARGUMENT"
