"""GPU parity of the two-layer MLP training step (forward, reverse-AD
backward, SGD) against the CPU oracle's restatement of the reference's rules
(src/autodiff/v0/Autodiff.cpp:195-231, src/training/v0/Training.cpp:343-381).

Tolerances: against the oracle with the same bf16 rounding points, relative
Frobenius error <= 1e-2; against pure f32 operands (the reference's f32
semantics), the north-star bf16 tolerance 2e-2.
"""
import numpy as np
import pytest

import thiran_b200 as thb
import oracle_lib as orc

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def xavier(rng, fan_in, fan_out):
    bound = np.sqrt(6.0 / (fan_in + fan_out))
    return rng.uniform(-bound, bound, (fan_in, fan_out)).astype(np.float32)


@pytest.mark.parametrize("batch,d_in,hidden,d_out", [(256, 256, 512, 256), (512, 384, 1024, 128)])
def test_mlp_step_matches_oracle(device, batch, d_in, hidden, d_out):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(4)
    x = rng.standard_normal((batch, d_in)).astype(np.float32)
    w1 = xavier(rng, d_in, hidden)
    w2 = xavier(rng, hidden, d_out)
    t = rng.standard_normal((batch, d_out)).astype(np.float32)
    lr = 0.05

    s = thb.MlpSession(batch, d_in, hidden, d_out)
    cuda = lambda a: torch.from_numpy(a).cuda()
    X, T = cuda(x), cuda(t)
    W1 = s.bind(thb.MLP_W1, torch.empty((d_in, hidden), device="cuda"))
    W2 = s.bind(thb.MLP_W2, torch.empty((hidden, d_out), device="cuda"))
    DW1 = s.bind(thb.MLP_DW1, torch.empty((d_in, hidden), device="cuda"))
    DW2 = s.bind(thb.MLP_DW2, torch.empty((hidden, d_out), device="cuda"))
    Y = s.bind(thb.MLP_Y, torch.empty((batch, d_out), device="cuda"))
    L = s.bind(thb.MLP_LOSS_SUM, torch.zeros(2, dtype=torch.float64, device="cuda"))
    stream = torch.cuda.current_stream().cuda_stream
    s.set_weights(cuda(w1), cuda(w2), stream)
    s.step(X, T, lr, stream)
    thb.check_device_status(0, stream)
    torch.cuda.synchronize()

    w1o, w2o = w1.copy(), w2.copy()
    loss, dw1, dw2, hidden_o, y = orc.mlp_step(x, t, w1o, w2o, lr)
    gpu_loss = L[0].item() / (batch * d_out)
    assert abs(gpu_loss - loss) <= 1e-2 * loss
    assert rel(Y.cpu().numpy(), y) <= 1e-2
    assert rel(DW2.cpu().numpy(), dw2) <= 1e-2
    assert rel(DW1.cpu().numpy(), dw1) <= 1e-2
    assert rel(W1.cpu().numpy(), w1o) <= 1e-3
    assert rel(W2.cpu().numpy(), w2o) <= 1e-3

    # Against f32 operands (no bf16 rounding): the bf16 contract, 2e-2, for
    # the GEMM outputs whose operands are fresh inputs. dW1 = X^T dH composes
    # three bf16 rounding points (X, dY, dH) and is ill-conditioned at this
    # initialisation: rounding X alone moves it by ~3 % (the oracle shows the
    # same deviation), so it is held to 5e-2 end to end.
    h32 = np.maximum(x @ w1, 0)
    y32 = h32 @ w2
    d32 = (y32 - t) * (2.0 / (batch * d_out))
    dw2_32 = h32.T @ d32
    dw1_32 = x.T @ ((d32 @ w2.T) * (h32 > 0))
    assert rel(Y.cpu().numpy(), y32) <= 2e-2
    assert rel(DW2.cpu().numpy(), dw2_32) <= 2e-2
    assert rel(DW1.cpu().numpy(), dw1_32) <= 5e-2
    assert abs(rel(DW1.cpu().numpy(), dw1_32) - rel(dw1, dw1_32)) <= 5e-3


def test_mlp_training_trajectory_matches_oracle(device):
    """Ten SGD steps on a learnable target: the GPU loss sequence follows the
    oracle's step for step and decreases."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(11)
    batch, d_in, hidden, d_out = 512, 256, 512, 128
    x = rng.standard_normal((batch, d_in)).astype(np.float32)
    t = (x @ xavier(rng, d_in, d_out)).astype(np.float32)
    w1, w2 = xavier(rng, d_in, hidden), xavier(rng, hidden, d_out)
    lr = 0.5
    s = thb.MlpSession(batch, d_in, hidden, d_out)
    L = s.bind(thb.MLP_LOSS_SUM, torch.zeros(2, dtype=torch.float64, device="cuda"))
    s.set_weights(torch.from_numpy(w1).cuda(), torch.from_numpy(w2).cuda())
    X, T = torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda()
    gpu, ref = [], []
    w1o, w2o = w1.copy(), w2.copy()
    for _ in range(10):
        s.step(X, T, lr)
        torch.cuda.synchronize()
        gpu.append(L[0].item() / (batch * d_out))
        ref.append(orc.mlp_step(x, t, w1o, w2o, lr)[0])
    thb.check_device_status(0)
    np.testing.assert_allclose(gpu, ref, rtol=1e-2)
    assert all(b < a for a, b in zip(gpu, gpu[1:]))


def test_mlp_rejects_bad_extents(device):
    with pytest.raises(thb.GpuError) as err:
        thb.MlpSession(100, 256, 512, 128)  # batch not a multiple of 8
    assert err.value.code == "GPU-MLP-ARGUMENT"
