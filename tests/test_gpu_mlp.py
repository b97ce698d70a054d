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
    s.forward_backward(X, T, stream)
    s.apply_sgd(lr, stream)
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


@pytest.mark.parametrize("batch,d_in,hidden,d_out,momentum", [(256, 256, 512, 256, 0.0), (256, 256, 512, 256, 0.9),
                                                              (200, 136, 520, 136, 0.5), (384, 256, 512, 256, 0.9)])
def test_mlp_biases_and_momentum_match_oracle(device, batch, d_in, hidden, d_out, momentum):
    """The examples/mlp.th structure (broadcast biases, their gradients the
    column sums of dH and dY) with SGD or SGD with momentum (Training.cpp:
    366-372): three steps follow the oracle. The last shape leaves partial
    M tiles (200 rows) and a partial N tile (520 columns), so rows past the
    batch must add nothing to the bias gradient."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(21)
    x = rng.standard_normal((batch, d_in)).astype(np.float32)
    t = rng.standard_normal((batch, d_out)).astype(np.float32)
    w1, w2 = xavier(rng, d_in, hidden), xavier(rng, hidden, d_out)
    b1 = (rng.standard_normal(hidden) * 0.1).astype(np.float32)
    b2 = (rng.standard_normal(d_out) * 0.1).astype(np.float32)
    lr = 0.1
    cuda = lambda a: torch.from_numpy(a).cuda()
    s = thb.MlpSession(batch, d_in, hidden, d_out)
    W1 = s.bind(thb.MLP_W1, torch.empty((d_in, hidden), device="cuda"))
    W2 = s.bind(thb.MLP_W2, torch.empty((hidden, d_out), device="cuda"))
    L = s.bind(thb.MLP_LOSS_SUM, torch.zeros(2, dtype=torch.float64, device="cuda"))
    s.set_weights(cuda(w1), cuda(w2))
    s.set_biases(cuda(b1), cuda(b2))
    s.set_momentum(momentum)
    B1 = s.bind(thb.MLP_B1, torch.empty(hidden, device="cuda"))
    B2 = s.bind(thb.MLP_B2, torch.empty(d_out, device="cuda"))
    B1.copy_(cuda(b1))
    B2.copy_(cuda(b2))
    DB1 = s.bind(thb.MLP_DB1, torch.empty(hidden, device="cuda"))
    DB2 = s.bind(thb.MLP_DB2, torch.empty(d_out, device="cuda"))
    X, T = cuda(x), cuda(t)
    ws = [w1.copy(), w2.copy(), b1.copy(), b2.copy()]
    vel = [np.zeros_like(a) for a in (w1, b1, w2, b2)] if momentum else None
    for step in range(3):
        s.step(X, T, lr)
        torch.cuda.synchronize()
        loss, dw1, dw2, db1, db2, _, _ = orc.mlp_step_ex(x, t, ws[0], ws[1], lr, ws[2], ws[3], momentum, vel)
        assert abs(L[0].item() / (batch * d_out) - loss) <= 1e-2 * loss, step
        assert rel(DB2.cpu().numpy(), db2) <= 1e-2, step
        assert rel(DB1.cpu().numpy(), db1) <= 1e-2, step
    thb.check_device_status(0)
    assert rel(W1.cpu().numpy(), ws[0]) <= 1e-3
    assert rel(W2.cpu().numpy(), ws[1]) <= 1e-3
    assert rel(B1.cpu().numpy(), ws[2]) <= 1e-3
    assert rel(B2.cpu().numpy(), ws[3]) <= 1e-3


@pytest.mark.parametrize("batch,d_in,hidden,d_out", [(512, 128, 256, 128), (256, 128, 256, 2056)])
def test_mlp_bias_gradient_against_f32_column_sums(device, batch, d_in, hidden, d_out):
    """db2 is exactly what the f32 loss gradient sums to (no bf16 rounding
    sits between Y and dY's column sums), 1e-5 relative per element; the
    second shape has more output columns than one loss block covers."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    x = rng.standard_normal((batch, d_in)).astype(np.float32)
    t = rng.standard_normal((batch, d_out)).astype(np.float32)
    w1, w2 = xavier(rng, d_in, hidden), xavier(rng, hidden, d_out)
    s = thb.MlpSession(batch, d_in, hidden, d_out)
    s.set_weights(torch.from_numpy(w1).cuda(), torch.from_numpy(w2).cuda())
    s.set_biases()
    Y = s.bind(thb.MLP_Y, torch.empty((batch, d_out), device="cuda"))
    DB2 = s.bind(thb.MLP_DB2, torch.empty(d_out, device="cuda"))
    s.forward_backward(torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda())
    torch.cuda.synchronize()
    y = Y.cpu().numpy()
    g = ((y - t) * np.float32(2.0 / (batch * d_out))).astype(np.float32)
    np.testing.assert_allclose(DB2.cpu().numpy(), g.astype(np.float64).sum(0), rtol=1e-5, atol=1e-9)


def test_mlp_momentum_bounds(device):
    s = thb.MlpSession(64, 64, 64, 64)
    for bad, code in ((-0.1, "OPT05"), (float("nan"), "OPT05"), (1.0, "OPT06")):
        with pytest.raises(thb.GpuError) as err:
            s.set_momentum(bad)
        assert err.value.code == code


def test_mlp_rejects_bad_extents(device):
    with pytest.raises(thb.GpuError) as err:
        thb.MlpSession(100, 256, 512, 128)  # batch not a multiple of 8
    assert err.value.code == "GPU-MLP-ARGUMENT"


@pytest.mark.parametrize("batch,d_in,hidden,d_out,momentum,biases", [(256, 256, 512, 256, 0.0, False),
                                                                     (384, 256, 512, 256, 0.9, True),
                                                                     (200, 136, 520, 136, 0.5, True)])
def test_mlp_fused_update_step_is_bit_identical(device, batch, d_in, hidden, d_out, momentum, biases):
    """thb_mlp_step applies the weight updates inside the dW GEMMs' read-out;
    three steps must give the same parameter bits (and the same loss) as
    forward_backward followed by the standalone SGD pass. The last shape
    leaves partial tiles, where the read-out takes its scalar path."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(17)
    x = torch.from_numpy(rng.standard_normal((batch, d_in)).astype(np.float32)).cuda()
    t = torch.from_numpy(rng.standard_normal((batch, d_out)).astype(np.float32)).cuda()
    w1 = torch.from_numpy(xavier(rng, d_in, hidden)).cuda()
    w2 = torch.from_numpy(xavier(rng, hidden, d_out)).cuda()
    b1 = torch.from_numpy((rng.standard_normal(hidden) * 0.1).astype(np.float32)).cuda()
    b2 = torch.from_numpy((rng.standard_normal(d_out) * 0.1).astype(np.float32)).cuda()
    runs = []
    for fused in (False, True):
        s = thb.MlpSession(batch, d_in, hidden, d_out)
        params = {"w1": s.bind(thb.MLP_W1, torch.empty_like(w1)), "w2": s.bind(thb.MLP_W2, torch.empty_like(w2))}
        loss = s.bind(thb.MLP_LOSS_SUM, torch.zeros(2, dtype=torch.float64, device="cuda"))
        s.set_weights(w1, w2)
        if biases:
            s.set_biases(b1, b2)
            params["b1"] = s.bind(thb.MLP_B1, b1.clone())
            params["b2"] = s.bind(thb.MLP_B2, b2.clone())
        s.set_momentum(momentum)
        losses = []
        for _ in range(3):
            if fused:
                s.step(x, t, 0.05)
            else:
                s.forward_backward(x, t)
                s.apply_sgd(0.05)
            losses.append(loss[0].item())
        thb.check_device_status(0)
        runs.append(({k: v.cpu() for k, v in params.items()}, losses))
        s.release()
    (plain, plain_losses), (fused_p, fused_losses) = runs
    assert plain_losses == fused_losses
    for k in plain:
        assert torch.equal(plain[k].view(torch.int32), fused_p[k].view(torch.int32)), k


def test_compact_reduction_on_one_rank(device):
    """The bf16 sharded reduction's kernels on a world of one (every tile
    owned here, the ranks' bf16 tiles read back through the peer path): three
    steps follow the single-process f32 step and the oracle, and the bf16
    weight copies are the rounding of the f32 weights."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(31)
    batch, d_in, hidden, d_out = 384, 256, 520, 136   # a ragged N tile in both layers
    x = rng.standard_normal((batch, d_in)).astype(np.float32)
    t = rng.standard_normal((batch, d_out)).astype(np.float32)
    w1, w2 = xavier(rng, d_in, hidden), xavier(rng, hidden, d_out)
    b1 = (rng.standard_normal(hidden) * 0.1).astype(np.float32)
    b2 = (rng.standard_normal(d_out) * 0.1).astype(np.float32)
    lr, momentum = 0.1, 0.9
    cuda = lambda a: torch.from_numpy(a).cuda()
    X, T = cuda(x), cuda(t)

    def make():
        s = thb.MlpSession(batch, d_in, hidden, d_out)
        s.set_weights(cuda(w1), cuda(w2))
        s.set_biases(cuda(b1), cuda(b2))
        s.set_momentum(momentum)
        return s, {"b1": s.bind(thb.MLP_B1, cuda(b1)), "b2": s.bind(thb.MLP_B2, cuda(b2))}

    plain, pp = make()
    pp["w1"] = plain.bind(thb.MLP_W1, cuda(w1))
    pp["w2"] = plain.bind(thb.MLP_W2, cuda(w2))
    plain.set_weights(cuda(w1), cuda(w2))
    for _ in range(3):
        plain.forward_backward(X, T)
        plain.apply_sgd(lr)

    s, cp = make()
    grads = {thb.MLP_DW1: torch.empty((d_in, hidden), dtype=torch.bfloat16, device="cuda"),
             thb.MLP_DW2: torch.empty((hidden, d_out), dtype=torch.bfloat16, device="cuda")}
    flags = {k: torch.zeros(s.reduction_flag_words(k), dtype=torch.int32, device="cuda") for k in grads}
    for k, g in grads.items():
        s.bind_reduction(k, [g.data_ptr()], [flags[k].data_ptr()], 0, 1)
        s.set_reduction_format(k, thb.REDUCE_BF16_SHARDED)
    params = {thb.MLP_W1: (torch.empty((d_in, hidden), device="cuda"),
                           torch.empty((d_in, hidden), dtype=torch.bfloat16, device="cuda")),
              thb.MLP_W2: (torch.empty((hidden, d_out), device="cuda"),
                           torch.empty((hidden, d_out), dtype=torch.bfloat16, device="cuda"))}
    for k, (p, c) in params.items():
        s.bind_update(k, [p.data_ptr()], [c.data_ptr()])
    s.set_weights(cuda(w1), cuda(w2))
    s.set_momentum(momentum)
    with pytest.raises(thb.GpuError):  # the compact form needs the update in the reduction
        s.forward_backward(X, T)
    for _ in range(3):
        s.forward_backward_update(X, T, lr)
        s.apply_sgd(lr)
    for k in params:
        s.gather_parameters(k)
    thb.check_device_status(0)
    torch.cuda.synchronize()
    got = {"w1": params[thb.MLP_W1][0], "w2": params[thb.MLP_W2][0], "b1": cp["b1"], "b2": cp["b2"]}
    for k in ("w1", "w2", "b1", "b2"):
        assert rel(got[k].cpu().numpy(), pp[k].cpu().numpy()) <= 1e-3, k
    ws = [w1.copy(), w2.copy(), b1.copy(), b2.copy()]
    vel = [np.zeros_like(a) for a in (w1, b1, w2, b2)]
    for _ in range(3):
        orc.mlp_step_ex(x, t, ws[0], ws[1], lr, ws[2], ws[3], momentum, vel)
    for k, ref in zip(("w1", "w2", "b1", "b2"), ws):
        assert rel(got[k].cpu().numpy(), ref) <= 1e-3, k
    for k, (p, c) in params.items():
        assert torch.equal(c, p.to(torch.bfloat16)), k
    s.release()
    plain.release()
