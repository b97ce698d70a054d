"""Parity at the sizes the benchmark lines are quoted on.

* The f32 chain ((x*1.5+0.25)*x - x)*0.5 + x on 2^28 elements (1 GiB per
  operand, x uniform[-1,1] from the device generator seeded 2): bit-exact
  against the oracle's IR-ordered, separately rounded restatement of the
  reference's native CPU path (src/backend/v0/NativeCpu.cpp:116-148), checked
  chunk by chunk.
* One MLP training step at batch 8192, 4096 -> 16384 -> 4096 with broadcast
  biases (zero-initialised), Xavier-uniform weights and N(0,1) inputs and
  targets. Full-size CPU GEMMs are impractical, so each GEMM output (H, Y,
  dW2, dW1; dH through the bias gradient db1) is checked on a 64 x 64 block of
  sampled rows and columns (4096 elements):
  - against the oracle's rule with the engine's own bf16 rounding points
    (the same bf16 operands, products summed in f64): the engine's
    accumulation order is the only difference, so 2e-3 per element,
    |d| <= 2e-3 (|ref| + rms(ref));
  - per GEMM against f32 operands (the reference's f32 semantics applied to
    the values each GEMM consumes, before their bf16 rounding), the bf16
    contract 2e-2 per element, |d| <= 2e-2 (|ref| + rms(ref)).
  The loss and the bias gradients are checked against f64 sums of the same
  quantities.

End to end against a pure f32 forward pass, dW1 differs by about 3 % (relative
Frobenius norm) for any bf16 rounding of X or W1: the rounding flips the ReLU
mask of pre-activations near zero, and dW1 = X^T (dY W2^T * mask) picks up
every flip. The oracle with the same rounding points shows the same
deviation (tests/test_gpu_mlp.py checks both); the per-GEMM bound above is
the contract the kernels are held to.
"""
import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions
import oracle_lib as orc

pytestmark = pytest.mark.gpu


def block_error(got, ref):
    """max |got - ref| / (|ref| + rms(ref)) over a block (f64)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref)))
    return float(np.max(np.abs(got - ref) / (np.abs(ref) + rms)))


def test_f32_chain_2p28_bit_exact(device):
    torch = pytest.importorskip("torch")
    n = 1 << 28
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.rand(n, device="cuda", generator=g) * 2 - 1
    y = torch.empty_like(x)
    spec = regions.f32_chain()
    region = spec.compile(device)
    stream = torch.cuda.current_stream().cuda_stream
    region.launch([x], y, stream)
    region.check_errors(stream)
    hx = x.cpu().numpy()
    hy = y.cpu().numpy()
    del x, y
    chunk = 1 << 24
    for start in range(0, n, chunk):
        want = orc.region_eval(spec, [hx[start:start + chunk]])
        got = hy[start:start + chunk]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"chunk at {start}"


def _bf16_of(torch, t):
    """bf16 rounding of a device tensor as f32 host values (round to nearest even)."""
    return t.to(torch.bfloat16).float().cpu().numpy()


def test_mlp_step_full_size_sampled(device):
    torch = pytest.importorskip("torch")
    torch.backends.cuda.matmul.allow_tf32 = False
    batch, d_in, hidden, d_out = 8192, 4096, 16384, 4096
    g = torch.Generator(device="cuda").manual_seed(4)
    b1 = (6.0 / (d_in + hidden)) ** 0.5
    b2 = (6.0 / (hidden + d_out)) ** 0.5
    X = torch.randn((batch, d_in), device="cuda", generator=g)
    W1 = (torch.rand((d_in, hidden), device="cuda", generator=g) * 2 - 1) * b1
    W2 = (torch.rand((hidden, d_out), device="cuda", generator=g) * 2 - 1) * b2
    T = torch.randn((batch, d_out), device="cuda", generator=g)

    s = thb.MlpSession(batch, d_in, hidden, d_out)
    Y = s.bind(thb.MLP_Y, torch.empty((batch, d_out), device="cuda"))
    H = s.bind(thb.MLP_H, torch.empty((batch, hidden), dtype=torch.bfloat16, device="cuda"))
    DW1 = s.bind(thb.MLP_DW1, torch.empty((d_in, hidden), device="cuda"))
    DW2 = s.bind(thb.MLP_DW2, torch.empty((hidden, d_out), device="cuda"))
    L = s.bind(thb.MLP_LOSS_SUM, torch.zeros(2, dtype=torch.float64, device="cuda"))
    stream = torch.cuda.current_stream().cuda_stream
    s.set_weights(W1, W2, stream)
    s.set_biases(stream=stream)
    from thiran_b200.distributed import bind_bias_gradients
    DB = bind_bias_gradients(s)
    s.forward_backward(X, T, stream)
    thb.check_device_status(device, stream)
    torch.cuda.synchronize()

    rng = np.random.default_rng(40)
    pick = lambda n: np.sort(rng.choice(n, 64, replace=False))
    scale = np.float32(2.0 / (batch * d_out))

    # Operands as the engine rounds them, and its outputs.
    Xb, W1b, W2b = _bf16_of(torch, X), _bf16_of(torch, W1), _bf16_of(torch, W2)
    x32, w1_32, w2_32, t32 = X.cpu().numpy(), W1.cpu().numpy(), W2.cpu().numpy(), T.cpu().numpy()
    h = H.float().cpu().numpy()           # bf16 values
    y = Y.cpu().numpy()
    dw1, dw2 = DW1.cpu().numpy(), DW2.cpu().numpy()
    db = DB.cpu().numpy()
    db1, db2 = db[:hidden], db[hidden:]
    d = (y - t32).astype(np.float32)      # D = Y - T, G = D * scale, dY = bf16(G)
    g32 = (d * scale).astype(np.float32)
    dyb = orc.round_bf16(g32)

    # H = relu(Xb W1b): the engine's bf16 output vs f64 sums of the same operands.
    I, J = pick(batch), pick(hidden)
    ref = np.maximum(Xb[I].astype(np.float64) @ W1b[:, J], 0)
    assert block_error(h[np.ix_(I, J)], ref) <= 2e-3 + 2 ** -8  # plus the output's bf16 rounding
    ref32 = np.maximum(x32[I].astype(np.float64) @ w1_32[:, J], 0)
    assert block_error(h[np.ix_(I, J)], ref32) <= 2e-2

    # Y = H W2b (H is the engine's bf16 activation).
    I, J = pick(batch), pick(d_out)
    ref = h[I].astype(np.float64) @ W2b[:, J]
    assert block_error(y[np.ix_(I, J)], ref) <= 2e-3
    assert block_error(y[np.ix_(I, J)], h[I].astype(np.float64) @ w2_32[:, J]) <= 2e-2

    # Loss (f64 sum of D^2) and db2 (column sums of G).
    loss = float(np.sum(d.astype(np.float64) ** 2))
    assert abs(L[0].item() - loss) <= 1e-5 * loss
    assert block_error(db2, g32.astype(np.float64).sum(axis=0)) <= 1e-5

    # dW2 = H^T dY.
    I, J = pick(hidden), pick(d_out)
    ref = h[:, I].T.astype(np.float64) @ dyb[:, J]
    assert block_error(dw2[np.ix_(I, J)], ref) <= 2e-3
    assert block_error(dw2[np.ix_(I, J)], h[:, I].T.astype(np.float64) @ g32[:, J]) <= 2e-2

    # dH = (dY W2b^T) * [H > 0] on sampled columns; db1 = its column sums
    # (f32, before the bf16 rounding); dW1 = Xb^T dH.
    I, J = pick(d_in), pick(hidden)
    mask = h[:, J] > 0
    dh_cols = (dyb.astype(np.float64) @ W2b[J].T) * mask          # [batch, 64]
    assert block_error(db1[J], dh_cols.sum(axis=0)) <= 2e-3
    dh_cols32 = (g32.astype(np.float64) @ w2_32[J].T) * mask
    assert block_error(db1[J], dh_cols32.sum(axis=0)) <= 2e-2
    dhb = orc.round_bf16(dh_cols.astype(np.float32))
    ref = Xb[:, I].T.astype(np.float64) @ dhb
    assert block_error(dw1[np.ix_(I, J)], ref) <= 2e-3
    assert block_error(dw1[np.ix_(I, J)], x32[:, I].T.astype(np.float64) @ dh_cols32) <= 2e-2
    s.release()
