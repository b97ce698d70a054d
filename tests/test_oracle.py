"""Pins the CPU oracle against the reference's own outputs (tests/golden/,
produced by tests/golden/make_golden.py from the reference's Evaluator and
native CPU path) and the known-answer vectors of the reference's tests."""
import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions
import oracle_lib as orc


def test_kat_f32_chain(golden):
    # tests/backend/v0/NativeGpuIntegrationTests.cpp:72-112
    out = orc.region_eval(regions.f32_chain4(), [golden["kat_f32_a"], golden["kat_f32_b"]])
    np.testing.assert_array_equal(out, golden["kat_f32_out"])


def test_kat_i64_odd_size(golden):
    # NativeGpuIntegrationTests.cpp:139-163: n=257, all 3 -> 18
    x = np.full(257, 3, np.int64)
    out = orc.region_eval(regions.i64_dynamic(), [x, x])
    np.testing.assert_array_equal(out, golden["kat_i64_257_out"])
    assert out[0] == 18 and out[-1] == 18


def test_kat_i64_differential(golden):
    # NativeGpuIntegrationTests.cpp:165-189: 100 generated cases, exact
    spec = regions.i64_dynamic()
    for case in range(100):
        out = orc.region_eval(spec, [golden["kat_i64_diff_left"][case], golden["kat_i64_diff_right"][case]])
        np.testing.assert_array_equal(out, golden["kat_i64_diff_out"][case])


def test_kat_overflow(fixtures):
    # NativeGpuIntegrationTests.cpp:277-283
    with pytest.raises(orc.OracleFailure) as err:
        orc.region_eval(regions.i64_dynamic(), [np.array([2**63 - 1], np.int64), np.array([1], np.int64)])
    assert err.value.code == fixtures["kat_i64_overflow"]["status"] == "TH-SPEC-I64-OVERFLOW"


@pytest.mark.parametrize("index", [256, 257, -1])
def test_kat_index_bounds(fixtures, index):
    b = thb.RegionBuilder("pick")
    x = b.input(thb.I64, [None])
    i = b.input(thb.I64, [])
    spec = b.build(b.index(b.alias(x), b.alias(i)))
    expected = fixtures[f"kat_pick_{index}"]
    try:
        value = orc.region_eval(spec, [np.full(257, 3, np.int64), index])
        assert expected["status"] == "ok" and value == expected["value"]
    except orc.OracleFailure as err:
        assert err.code == expected["status"] == "TH-SPEC-BOUNDS"


def test_kat_square_linear(golden):
    # examples/research_extension: x*x + x
    op = thb.Operation("research_square_linear",
                       [(thb.SCALAR_INPUT, 0, 0, 0, 0.0), (thb.SCALAR_MULTIPLY, 0, 0, 0, 0.0),
                        (thb.SCALAR_ADD, 1, 0, 0, 0.0)], root=2)
    b = thb.RegionBuilder("f")
    x = b.input(thb.F32, [None])
    spec = b.build(b.extension(op, b.alias(x)))
    out = orc.region_eval(spec, [golden["kat_square_linear_in"]])
    np.testing.assert_array_equal(out, golden["kat_square_linear_out"])
    np.testing.assert_array_equal(out, np.array([2.0, -0.25, 0.0, 3.75, 12.0, 59.8125, 72.0], np.float32))


def test_chain_matches_reference_native_cpu_bitwise(golden):
    out = orc.region_eval(regions.f32_chain(), [golden["chain_x"]])
    assert out.view(np.uint32).tolist() == golden["chain_native_cpu"].view(np.uint32).tolist()
    assert out.view(np.uint32).tolist() == golden["chain_eval"].view(np.uint32).tolist()


def test_i64_region_matches_reference_native_cpu(golden, fixtures):
    out = orc.region_eval(regions.i64_region(), [golden["i64_a"], golden["i64_b"]])
    np.testing.assert_array_equal(out, golden["i64_native_cpu"])
    np.testing.assert_array_equal(out, golden["i64_eval"])
    big = np.array([[3037000500, 1]], np.int64)
    with pytest.raises(orc.OracleFailure) as err:
        orc.region_eval(regions.i64_region(), [big, np.zeros_like(big)])
    assert err.value.code == fixtures["i64_region"]["overflow_id"]


def test_sums_against_reference_evaluator(golden):
    m = golden["sum_in"]
    # The reference sums sequentially in f32 (Evaluator.cpp:221-226); the
    # oracle accumulates in f64. They agree to the f32 ordering error.
    np.testing.assert_allclose(orc.sum_rows(m), golden["sum_rows"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(orc.sum_cols(m), golden["sum_cols"], rtol=1e-5, atol=1e-5)
    total = orc.sum_all_f64(m)
    assert abs(total - float(golden["sum_total"])) <= 1e-4 * max(1.0, abs(total))
    # The sequential-f32 restatement reproduces the reference exactly for a
    # row-major flat sum of one row (same order).
    row = np.ascontiguousarray(m[0])
    assert orc.sum_all_sequential_f32(row) == np.float32(golden["sum_rows"][0]) or \
        abs(orc.sum_all_sequential_f32(row) - golden["sum_rows"][0]) == 0


def test_matmul_evaluator_order_bitwise(golden):
    out = orc.matmul_f32(golden["mm_a"], golden["mm_b"])
    assert out.view(np.uint32).tolist() == golden["mm_out"].view(np.uint32).tolist()
    odd = orc.region_eval(regions.matmul(thb.F32, exact=True), [golden["mm_odd_a"], golden["mm_odd_b"]])
    assert odd.view(np.uint32).tolist() == golden["mm_odd_out"].view(np.uint32).tolist()


def test_matmul_i64_checked_against_reference(golden, fixtures):
    spec = regions.matmul(thb.I64)
    out = orc.region_eval(spec, [golden["mm_i64_a"], golden["mm_i64_b"]])
    np.testing.assert_array_equal(out, golden["mm_i64_out"])
    half = np.array([[1 << 62, 1 << 62]], np.int64)
    root = np.array([[3037000500]], np.int64)
    for key, (a, b) in (("mm_i64_sum_overflow", (half, np.array([[1], [1]], np.int64))),
                        ("mm_i64_product_overflow", (root, root))):
        with pytest.raises(orc.OracleFailure) as err:
            orc.region_eval(spec, [a, b])
        assert err.value.code == fixtures[key] == "TH-SPEC-I64-OVERFLOW"


def test_softmax_restatement_against_numpy():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((33, 257)).astype(np.float32)
    y = orc.softmax_rows(x)
    xd = x.astype(np.float64)
    e = np.exp(xd - xd.max(axis=1, keepdims=True))
    np.testing.assert_allclose(y, e / e.sum(axis=1, keepdims=True), rtol=1e-6, atol=0)


def test_softmax_restatement_against_torch_cpu():
    # The legacy stack lowers softmax to torch.softmax(x, dim=-1)
    # (src/region/RegionPythonEmitter.cpp:293-294).
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(8)
    x = rng.standard_normal((16, 4096)).astype(np.float32)
    ref = torch.softmax(torch.from_numpy(x), dim=-1).numpy()
    np.testing.assert_allclose(orc.softmax_rows(x), ref, rtol=1e-5, atol=1e-9)


def test_relu_restatement_against_torch_cpu():
    torch = pytest.importorskip("torch")
    x = np.array([-2.0, -0.0, 0.0, 1.5, np.inf, -np.inf, np.nan], np.float32)
    b = thb.RegionBuilder("r")
    v = b.input(thb.F32, [None])
    out = orc.region_eval(b.build(b.relu(v)), [x])
    ref = torch.relu(torch.from_numpy(x)).numpy()
    np.testing.assert_array_equal(np.isnan(out), np.isnan(ref))
    np.testing.assert_array_equal(out[~np.isnan(out)], ref[~np.isnan(ref)])


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(4096) * 10).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    np.testing.assert_array_equal(orc.round_bf16(x), ref)


def test_planted_mistake_is_caught(golden):
    """A wrong oracle must fail the fixture comparison (harness is not blind)."""
    out = orc.region_eval(regions.f32_chain(), [golden["chain_x"]])
    out[123] = np.nextafter(out[123], np.float32(2))
    assert out.view(np.uint32).tolist() != golden["chain_native_cpu"].view(np.uint32).tolist()


def test_ad_extension_gradients_match_reference(golden):
    """Gradient recipes of extension descriptors, evaluated elementwise, equal
    the reference's reverse mode (Autodiff.cpp:231-270) bit for bit."""
    spec = regions.extension_gradient(regions.square_linear_operation())
    out = orc.region_eval(spec, [golden["kat_square_linear_in"], golden["ad_square_linear_dz"]])
    assert out.view(np.uint32).tolist() == golden["ad_square_linear_grad"].view(np.uint32).tolist()
    spec = regions.extension_gradient(regions.chain_operation())
    out = orc.region_eval(spec, [golden["ad_chain_x"], golden["ad_chain_dz"]])
    assert out.view(np.uint32).tolist() == golden["ad_chain_grad"].view(np.uint32).tolist()


@pytest.mark.parametrize("name", ["dx", "dw1", "db1", "dw2", "db2", "dt"])
def test_ad_biased_linear_loss_backward_matches_reference(golden, name):
    """With broadcast biases (the examples/mlp.th structure) the generated
    backward adds ReduceToShape onto each bias; restated as a region it
    reproduces the reference's vjp bit for bit."""
    args = [golden[f"ad_linb_{k}"] for k in ("x", "w1", "b1", "w2", "b2", "t")] + [1.0]
    out = orc.region_eval(regions.linear_bias_loss_backward(name), args)
    assert out.view(np.uint32).tolist() == golden[f"ad_linb_{name}"].view(np.uint32).tolist()


def test_momentum_update_matches_reference_training_tests():
    """SGDMomentum known answers of the reference (TrainingTests.cpp:168-193,
    204-210): lr 0.01, mu 0.5, parameters (bias, weight) from 0, gradients
    (-32, -68) then (-21.28, -45.12); and lr 0.1 with v = 4, g = 0."""
    p = np.zeros(2, np.float32)
    v = np.zeros(2, np.float32)
    orc.sgd_update(p, np.array([-32, -68], np.float32), 0.01, v, 0.5)
    np.testing.assert_allclose(v, [-32, -68], rtol=0, atol=1e-6)
    np.testing.assert_allclose(p, [0.32, 0.68], rtol=0, atol=1e-6)
    plain = np.zeros(2, np.float32)
    orc.sgd_update(plain, np.array([-32, -68], np.float32), 0.01)
    assert plain.view(np.uint32).tolist() == p.view(np.uint32).tolist()  # TRAIN15
    orc.sgd_update(p, np.array([-21.28, -45.12], np.float32), 0.01, v, 0.5)
    np.testing.assert_allclose(v, [-37.28, -79.12], rtol=0, atol=2e-5)
    np.testing.assert_allclose(p, [0.6928, 1.4712], rtol=0, atol=2e-5)
    q = np.array([3.0], np.float32)
    vq = np.array([4.0], np.float32)
    orc.sgd_update(q, np.zeros(1, np.float32), 0.1, vq, 0.5)
    np.testing.assert_allclose([vq[0], q[0]], [2.0, 2.8], rtol=0, atol=1e-6)


def test_mlp_step_with_biases_matches_column_sum_rule():
    """The oracle's biased MLP step: bias gradients are the column sums of
    dY and the masked dH, and a momentum step from zero velocity equals the
    plain SGD step."""
    rng = np.random.default_rng(12)
    x = rng.standard_normal((32, 16)).astype(np.float32)
    t = rng.standard_normal((32, 8)).astype(np.float32)
    w1 = (rng.uniform(-1, 1, (16, 24)) * 0.3).astype(np.float32)
    w2 = (rng.uniform(-1, 1, (24, 8)) * 0.3).astype(np.float32)
    b1 = (rng.standard_normal(24) * 0.1).astype(np.float32)
    b2 = (rng.standard_normal(8) * 0.1).astype(np.float32)
    runs = []
    for momentum in (0.0, 0.9):
        ws = [w1.copy(), w2.copy(), b1.copy(), b2.copy()]
        vel = [np.zeros_like(a) for a in (w1, b1, w2, b2)] if momentum else None
        loss, dw1, dw2, db1, db2, hidden, y = orc.mlp_step_ex(x, t, ws[0], ws[1], 0.05, ws[2], ws[3], momentum, vel)
        runs.append(ws)
    xb, w1b, w2b = (orc.round_bf16(a) for a in (x, w1, w2))
    h = np.maximum(xb.astype(np.float64) @ w1b + b1, 0)
    yy = orc.round_bf16(h.astype(np.float32)).astype(np.float64) @ w2b + b2
    dy = 2 * (yy - t) / (32 * 8)
    np.testing.assert_allclose(db2, dy.sum(0), rtol=1e-4, atol=1e-6)
    dh = (orc.round_bf16(dy.astype(np.float32)).astype(np.float64) @ w2b.T) * (h > 0)
    np.testing.assert_allclose(db1, dh.sum(0), rtol=1e-3, atol=1e-6)
    for a, b in zip(*runs):
        assert a.view(np.uint32).tolist() == b.view(np.uint32).tolist()


@pytest.mark.parametrize("name", ["dx", "dw1", "dw2", "dt"])
def test_ad_linear_loss_backward_matches_reference(golden, name):
    """The reference's generated backward (BroadcastToShape, ReduceToShape,
    Transpose, MatMul, Negate) restated as a region reproduces its vjp."""
    args = [golden["ad_lin_x"], golden["ad_lin_w1"], golden["ad_lin_w2"], golden["ad_lin_t"], 1.0]
    out = orc.region_eval(regions.linear_loss_backward(name), args)
    assert out.view(np.uint32).tolist() == golden[f"ad_lin_{name}"].view(np.uint32).tolist()


def cube_scene():
    """The reference's TH-019 cube (tests/graphics/v0/GraphicsTests.cpp:358-376)."""
    g = orc.gfx
    positions = np.array([-1, -1, -1, 1, -1, -1, 1, 1, -1, -1, 1, -1, -1, -1, 1, 1, -1, 1, 1, 1, 1, -1, 1, 1],
                         np.float32).reshape(8, 3)
    indices = np.array([0, 2, 1, 0, 3, 2, 4, 5, 6, 4, 6, 7, 0, 1, 5, 0, 5, 4, 3, 7, 6, 3, 6, 2, 0, 4, 7, 0, 7, 3,
                        1, 2, 6, 1, 6, 5], np.int64).reshape(12, 3)
    colors = np.array([1, 0, 0, 1, 0, 1, 0, 1, 0, 0, 1, 1, 1, 1, 0, 1, 1, 0, 1, 1, 0, 1, 1, 1, 1, 1, 1, 1,
                       .25, .5, .75, 1], np.float32).reshape(8, 4)
    model = g.multiply(g.rotation_y(np.float32(.55)), g.rotation_x(np.float32(.25)))
    view = g.look_at([3, 2, 4], [0, 0, 0], [0, 1, 0])
    projection = g.perspective(np.float32(1.04719755119659774615), 1, np.float32(.1), 100)
    return positions, indices, colors, model, view, projection


def test_renderer_cube_known_answer():
    """The reference's own cube digests and statistics (GraphicsTests.cpp:383-389)."""
    color, depth, stats = orc.render(*cube_scene(), 96, 96)
    assert stats.tolist() == [12, 12, 3150, 2218]
    assert orc.fnv_floats(color) == "fnv1a64:0d0c47343db9df53"
    assert orc.fnv_floats(depth) == "fnv1a64:4e244c6d47059a59"


@pytest.mark.parametrize("scene", ["random", "ties", "ortho"])
def test_renderer_matches_reference_scenes(golden, scene):
    """Scenes rendered by the reference's graphics::render: bit-exact colour
    and depth, equal statistics (clipping, overlap, equal-depth ties)."""
    k = lambda key: golden[f"gfx_{scene}_{key}"]
    color, depth, stats = orc.render(k("positions"), k("indices"), k("colors"), k("model").reshape(16),
                                     k("view").reshape(16), k("projection").reshape(16), int(k("width")),
                                     int(k("height")))
    assert stats.tolist() == k("stats").tolist()
    assert color.view(np.uint32).tolist() == k("color").view(np.uint32).tolist()
    assert depth.view(np.uint32).tolist() == k("depth").view(np.uint32).tolist()


def test_renderer_failure_ids():
    g = orc.gfx
    eye = g.identity()
    tri = np.zeros((3, 3), np.float32)
    with pytest.raises(orc.OracleFailure) as err:
        orc.render(tri, np.array([[0, 1, 3]]), np.zeros((3, 4), np.float32), eye, eye, eye, 4, 4)
    assert err.value.code == "TH019-INDEX"
    with pytest.raises(orc.OracleFailure) as err:
        orc.render(tri, np.array([[0, 1, 2]]), np.full((3, 4), 2, np.float32), eye, eye, eye, 4, 4)
    assert err.value.code == "TH019-COLOR-RANGE"
    with pytest.raises(orc.OracleFailure) as err:
        g.perspective(np.float32(0), 1, np.float32(.1), 100)
    assert err.value.code == "TH019-PROJECTION"


def _training_fixture_regions():
    """The reference's bounded training fixture (docs/spec/TRAINING_V0.md,
    "Determinism and fixture"): prediction = x * weight + bias, loss = the
    sum of squared errors, as a loss region and a region per parameter
    gradient. The gradient regions follow the reverse rules the reference's
    Autodiff.cpp emits for them: Mul -> cot*e + e*cot (2e with cot = 1),
    bias -> ReduceToShape, MatMul -> Transpose(x) . cot."""
    def forward(b):
        x = b.input(thb.F32, [4, 1])
        w = b.input(thb.F32, [1, 1])
        bias = b.input(thb.F32, [1])
        t = b.input(thb.F32, [4, 1])
        xw = b.matmul(x, w)
        e = b.sub(b.add(xw, b.broadcast_to_shape(bias, xw, 0)), t)
        return x, bias, e

    lb = thb.RegionBuilder("loss")
    _, _, e = forward(lb)
    loss = lb.build(lb.sum(lb.sum(lb.mul(e, e), 1), 0))
    gb = thb.RegionBuilder("dbias")
    _, bias, e = forward(gb)
    dbias = gb.build(gb.reduce_to_shape(gb.add(e, e), bias))
    gw = thb.RegionBuilder("dweight")
    x, _, e = forward(gw)
    dweight = gw.build(gw.matmul(gw.transpose(x), gw.add(e, e)))
    return loss, dbias, dweight


def test_training_fixture_known_answers():
    """Loss 84, dLoss/dbias = [-32], dLoss/dweight = [[-68]] at the initial
    state; one plain SGD step at lr 0.02 gives bias 0.64, weight 1.36; 200
    full-batch steps end within 0.001 of bias 1, weight 2 (the reference's
    predeclared convergence run)."""
    loss, dbias, dweight = _training_fixture_regions()
    x = np.array([[0], [1], [2], [3]], np.float32)
    t = np.array([[1], [3], [5], [7]], np.float32)
    p = np.zeros(2, np.float32)  # plan order [bias, weight]

    def state():
        return [x, p[1:2].reshape(1, 1).copy(), p[0:1].copy(), t]

    assert orc.region_eval(loss, state()) == 84.0
    g = np.array([orc.region_eval(dbias, state())[0], orc.region_eval(dweight, state())[0, 0]], np.float32)
    assert g.tolist() == [-32.0, -68.0]
    orc.sgd_update(p, g, 0.02)
    np.testing.assert_allclose(p, [0.64, 1.36], rtol=0, atol=1e-6)
    for _ in range(199):
        g = np.array([orc.region_eval(dbias, state())[0], orc.region_eval(dweight, state())[0, 0]], np.float32)
        orc.sgd_update(p, g, 0.02)
    np.testing.assert_allclose(p, [1.0, 2.0], rtol=0, atol=1e-3)


def _qualification_inputs(n):
    """The reference's deterministic qualification inputs
    (docs/spec/PERFORMANCE_QUALIFICATION_V0.md, "Deterministic inputs"):
    x[i] = f32((i*17) % 1009 - 504) / f32(37),
    y[i] = f32((i*29 + 11) % 1013 - 506) / f32(41)."""
    i = np.arange(n, dtype=np.int64)
    x = ((i * 17) % 1009 - 504).astype(np.float32) / np.float32(37)
    y = ((i * 29 + 11) % 1013 - 506).astype(np.float32) / np.float32(41)
    return x, y


def _qualification_chain():
    """Workload A: a = x + y; b = -a; c = b .* y; d = c - x; e = d .* y."""
    b = thb.RegionBuilder("elementwise_chain")
    x = b.input(thb.F32, [None])
    y = b.input(thb.F32, [None])
    c = b.mul(b.neg(b.add(x, y)), y)
    return b.build(b.mul(b.sub(c, x), y))


# Input and output digests the reference recorded for its fused CPU chain
# (benchmarks/results/TH-023-machine.json, elementwise_chain, thiran_fused).
@pytest.mark.parametrize("n,input_digest,output_digest", [
    (1 << 10, "fnv1a64:361d96caefeb88fd", "fnv1a64:61261595fdc3d150"),
    (1 << 20, "fnv1a64:f2764d4c05bf9a50", "fnv1a64:32dc138129eebb43"),
    (1 << 24, "fnv1a64:9c44e6d000b9f1cf", "fnv1a64:03e29fd051c79b66"),
])
def test_qualification_chain_digests(n, input_digest, output_digest):
    basis = 1469598103934665603
    x, y = _qualification_inputs(n)
    assert orc.fnv_floats(np.concatenate([x, y]), basis) == input_digest
    e = orc.region_eval(_qualification_chain(), [x, y])
    assert orc.fnv_floats(e, basis) == output_digest


def _qualification_extension(builtin):
    """Workload B: a = -x; b = research_square_linear(a) (a*a + a), or its
    built-in equivalent s = a .* a; b = s + a; then c = b + y."""
    b = thb.RegionBuilder("generic_extension")
    x = b.input(thb.F32, [None])
    y = b.input(thb.F32, [None])
    a = b.neg(x)
    sq = b.add(b.mul(a, a), a) if builtin else b.extension(regions.square_linear_operation(), a)
    return b.build(b.add(sq, y))


def _qualification_barrier():
    """Workload C: a = x + y; b = -a; c = a .* y; d = b + c; e = d - x
    (`a` has two consumers and materialises)."""
    b = thb.RegionBuilder("planned")
    x = b.input(thb.F32, [None])
    y = b.input(thb.F32, [None])
    a = b.add(x, y)
    d = b.add(b.neg(a), b.mul(a, y))
    return b.build(b.sub(d, x))


# Output digests the reference recorded at 2^20 for workloads B
# (generic_extension; its built-in equivalent must agree bit for bit) and C
# (thiran_planned), benchmarks/results/TH-023-machine.json.
@pytest.mark.parametrize("spec,output_digest", [
    (lambda: _qualification_extension(False), "fnv1a64:726e0e9b047863a9"),
    (lambda: _qualification_extension(True), "fnv1a64:726e0e9b047863a9"),
    (_qualification_barrier, "fnv1a64:eacc3ead55e92def"),
])
def test_qualification_workload_digests(spec, output_digest):
    x, y = _qualification_inputs(1 << 20)
    e = orc.region_eval(spec(), [x, y])
    assert orc.fnv_floats(e, 1469598103934665603) == output_digest


def _sum_i64_region(kind):
    b = thb.RegionBuilder("s")
    if kind == "total":
        x = b.input(thb.I64, [None])
        return b.build(b.sum(x, 0))
    x = b.input(thb.I64, [None, None])
    return b.build(b.sum(x, 1 if kind == "rows" else 0))


def test_sum_i64_checked_against_reference(golden, fixtures):
    m = golden["sum_i64_in"]
    for kind in ("rows", "cols"):
        np.testing.assert_array_equal(orc.region_eval(_sum_i64_region(kind), [m]), golden[f"sum_i64_{kind}"])
    assert orc.region_eval(_sum_i64_region("total"), [m.reshape(-1).copy()]) == int(golden["sum_i64_total"])
    edge = np.array([np.iinfo(np.int64).max, 1, -1], np.int64)
    for kind, value in (("total", edge), ("rows", edge.reshape(1, 3)), ("cols", edge.reshape(3, 1))):
        with pytest.raises(orc.OracleFailure) as err:
            orc.region_eval(_sum_i64_region(kind), [value])
        key = {"total": "sum_i64_prefix_overflow", "rows": "sum_i64_rows_prefix_overflow",
               "cols": "sum_i64_cols_prefix_overflow"}[kind]
        assert err.value.code == fixtures[key] == "TH-SPEC-I64-OVERFLOW"
