"""Standard TensorRegions of the benchmark workloads.

Each builder reproduces, node for node, the region the reference's
extractStrictRegion (src/backend/v0/TensorRegion.cpp:230-447) produces for the
corresponding V0 source, including the Alias node every `let` binding and
parameter use introduces, so node ids and fusion groups can be compared with
the reference planner's output directly.
"""
from __future__ import annotations

from . import (F32, I64, RegionBuilder, Operation, SCALAR_ADD, SCALAR_MULTIPLY, SCALAR_SUBTRACT,
               recipe_from_expression)

# ((x*1.5 + 0.25)*x - x)*0.5 + x as one V0 extension scalar recipe: the form
# in which the reference runs this chain natively (a ConstantF32 recipe; the
# literal scalar-broadcast source is rejected by its native extractor).
CHAIN_RECIPE = recipe_from_expression([
    ("x", 0),                      # 0 x
    ("c", 1.5),                    # 1
    (SCALAR_MULTIPLY, 0, 1),       # 2 x*1.5
    ("c", 0.25),                   # 3
    (SCALAR_ADD, 2, 3),            # 4 +0.25
    (SCALAR_MULTIPLY, 4, 0),       # 5 *x
    (SCALAR_SUBTRACT, 5, 0),       # 6 -x
    ("c", 0.5),                    # 7
    (SCALAR_MULTIPLY, 6, 7),       # 8 *0.5
    (SCALAR_ADD, 8, 0),            # 9 +x
])


# d/dx of the chain over (x, y, dz): dz * ((((x*1.5 + 0.25) + x*1.5) - 1) * 0.5 + 1)
CHAIN_GRADIENT = recipe_from_expression([
    ("x", 0),                      # 0 x
    ("c", 1.5),                    # 1
    (SCALAR_MULTIPLY, 0, 1),       # 2 x*1.5
    ("c", 0.25),                   # 3
    (SCALAR_ADD, 2, 3),            # 4 x*1.5+0.25
    (SCALAR_ADD, 4, 2),            # 5 + x*1.5
    ("c", 1.0),                    # 6
    (SCALAR_SUBTRACT, 5, 6),       # 7 - 1
    ("c", 0.5),                    # 8
    (SCALAR_MULTIPLY, 7, 8),       # 9 * 0.5
    (SCALAR_ADD, 9, 6),            # 10 + 1
    ("x", 2),                      # 11 dz
    (SCALAR_MULTIPLY, 11, 10),     # 12 dz * (...)
])

# examples/research_extension: x*x + x, gradient dz * (2x + 1).
SQUARE_LINEAR_RECIPE = recipe_from_expression([("x", 0), (SCALAR_MULTIPLY, 0, 0), (SCALAR_ADD, 1, 0)])
SQUARE_LINEAR_GRADIENT = recipe_from_expression([
    ("x", 2), ("c", 2.0), ("x", 0), (SCALAR_MULTIPLY, 1, 2), ("c", 1.0), (SCALAR_ADD, 3, 4), (SCALAR_MULTIPLY, 0, 5),
])


def chain_operation() -> Operation:
    return Operation("research_chain", CHAIN_RECIPE, root=9, arity=1, gradients=[(CHAIN_GRADIENT, 12)])


def square_linear_operation() -> Operation:
    return Operation("research_square_linear", SQUARE_LINEAR_RECIPE, root=2, arity=1,
                     gradients=[(SQUARE_LINEAR_GRADIENT, 6)])


def extension_gradient(operation: Operation, n=None):
    """Backward of y = op(x): dx = gradient recipe over (x, y, dz)."""
    b = RegionBuilder("grad")
    x = b.input(F32, [n])
    dz = b.input(F32, [n])
    y = b.extension(operation, b.alias(x))
    return b.build(b.extension_gradient(operation, 0, b.alias(x), y, b.alias(dz)))


def linear_loss_backward(output="dw1"):
    """The reverse-mode backward the reference generates for
        fn loss(x, w1, w2, t) -> f32 { h = x*w1; y = h*w2; e = y - t; s = e.*e;
                                        return sum(sum(s,1),0) }
    (src/autodiff/v0/Autodiff.cpp:195-231), with the forward values it saves
    recomputed in the same region. `output` selects dx, dw1, dw2 or dt."""
    b = RegionBuilder("loss_backward")
    x = b.input(F32, [None, None])
    w1 = b.input(F32, [None, None])
    w2 = b.input(F32, [None, None])
    t = b.input(F32, [None, None])
    ct = b.input(F32, [])
    h = b.matmul(x, w1)
    y = b.matmul(h, w2)
    e = b.sub(y, t)
    s = b.mul(e, e)
    rows = b.sum(s, 1)
    d16 = b.broadcast_to_shape(ct, rows, 0)
    d17 = b.broadcast_to_shape(d16, s, 1)
    d19 = b.reduce_to_shape(b.mul(d17, e), e)
    d21 = b.reduce_to_shape(b.mul(d17, e), e)
    d22 = b.add(d21, d19)
    dy = b.reduce_to_shape(d22, y)
    dt = b.neg(b.reduce_to_shape(d22, t))
    dh = b.matmul(dy, b.transpose(w2))
    dw2 = b.matmul(b.transpose(h), dy)
    dx = b.matmul(dh, b.transpose(w1))
    dw1 = b.matmul(b.transpose(x), dh)
    return b.build({"dx": dx, "dw1": dw1, "dw2": dw2, "dt": dt}[output])


def linear_bias_loss_backward(output="dw1"):
    """The reverse-mode backward the reference generates for the biased
    two-layer loss (the examples/mlp.th structure without the ReLU, which the
    V0 language lacks)
        fn loss(x, w1, b1: Tensor<f32,1>, w2, b2: Tensor<f32,1>, t) -> f32 {
            h = x*w1 + b1; y = h*w2 + b2; e = y - t; s = e.*e;
            return sum(sum(s,1),0) }
    Broadcast adds (Evaluator.cpp:95-124) run as BroadcastToShape + Add; the
    bias gradients are ReduceToShape onto the bias (Evaluator.cpp:258-277).
    `output` selects dx, dw1, db1, dw2, db2 or dt."""
    b = RegionBuilder("loss_backward")
    x = b.input(F32, [None, None])
    w1 = b.input(F32, [None, None])
    b1 = b.input(F32, [None])
    w2 = b.input(F32, [None, None])
    b2 = b.input(F32, [None])
    t = b.input(F32, [None, None])
    ct = b.input(F32, [])
    xw1 = b.matmul(x, w1)
    h = b.add(xw1, b.broadcast_to_shape(b1, xw1, 0))
    hw2 = b.matmul(h, w2)
    y = b.add(hw2, b.broadcast_to_shape(b2, hw2, 0))
    e = b.sub(y, t)
    s = b.mul(e, e)
    rows = b.sum(s, 1)
    d1 = b.broadcast_to_shape(ct, rows, 0)
    d2 = b.broadcast_to_shape(d1, s, 1)
    de = b.add(b.reduce_to_shape(b.mul(d2, e), e), b.reduce_to_shape(b.mul(d2, e), e))
    dy = b.reduce_to_shape(de, y)
    dt = b.neg(b.reduce_to_shape(de, t))
    dhw2 = b.reduce_to_shape(dy, hw2)
    db2 = b.reduce_to_shape(dy, b2)
    dh = b.matmul(dhw2, b.transpose(w2))
    dw2 = b.matmul(b.transpose(h), dhw2)
    dxw1 = b.reduce_to_shape(dh, xw1)
    db1 = b.reduce_to_shape(dh, b1)
    dx = b.matmul(dxw1, b.transpose(w1))
    dw1 = b.matmul(b.transpose(x), dxw1)
    return b.build({"dx": dx, "dw1": dw1, "db1": db1, "dw2": dw2, "db2": db2, "dt": dt}[output])


def f32_chain(n=None):
    """fn f(x: Tensor<f32,1>) -> Tensor<f32,1> { return research_chain(x) }"""
    b = RegionBuilder("f")
    x = b.input(F32, [n])
    xa = b.alias(x)
    y = b.extension(chain_operation(), xa)
    return b.build(y)


def f32_chain_literal(n=None):
    """fn f(x: Tensor<f32,1>) -> Tensor<f32,1> { return ((x*1.5+0.25).*x - x)*0.5 + x }
    in its literal form: scalar constants broadcast inside the chain. The
    reference runs this only in its Evaluator (its native extractor rejects
    tensor-scalar operands); here it is one fused kernel with the constants
    compiled in."""
    b = RegionBuilder("f")
    x = b.input(F32, [n])
    t = b.mul(b.alias(x), b.float(1.5))
    t = b.add(t, b.float(0.25))
    t = b.mul(t, b.alias(x))
    t = b.sub(t, b.alias(x))
    t = b.mul(t, b.float(0.5))
    t = b.add(t, b.alias(x))
    return b.build(t)


def i64_region(rows=None, cols=None):
    """fn f(a,b: Tensor<i64,2>) { let s = a + b; let m = s .* a; return m - b }"""
    b = RegionBuilder("f")
    a = b.input(I64, [rows, cols])
    c = b.input(I64, [rows, cols])
    s = b.add(b.alias(a), b.alias(c))
    m = b.mul(b.alias(s), b.alias(a))
    o = b.sub(b.alias(m), b.alias(c))
    return b.build(o)


def f32_chain4(n=None):
    """The reference GPU integration chain: C=A+B; D=C.*B; E=D-A; return E+B."""
    b = RegionBuilder("f")
    A = b.input(F32, [n])
    B = b.input(F32, [n])
    C = b.add(b.alias(A), b.alias(B))
    D = b.mul(b.alias(C), b.alias(B))
    E = b.sub(b.alias(D), b.alias(A))
    F = b.add(b.alias(E), b.alias(B))
    return b.build(F)


def i64_dynamic(n=None):
    """fn f(x,y: Tensor<i64,1>) { let z=x+y; return z.*y }"""
    b = RegionBuilder("f")
    x = b.input(I64, [n])
    y = b.input(I64, [n])
    z = b.add(b.alias(x), b.alias(y))
    r = b.mul(b.alias(z), b.alias(y))
    return b.build(r)


def softmax_rows(rows=None, cols=None):
    """Row-wise softmax over the last axis (engine-side op)."""
    b = RegionBuilder("softmax")
    x = b.input(F32, [rows, cols])
    return b.build(b.softmax(x))


def full_sum(n=None):
    """Full-tensor sum of a flattened tensor: sum(x, 0) -> f32."""
    b = RegionBuilder("total")
    x = b.input(F32, [n])
    return b.build(b.sum(x, 0))


def matmul(dtype=F32, exact=False):
    """fn mm(A: Tensor<T,2>, B: Tensor<T,2>) -> Tensor<T,2> { return A * B }
    (the reference runs this only in its Evaluator, Evaluator.cpp:125-154).
    f32: tensor cores (bf16 operands), or with `exact` the Evaluator's
    sequential f32 sums; i64: checked multiply and add."""
    b = RegionBuilder("mm")
    x = b.input(dtype, [None, None])
    y = b.input(dtype, [None, None])
    return b.build(b.matmul(b.alias(x), b.alias(y), exact=exact))


def transformer_block(exact=True):
    """examples/transformer.th: one attention block on X [2,4] with Wq, Wk
    [4,4], Wv [4,8] and Wo [8,4] (inputs in that order):
        Q = X Wq; K = X Wk; Scores = Q K^T; Attention = softmax(Scores);
        V = X Wv; Context = Attention V; O = Context Wo + X
    The legacy stack lowers MatMul / Transpose / Softmax / Add to torch
    (src/backend/PythonExecutorEmitter.cpp:87-97); here every node is an
    engine op, the matmuls exact (or on the tensor cores)."""
    b = RegionBuilder("transformer")
    x = b.input(F32, [None, None])
    wq = b.input(F32, [None, None])
    wk = b.input(F32, [None, None])
    wv = b.input(F32, [None, None])
    wo = b.input(F32, [None, None])
    q = b.matmul(x, wq, exact=exact)
    k = b.matmul(x, wk, exact=exact)
    scores = b.matmul(q, b.transpose(k), exact=exact)
    attention = b.softmax(scores)
    v = b.matmul(x, wv, exact=exact)
    context = b.matmul(attention, v, exact=exact)
    projected = b.matmul(context, wo, exact=exact)
    return b.build(b.add(projected, x))
