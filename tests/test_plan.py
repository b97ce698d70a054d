"""Device-free planning and code generation (the reference's NativeGpuTests.cpp
checks: fusion structure, emission determinism, early rejection)."""
import re

import numpy as np
import pytest

import thiran_b200 as thb
from thiran_b200 import regions


def groups(spec, fusion=True):
    text, counts = spec.describe(thb.DESCRIBE_PLAN, fusion=fusion)
    out = []
    for line in text.splitlines():
        m = re.match(r"\s*group g\d+ nodes=(\S+)", line)
        if m:
            out.append([int(v[1:]) for v in m.group(1).split(",")])
    return out, counts


@pytest.mark.parametrize("name,builder,key", [
    ("kat_f32_chain", regions.f32_chain4, "kat_f32_chain"),
    ("i64_region", regions.i64_region, "i64_region"),
])
def test_fusion_groups_match_reference_planner(fixtures, name, builder, key):
    fused, counts = groups(builder(), fusion=True)
    assert fused == fixtures[key]["groups_fused"]
    assert counts[0] == 1 and counts[1] == 1
    unfused, counts = groups(builder(), fusion=False)
    assert unfused == fixtures[key]["groups_unfused"]
    assert counts[1] == 0


def test_chain_and_dynamic_groups_match_reference(fixtures):
    assert groups(regions.f32_chain())[0] == fixtures["chain"]["groups_fused"]
    assert groups(regions.i64_dynamic())[0] == fixtures["kat_i64_257"]["groups_fused"]


def test_slot_reuse_when_unfused():
    # Unfused chain C,D,E,F: two reusable temporaries, one reused
    # (NativeGpuIntegrationTests.cpp:126-137 expects 2 temporary slots, 1 reuse).
    text, _ = regions.f32_chain4().describe(thb.DESCRIBE_PLAN, fusion=False)
    temp_slots = [l for l in text.splitlines() if "slot s" in l and "external=no reusable=yes" in l]
    assert len(temp_slots) == 2
    assert any(l.count(",v") >= 1 for l in temp_slots)


def test_emission_is_deterministic_and_compiles_for_sm100a():
    spec = regions.i64_region()
    a, _ = spec.describe(thb.DESCRIBE_SOURCE)
    b, _ = regions.i64_region().describe(thb.DESCRIBE_SOURCE)
    assert a == b
    # No approximate or flush-to-zero arithmetic in generated code
    # (the reference audits its PTX the same way, NativeGpuTests.cpp:157-172).
    assert ".approx" not in a and "ftz" not in a.replace("--ftz=false", "")
    assert "thb_mul(" in a and "thb_add(" in a and "thb_sub(" in a
    size, _ = spec.describe(thb.DESCRIBE_CUBIN)
    assert int(size) > 0


def test_chain_source_uses_rounded_ops_in_ir_order():
    src, _ = regions.f32_chain().describe(thb.DESCRIBE_SOURCE)
    body = src[src.index("thb_g1_body"):]
    order = [m.group(1) for m in re.finditer(r"__f(add|sub|mul)_rn", body.split("extern")[0])]
    assert order == ["mul", "add", "mul", "sub", "mul", "add"]
    assert "__int_as_float(0x3fc00000)" in body  # 1.5f, bit-exact constant


def test_divide_recipe_sets_flag_and_is_not_fused():
    op = thb.Operation("ratio", [(thb.SCALAR_INPUT, 0, 0, 0, 0.0), (thb.SCALAR_INPUT, 0, 0, 1, 0.0),
                                 (thb.SCALAR_DIVIDE, 0, 1, 0, 0.0)], root=2, arity=2,
                       effect=thb.EFFECT_MAY_TRAP, fusible=False)
    b = thb.RegionBuilder("d")
    x = b.input(thb.F32, [None])
    y = b.input(thb.F32, [None])
    s = b.add(x, y)
    q = b.extension(op, s, y)
    spec = b.build(b.add(q, x))
    g, counts = groups(spec)
    assert g == [[3], [4], [5]]
    src, _ = spec.describe(thb.DESCRIBE_SOURCE)
    assert "thb_div(" in src
    assert int(spec.describe(thb.DESCRIBE_CUBIN)[0]) > 0


@pytest.mark.parametrize("mutate,code", [
    (lambda b: b.nodes[2].update(deps=[1, 99]), "TRV02"),
    (lambda b: b.nodes[2].update(dtype=thb.I64), "TRV05"),
    (lambda b: b.nodes[1].update(id=1), "TRV01"),
])
def test_malformed_regions_rejected_before_device(mutate, code):
    b = thb.RegionBuilder("bad")
    x = b.input(thb.F32, [4])
    y = b.input(thb.F32, [4])
    z = b.add(x, y)
    mutate(b)
    spec = b.build(z)
    with pytest.raises(thb.GpuError) as err:
        spec.describe(thb.DESCRIBE_PLAN)
    assert err.value.code == "GPU-INVALID-REGION" and code in err.value.message
    with pytest.raises(thb.GpuError) as err:
        spec.compile()
    assert err.value.code == "GPU-INVALID-REGION"


def _set_output(b, value):
    b.output = value


# The reference's manually built negative matrix over the region
# [2,2] i64: Input 1, Input 2, Add 3 (NativeCpuTests.cpp:198-221), one
# mutation per verifier rule.
@pytest.mark.parametrize("mutate,code", [
    (lambda b: b.nodes[1].update(id=1), "TRV01"),
    (lambda b: b.nodes[2].update(deps=[1, 99]), "TRV02"),
    (lambda b: b.nodes[2].update(deps=[1, 3]), "TRV03"),
    (lambda b: b.nodes[2].update(shape=[]), "TRV04"),
    (lambda b: b.nodes[1].update(shape=[2]), "TRV05"),
    (lambda b: b.nodes[1].update(shape=[2, 3]), "TRV06"),
    (lambda b: b.nodes[2].update(op=thb.OP_INDEX, deps=[1], indices=[]), "TRV07"),
    (lambda b: b.nodes[2].update(op=thb.OP_INDEX, deps=[1], indices=[1, 2]), "TRV08"),
    (lambda b: _set_output(b, 99), "TRV09"),
    (lambda b: b.nodes[2].update(op=thb.OP_UNSUPPORTED), "TRV10"),
])
def test_reference_negative_matrix(mutate, code):
    b = thb.RegionBuilder("manual")
    x = b.input(thb.I64, [2, 2])
    y = b.input(thb.I64, [2, 2])
    b.add(x, y)
    assert b.build(3).describe(thb.DESCRIBE_PLAN)[1][0] == 1  # the base verifies
    mutate(b)
    spec = b.build(b.output)
    with pytest.raises(thb.GpuError) as err:
        spec.describe(thb.DESCRIBE_PLAN)
    assert err.value.code == "GPU-INVALID-REGION" and code in err.value.message, err.value.message


def test_invalid_recipe_rejected():
    op = thb.Operation("bad", [(thb.SCALAR_INPUT, 0, 0, 0, 0.0), (thb.SCALAR_ADD, 0, 5, 0, 0.0)], root=1)
    b = thb.RegionBuilder("f")
    x = b.input(thb.F32, [None])
    spec = b.build(b.extension(op, x))
    with pytest.raises(thb.GpuError) as err:
        spec.describe(thb.DESCRIBE_PLAN)
    assert "TRV11" in err.value.message


def test_reductions_are_their_own_groups():
    b = thb.RegionBuilder("red")
    x = b.input(thb.F32, [None, None])
    r = b.relu(x)
    s = b.softmax(r)
    m = b.row_max(s)
    spec = b.build(m)
    g, counts = groups(spec)
    assert g == [[2], [3], [4]] and counts[2] == 3


def _engine_op_region(kind):
    """A well-formed one-op region over the engine's lowered operations
    (Sum, RowMax, Softmax, Transpose, MatMul, BroadcastToShape,
    ReduceToShape, ZeroLike) and its result id."""
    b = thb.RegionBuilder(kind)
    a = b.input(thb.F32, [4, 6])
    if kind == "sum":
        r = b.sum(a, 1)
    elif kind == "row_max":
        r = b.row_max(a)
    elif kind == "softmax":
        r = b.softmax(a)
    elif kind == "transpose":
        r = b.transpose(a)
    elif kind == "matmul":
        r = b.matmul(a, b.input(thb.F32, [6, 3]))
    elif kind == "broadcast":
        r = b.broadcast_to_shape(b.input(thb.F32, [6]), a, 0)
    elif kind == "reduce":
        r = b.reduce_to_shape(a, b.input(thb.F32, [4, 1]))
    else:
        r = b.zero_like(a)
    return b, r


# One malformed variant per engine operation: each breaks the operation's
# type or extent rule (axis range, rank, inner dimension, dtype).
@pytest.mark.parametrize("kind,mutate", [
    ("sum", lambda n: n.update(axis=2)),
    ("sum", lambda n: n.update(shape=[5])),
    ("row_max", lambda n: n.update(axis=0)),
    ("softmax", lambda n: n.update(axis=0)),
    ("transpose", lambda n: n.update(shape=[4, 6])),
    ("matmul", lambda n: n.update(shape=[4, 4])),
    ("matmul", lambda n: n.update(axis=2)),                 # no such f32 mode
    ("matmul", lambda n: n.update(dtype=thb.I64)),          # i64 result of f32 operands
    ("broadcast", lambda n: n.update(axis=2)),
    ("reduce", lambda n: n.update(shape=[4])),
    ("zero_like", lambda n: n.update(dtype=thb.I64)),
])
def test_engine_operations_negative_matrix(kind, mutate):
    b, r = _engine_op_region(kind)
    assert b.build(r).describe(thb.DESCRIBE_PLAN)[1][0] >= 1  # the well-formed region verifies
    mutate(b.nodes[r - 1])
    with pytest.raises(thb.GpuError) as err:
        b.build(r).describe(thb.DESCRIBE_PLAN)
    assert err.value.code == "GPU-INVALID-REGION" and "TRV12" in err.value.message, err.value.message


def test_matmul_inner_dimension_mismatch_rejected():
    b = thb.RegionBuilder("mm")
    x = b.input(thb.F32, [4, 6])
    w = b.input(thb.F32, [5, 3])
    with pytest.raises(thb.GpuError) as err:
        b.build(b.matmul(x, w)).describe(thb.DESCRIBE_PLAN)
    assert "TRV12 malformed MatMul" in err.value.message


def test_matmul_i64_and_exact_modes_verify():
    for dtype, exact in ((thb.I64, False), (thb.F32, True), (thb.F32, False)):
        spec = regions.matmul(dtype, exact)
        assert spec.describe(thb.DESCRIBE_PLAN)[1][0] >= 1
    b = thb.RegionBuilder("mm")
    x = b.input(thb.I64, [4, 6])
    w = b.input(thb.F32, [6, 3])
    with pytest.raises(thb.GpuError) as err:
        b.build(b.matmul(x, w)).describe(thb.DESCRIBE_PLAN)
    assert "TRV12 malformed MatMul" in err.value.message
