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
