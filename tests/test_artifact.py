"""`.tha` artifacts without a GPU: the reference's own GPU artifacts
(tests/golden/ref_*.tha, written by its buildGpuAot,
src/artifact/v0/NativeArtifacts.cpp:1056-1097) load and plan like the
reference planner; every malformed form is refused with the reference's
failure id (validateArtifact / loadArtifactBytes, :574-630, :1100-1140); and
this engine's own artifacts (payload kind 3) round-trip."""
import os
import struct

import pytest

import thiran_b200 as thb
from thiran_b200 import regions

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def ref(name):
    with open(os.path.join(GOLDEN, name), "rb") as f:
        return f.read()


def refused(data):
    with pytest.raises(thb.GpuError) as err:
        thb.Artifact.load(bytes(data))
    assert err.value.status == thb.STATUS_ABI
    return err.value.code


@pytest.mark.parametrize("name,dtype,rank,inputs", [("ref_f32_chain.tha", "f32", 1, 1),
                                                    ("ref_i64_region.tha", "i64", 2, 2)])
def test_reference_gpu_artifact_manifest(name, dtype, rank, inputs):
    m = thb.Artifact.load(os.path.join(GOLDEN, name)).manifest
    assert m["backend"] == "gpu" and m["payload_kind"] == "ptx"
    assert m["target"] == "ptx60-sm50-min-cc50"
    assert m["runtime_requirement"] == "native-runtime-abi=1;libcuda.so.1;driver-ptx-jit;min-cc=5.0"
    assert m["entry"] == "f"
    assert len(m["parameters"]) == inputs
    for p in m["parameters"] + [m["result"]]:
        assert p == {"kind": "tensor", "dtype": dtype, "rank": rank, "extents": [None] * rank}
    assert m["region_size"] > 0 and m["payload_size"] > 0


def test_reference_artifact_plans_like_the_reference_planner(fixtures):
    """The i64 region (a+b).*a-b: the reference's planner fuses its three
    elementwise nodes into one group, or keeps three without fusion
    (fixtures from its buildPhysicalPlan); the artifact's region plans the
    same way here."""
    fused = thb.Artifact.load(os.path.join(GOLDEN, "ref_i64_region.tha")).manifest
    unfused = thb.Artifact.load(os.path.join(GOLDEN, "ref_i64_region_nofusion.tha")).manifest
    assert unfused["enable_fusion"] is False
    assert fused["fusion_groups"] == len(fixtures["i64_region"]["groups_fused"])
    assert unfused["fusion_groups"] == len(fixtures["i64_region"]["groups_unfused"])
    chain = thb.Artifact.load(os.path.join(GOLDEN, "ref_f32_chain.tha")).manifest
    assert chain["fusion_groups"] == 1
    assert "research_chain" in chain["region"]


def test_file_and_bytes_load_agree():
    a = thb.Artifact.load(os.path.join(GOLDEN, "ref_f32_chain.tha")).manifest
    b = thb.Artifact.load(ref("ref_f32_chain.tha")).manifest
    assert a == b


def test_missing_file():
    with pytest.raises(thb.GpuError) as err:
        thb.Artifact.load(os.path.join(GOLDEN, "no_such.tha"))
    assert err.value.code == "ARTIFACT-IO"


# Byte offsets of the fixed manifest fields (serializeArtifact,
# NativeArtifacts.cpp:547-556): magic 0..7, three u32 versions, then backend,
# payload kind, reuse, fusion, then the target text.
BACKEND, PAYLOAD_KIND = 20, 21


def text_at(data, offset):
    (n,) = struct.unpack_from("<Q", data, offset)
    return offset + 8, n


def test_malformed_forms_are_refused_with_reference_ids():
    good = bytearray(ref("ref_i64_region.tha"))
    bad = bytearray(good)
    bad[0] = ord("X")
    assert refused(bad) == "ARTIFACT-MAGIC"
    assert refused(good[:64]) == "ARTIFACT-TRUNCATED"
    assert refused(good + b"\0") == "ARTIFACT-TRAILING-DATA"
    bad = bytearray(good)
    struct.pack_into("<I", bad, 8, 7)
    assert refused(bad) == "ARTIFACT-FORMAT-VERSION"
    bad = bytearray(good)
    struct.pack_into("<I", bad, 12, 2)
    assert refused(bad) == "ARTIFACT-COMPILER-ABI"
    bad = bytearray(good)
    struct.pack_into("<I", bad, 16, 9)
    assert refused(bad) == "ARTIFACT-RUNTIME-ABI"
    bad = bytearray(good)
    bad[BACKEND] = 1
    assert refused(bad) == "ARTIFACT-BACKEND"
    bad = bytearray(good)
    bad[PAYLOAD_KIND] = 1
    assert refused(bad) == "ARTIFACT-PAYLOAD-KIND"
    bad = bytearray(good)
    start, n = text_at(bad, 24)
    bad[start] ^= 0x20  # target text
    assert refused(bad) == "ARTIFACT-TARGET"
    bad = bytearray(good)
    start, n = text_at(bad, start + n)
    bad[start + 3] ^= 0x20  # runtime requirement text
    assert refused(bad) == "ARTIFACT-RUNTIME-REQUIREMENT"
    bad = bytearray(good)
    bad[-1] ^= 0x01  # last payload byte
    assert refused(bad) == "ARTIFACT-PAYLOAD-INTEGRITY"


def region_offset(data):
    """Offset of the serialized region: the end of the manifest."""
    off = 24
    for _ in range(3):  # target, runtime requirement, entry name
        off, n = text_at(data, off)
        off += n
    (count,) = struct.unpack_from("<I", data, off)
    off += 4

    def skip_type(o):
        o += 1 + 1 + 4
        (extents,) = struct.unpack_from("<I", data, o)
        o += 4
        for _ in range(extents):
            present = data[o]
            o += 1 + (8 if present else 0)
        return o

    for _ in range(count + 1):
        off = skip_type(off)
    off, n = text_at(data, off)  # plan digest
    off += n
    off += 8  # region size
    off, n = text_at(data, off)  # region digest
    off += n
    off += 8  # payload size
    off, n = text_at(data, off)  # payload digest
    return off + n


def test_region_tampering_is_refused():
    good = ref("ref_f32_chain.tha")
    bad = bytearray(good)
    bad[region_offset(good) + 6] ^= 0x01  # inside the region name
    assert refused(bad) == "ARTIFACT-REGION-INTEGRITY"


def test_engine_artifact_round_trip():
    spec = regions.f32_chain()
    data = thb.build_artifact(spec)
    m = thb.Artifact.load(data).manifest
    assert m["payload_kind"] == "b200-cubin" and m["target"] == "sm_100a"
    assert m["runtime_requirement"] == "thiran-b200-runtime-abi=1;libcudart;sm_100a"
    assert m["fusion_groups"] == spec.describe()[1][0]
    assert data[:8] == b"THIRAN16"
    bad = bytearray(data)
    bad[-100] ^= 0x01  # inside the cubin
    assert refused(bad) == "ARTIFACT-PAYLOAD-INTEGRITY"


@pytest.mark.parametrize("builder", [regions.softmax_rows, regions.full_sum, regions.i64_region])
def test_engine_artifacts_of_engine_regions(builder):
    """Engine-only ops (softmax, sums) travel in kind-3 artifacts, with the
    axis in the node's integer field, and plan the same after loading."""
    spec = builder()
    m = thb.Artifact.load(thb.build_artifact(spec)).manifest
    assert m["fusion_groups"] == spec.describe()[1][0]


def test_engine_only_ops_are_refused_in_reference_artifacts():
    """A reference-kind artifact whose region carries an engine op number
    fails region validation (the reference's RegionOp stops at 12)."""
    good = ref("ref_f32_chain.tha")
    off = region_offset(good)
    # region: function u32, name text, node count u32, then node 0: id u32, op u8.
    off += 4
    off, n = text_at(good, off)
    off += n + 4 + 4
    bad = bytearray(good)
    bad[off] = thb.OP_SOFTMAX
    code = refused(bad)
    assert code in ("ARTIFACT-REGION-INTEGRITY", "ARTIFACT-REGION")
