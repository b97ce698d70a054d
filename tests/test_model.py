"""`.thm` model bundles without a GPU: the reference's own bundle
(tests/golden/ref_research_model.thm, written by its createModelBundle /
writeModelBundle, src/model/v0/ModelBundle.cpp:328-360) loads and validates,
and malformed bundles are refused with the reference's MODEL-* ids
(loadModelBundle / validateModelBundle, :242-326, :362-430)."""
import os
import struct

import pytest

import thiran_b200 as thb

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
PATH = os.path.join(GOLDEN, "ref_research_model.thm")


def raw():
    with open(PATH, "rb") as f:
        return bytearray(f.read())


def refused(data, identity=None):
    with pytest.raises(thb.GpuError) as err:
        thb.Model.load(bytes(data), identity)
    assert err.value.status == thb.STATUS_ABI
    return err.value.code


def fnv(data):
    h = 1469598103934665603
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def reseal(data):
    """Recomputes the bundle's payload digest (header: magic, two u32, u64
    size, u64 digest)."""
    struct.pack_into("<Q", data, 24, fnv(data[32:]))
    return data


def test_reference_bundle_manifest():
    m = thb.Model.load(PATH).manifest
    assert m["model_identity"] == "research-model@1" and m["inference_entry"] == "f"
    assert [(p["id"], p["name"], p["shape"]) for p in m["parameters"]] == [(1, "p1", [96, 200]), (2, "p2", [96, 200])]
    assert m["public_abi"] == [{"kind": "tensor", "dtype": "f32", "rank": 2, "extents": [96, 200]}]
    assert m["result"] == m["public_abi"][0]
    assert m["backend_gpu"] and not m["backend_cpu"] and m["gpu_payload_kind"] == "ptx"
    assert thb.Model.load(raw()).manifest == m


def test_identity_check():
    assert thb.Model.load(PATH, "research-model@1").manifest["model_identity"] == "research-model@1"
    assert refused(raw(), "other-model@1") == "MODEL-IDENTITY"


def test_malformed_bundles():
    good = raw()
    bad = bytearray(good)
    bad[3] = ord("x")
    assert refused(bad) == "MODEL-MAGIC"
    bad = bytearray(good)
    struct.pack_into("<I", bad, 8, 3)
    assert refused(bad) == "MODEL-FORMAT-VERSION"
    bad = bytearray(good)
    struct.pack_into("<I", bad, 12, 2)
    assert refused(bad) == "MODEL-RUNTIME-ABI"
    assert refused(good + b"\0") == "MODEL-TRAILING-DATA"
    assert refused(good[:100]) == "MODEL-TRUNCATED"
    bad = bytearray(good)
    bad[-10] ^= 1
    assert refused(bad) == "MODEL-BUNDLE-INTEGRITY"


def test_frozen_parameter_tampering_is_refused():
    """A changed parameter byte under a valid bundle digest still fails the
    frozen-parameter digest (persistence::parameterDigest)."""
    data = raw()
    # payload: identity text, entry text, digest text, u32 count, then
    # parameter 1: u64 id, name text, kind, dtype, u32 rank, 2 x u64 shape,
    # u64 byte count, bytes.
    off = 32
    for _ in range(3):
        (n,) = struct.unpack_from("<Q", data, off)
        off += 8 + n
    off += 4 + 8
    (n,) = struct.unpack_from("<Q", data, off)
    off += 8 + n + 1 + 1 + 4 + 16 + 8
    data[off + 5] ^= 0x40
    assert refused(reseal(data)) == "MODEL-PARAMETER-DIGEST"


def test_engine_rejects_missing_file():
    with pytest.raises(thb.GpuError) as err:
        thb.Model.load(os.path.join(GOLDEN, "missing.thm"))
    assert err.value.code == "MODEL-IO"
