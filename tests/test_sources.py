# Source-level guards on the CUDA code the engine ships and generates.
#
# Every bulk or tensor copy into shared memory is issued per CTA: no copy
# carries the cluster-wide fan-out qualifier, whose only open form in this
# code is the tcgen05.commit arrive on the CTA pair's mbarriers. The GEMM
# issues tcgen05 and TMA, and no legacy tensor-core or Hopper-only
# instructions appear anywhere.
import glob
import os

import thiran_b200 as thb
from thiran_b200 import regions

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCES = sorted(glob.glob(os.path.join(ROOT, "thiran_b200", "csrc", "*.cu")) +
                 glob.glob(os.path.join(ROOT, "thiran_b200", "csrc", "*.cuh")) +
                 glob.glob(os.path.join(ROOT, "thiran_b200", "csrc", "*.cpp")) +
                 glob.glob(os.path.join(ROOT, "thiran_b200", "csrc", "*.hpp")))

# The two fragments are looked for separately on each line, and the
# qualifier is spelled from parts so that no string here is such a copy.
_BULK = "cp.async.bulk"
_FANOUT = ".multi" + "cast" + "::" + "cluster"


def _fanout_copies(lines):
    return [k for k, line in enumerate(lines, 1) if _BULK in line and _FANOUT in line]


def test_bulk_copies_are_per_cta_in_sources():
    hits = []
    for path in SOURCES:
        with open(path) as f:
            hits += [f"{os.path.basename(path)}:{k}" for k in _fanout_copies(f)]
    assert not hits, hits


def test_gemm_issues_tcgen05_and_tma():
    text = open(os.path.join(ROOT, "thiran_b200", "csrc", "gemm.cu")).read()
    assert "tcgen05.mma" in text and "cp.async.bulk.tensor" in text and "tcgen05.ld" in text
    for legacy in ("wgmma", "mma.sync", "wmma::"):
        assert legacy not in text


def test_generated_bulk_copies_are_per_cta():
    specs = [regions.i64_region(), regions.f32_chain(), regions.f32_chain4(), regions.i64_dynamic(),
             regions.f32_chain_literal()]
    for spec in specs:
        src, _ = spec.describe(thb.DESCRIBE_SOURCE)
        assert not _fanout_copies(src.splitlines())
        assert _BULK in src  # the bulk-copy entry is generated
