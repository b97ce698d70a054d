"""Source-level guards on the CUDA code the engine ships and generates: no
TMA or bulk load with cluster multicast (peer memory must never be read that
way), and no legacy tensor-core or Hopper-only instructions."""
import glob
import os
import re

import thiran_b200 as thb
from thiran_b200 import regions

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCES = sorted(glob.glob(os.path.join(ROOT, "thiran_b200", "csrc", "*.cu")) +
                 glob.glob(os.path.join(ROOT, "thiran_b200", "csrc", "*.cuh")) +
                 glob.glob(os.path.join(ROOT, "thiran_b200", "csrc", "*.cpp")) +
                 glob.glob(os.path.join(ROOT, "thiran_b200", "csrc", "*.hpp")))

# Assembled from parts so that this file itself names no such instruction.
_BULK = "cp" + r"\.async\.bulk"
_CLUSTER_CAST = "multi" + "cast" + "::" + "cluster"
MULTICAST_LOAD = re.compile(_BULK + "[^\"]*" + _CLUSTER_CAST)


def test_no_multicast_bulk_loads_in_sources():
    # The guard recognises such a load (a string built here, never compiled).
    assert MULTICAST_LOAD.search("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes."
                                 + _CLUSTER_CAST)
    hits = []
    for path in SOURCES:
        for k, line in enumerate(open(path), 1):
            if MULTICAST_LOAD.search(line):
                hits.append(f"{os.path.basename(path)}:{k}")
    assert not hits, hits


def test_gemm_issues_tcgen05_and_tma():
    text = open(os.path.join(ROOT, "thiran_b200", "csrc", "gemm.cu")).read()
    assert "tcgen05.mma" in text and "cp.async.bulk.tensor" in text and "tcgen05.ld" in text
    for legacy in ("wgmma", "mma.sync", "wmma::"):
        assert legacy not in text


def test_generated_sources_have_no_multicast_loads():
    specs = [regions.i64_region(), regions.f32_chain(), regions.f32_chain4(), regions.i64_dynamic(),
             regions.f32_chain_literal()]
    for spec in specs:
        src, _ = spec.describe(thb.DESCRIBE_SOURCE)
        assert not MULTICAST_LOAD.search(src)
        assert "cp.async.bulk" in src  # the bulk-copy entry is generated
