"""Renderer boundary without a GPU: invalid scenes fail with the reference's
TH019-* ids before any driver call (prepareRender runs on the host), and a
valid scene fails with GPU-DRIVER-NOT-FOUND: there is no CPU fallback."""
import numpy as np
import pytest

import oracle_lib as orc
import thiran_b200 as thb


def eye():
    return orc.gfx.identity()


TRI = np.array([[-.5, -.5, .5], [.5, -.5, .5], [0, .5, .5]], np.float32)
COLORS = np.ones((3, 4), np.float32)


@pytest.mark.parametrize("mutate,code", [
    (lambda s: s.update(indices=np.array([[0, 1, 3]])), "TH019-INDEX"),
    (lambda s: s.update(colors=np.full((3, 4), 1.5, np.float32)), "TH019-COLOR-RANGE"),
    (lambda s: s.update(positions=np.array([[np.inf, 0, 0], [1, 0, 0], [0, 1, 0]], np.float32)),
     "TH019-NONFINITE-VERTEX"),
    (lambda s: s.update(clear=(0, 0, 2, 0)), "TH019-CLEAR-COLOR"),
    (lambda s: s.update(model=np.full(16, np.nan, np.float32)), "TH019-NONFINITE-MATRIX"),
])
def test_invalid_scenes_fail_before_the_driver(mutate, code):
    scene = dict(positions=TRI, indices=np.array([[0, 1, 2]]), colors=COLORS, model=eye(), view=eye(),
                 projection=eye(), clear=(0, 0, 0, 0))
    mutate(scene)
    with pytest.raises(thb.GpuError) as err:
        thb.render(scene["positions"], scene["indices"], scene["colors"], scene["model"], scene["view"],
                   scene["projection"], 8, 8, scene["clear"])
    assert err.value.status == thb.STATUS_SEMANTIC and err.value.code == code


def test_valid_scene_has_no_cpu_fallback():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(thb.GpuError) as err:
        thb.render(TRI, np.array([[0, 1, 2]]), COLORS, eye(), eye(), eye(), 8, 8)
    assert err.value.code == "GPU-DRIVER-NOT-FOUND"
