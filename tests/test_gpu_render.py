"""GPU renderer parity: the reference's cube known answer (colour and depth
FNV digests, all four statistics; GraphicsTests.cpp:383-389), scenes the
reference itself rendered (bit-exact), and large random scenes against the
oracle renderer (pinned to the reference)."""
import numpy as np
import pytest

import oracle_lib as orc
import thiran_b200 as thb
from test_oracle import cube_scene

pytestmark = pytest.mark.gpu


def test_cube_known_answer(device):
    scene = cube_scene()
    color, depth, stats = thb.render(*scene, 96, 96, device=device)
    assert stats.tolist() == [12, 12, 3150, 2218]
    assert orc.fnv_floats(color) == "fnv1a64:0d0c47343db9df53"
    assert orc.fnv_floats(depth) == "fnv1a64:4e244c6d47059a59"
    # The raw geometry crosses PCIe (positions, colours, indices); transform,
    # clipping, setup and binning run as kernels before the raster kernel.
    positions, indices, colors = scene[0], scene[1], scene[2]
    ev = thb.render.evidence
    assert ev["host_to_device_bytes"] == positions.size * 4 + colors.size * 4 + indices.size * 8
    assert ev["kernel_launches"] > 1


def test_transform_failure_on_the_device(device):
    """A vertex whose transformed coordinate overflows f32 fails with the
    reference's TH019-NONFINITE-TRANSFORMED (found by the transform kernel)."""
    g = orc.gfx
    positions = np.array([[3e38, 0, 0], [0, 1, 0], [1, 0, 0]], np.float32)
    scale = np.diag(np.array([10, 10, 10, 1], np.float32)).astype(np.float32)
    eye = g.identity()
    with pytest.raises(thb.GpuError) as err:
        thb.render(positions, np.array([[0, 1, 2]]), np.full((3, 4), 0.5, np.float32), scale, eye, eye, 8, 8,
                   device=device)
    assert err.value.code == "TH019-NONFINITE-TRANSFORMED"


@pytest.mark.parametrize("scene", ["random", "ties", "ortho"])
def test_reference_scenes(device, golden, scene):
    k = lambda key: golden[f"gfx_{scene}_{key}"]
    color, depth, stats = thb.render(k("positions"), k("indices"), k("colors"), k("model"), k("view"),
                                     k("projection"), int(k("width")), int(k("height")), device=device)
    assert stats.tolist() == k("stats").tolist()
    assert color.view(np.uint32).tolist() == k("color").view(np.uint32).tolist()
    assert depth.view(np.uint32).tolist() == k("depth").view(np.uint32).tolist()


@pytest.mark.parametrize("triangles,width,height,seed", [(5000, 640, 360, 1), (20000, 333, 257, 2)])
def test_random_scene_matches_oracle(device, triangles, width, height, seed):
    """Many small and large triangles, partly outside the frustum, with a
    non-zero clear colour; ragged tiles at the right and bottom edges."""
    g = orc.gfx
    rng = np.random.default_rng(seed)
    centers = rng.uniform(-2, 2, (triangles, 1, 3)).astype(np.float32)
    positions = (centers + rng.normal(0, 0.15, (triangles, 3, 3))).astype(np.float32).reshape(-1, 3)
    colors = rng.uniform(0, 1, (triangles * 3, 4)).astype(np.float32)
    indices = np.arange(triangles * 3, dtype=np.int64).reshape(-1, 3)
    model = g.rotation_y(np.float32(0.7))
    view = g.look_at([0.3, 0.8, 4.5], [0, 0, 0], [0, 1, 0])
    projection = g.perspective(np.float32(1.0), np.float32(width / height), np.float32(0.2), np.float32(30))
    clear = (0.1, 0.2, 0.3, 1.0)
    ref = orc.render(positions, indices, colors, model, view, projection, width, height, clear)
    got = thb.render(positions, indices, colors, model, view, projection, width, height, clear, device=device)
    assert got[2].tolist() == ref[2].tolist()
    assert np.array_equal(got[0].view(np.uint32), ref[0].view(np.uint32))
    assert np.array_equal(got[1].view(np.uint32), ref[1].view(np.uint32))


def test_empty_scene_and_framebuffer(device):
    eye = orc.gfx.identity()
    color, depth, stats = thb.render(np.zeros((0, 3), np.float32), np.zeros((0, 3), np.int64),
                                     np.zeros((0, 4), np.float32), eye, eye, eye, 7, 5, (0.5, 0, 0, 1), device=device)
    assert stats.tolist() == [0, 0, 0, 0]
    assert np.all(color == np.array([0.5, 0, 0, 1], np.float32)) and np.all(np.isinf(depth))
    color, depth, stats = thb.render(np.zeros((0, 3), np.float32), np.zeros((0, 3), np.int64),
                                     np.zeros((0, 4), np.float32), eye, eye, eye, 0, 0, device=device)
    assert color.shape == (0, 4) and depth.shape == (0,)
