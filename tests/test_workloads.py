"""The synthetic workloads match the configurations they stand for
(BASELINE.json configs[0..4] = cfg1..cfg5): mesh sizes, view counts,
resolutions, texture shapes and value ranges.  CPU only."""
import numpy as np

from diffrast import scenes


def test_cfg1_single_triangle():
    s = scenes.scene_cfg1()
    want = np.array([[[-0.8, -0.8, 0, 1], [0.8, -0.8, 0, 1], [0, 0.8, 0, 1]]], np.float32)
    assert s["pos"].dtype == np.float32 and np.array_equal(s["pos"], want)
    assert s["tri"].tolist() == [[0, 1, 2]] and s["res"] == (256, 256)
    assert s["attr"].shape == (3, 3) and 0 <= s["attr"].min() and s["attr"].max() <= 1


def test_cfg2_cfg3_icosphere_level4():
    s = scenes.scene_cfg2()
    assert s["pos"].shape == (8, 2562, 4) and s["tri"].shape == (5120, 3) and s["res"] == (512, 512)
    assert s["tex"].shape == (1, 512, 512, 3)
    s = scenes.scene_cfg3(n_views=2)
    assert s["tex"].shape == (1, 2048, 2048, 4) and s["res"] == (1024, 1024)
    assert -1 <= s["bias_map"].min() and s["bias_map"].max() <= 1


def test_cfg4_million_triangle_soup():
    s = scenes.scene_cfg4(n_views=2)
    tri = s["tri"]
    assert tri.shape == (1_000_000, 3) and s["attr"].shape[1] == 8 and s["res"] == (1024, 1024)
    # 20% of the triangles share edges in strips: vertices shared by > 1 triangle
    uses = np.bincount(tri.reshape(-1), minlength=s["base"].shape[0])
    shared_tris = np.any(uses[tri] > 1, axis=1).sum()
    assert abs(shared_tris / tri.shape[0] - 0.2) < 0.01
    assert s["sim"].shape == (2, 4, 4)


def test_cfg5_geodesic_sphere_f158():
    s = scenes.scene_cfg5(n_views=2, res=64, cube=8)
    assert s["tri"].shape == (20 * 158 ** 2, 3) and s["verts"].shape == (10 * 158 ** 2 + 2, 3)
    assert s["cube"].shape == (1, 6, 8, 8, 3) and s["mvps"].shape == (2, 4, 4)
