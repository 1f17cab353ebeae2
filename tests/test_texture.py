"""Texture known-answer tests and gradchecks, restated from the reference's
Tests/MLXDiffRastTests/TextureTests.swift, on the oracle and the CUDA path."""
import numpy as np
import pytest

from helpers import fd_grad, wsum

T22 = np.array([10, 20, 30, 40], np.float32).reshape(1, 2, 2, 1)


def test_forward_texel_centers(backend):
    # TextureTests.swift:11-28
    uv = np.array([[0.25, 0.25], [0.75, 0.25], [0.25, 0.75], [0.75, 0.75]], np.float32).reshape(1, 2, 2, 2)
    out = backend.texture(T22, uv)
    assert out.reshape(-1).tolist() == [10, 20, 30, 40]


def test_forward_center_is_mean(backend):
    # TextureTests.swift:30-39
    out = backend.texture(T22, np.array([0.5, 0.5], np.float32).reshape(1, 1, 1, 2))
    assert abs(out.item() - 25) < 1e-5


def test_boundary_zero(backend):
    # TextureTests.swift:41-46
    out = backend.texture(np.ones((1, 2, 2, 1), np.float32), np.array([5.0, 5.0], np.float32).reshape(1, 1, 1, 2),
                          boundary_mode="zero")
    assert abs(out.item()) < 1e-6


def test_boundary_clamp(backend):
    # TextureTests.swift:49-58
    out = backend.texture(T22, np.array([10.0, 10.0], np.float32).reshape(1, 1, 1, 2), boundary_mode="clamp")
    assert abs(out.item() - 40) < 1e-6


def test_boundary_wrap_periodic(backend):
    # TextureTests.swift:61-71
    a = backend.texture(T22, np.array([0.4, 0.6], np.float32).reshape(1, 1, 1, 2), boundary_mode="wrap")
    b = backend.texture(T22, np.array([1.4, 0.6], np.float32).reshape(1, 1, 1, 2), boundary_mode="wrap")
    assert abs(a.item() - b.item()) < 1e-5


def test_cube_face_selection(backend):
    # TextureTests.swift:78-101
    tex = np.array([10, 20, 30, 40, 50, 60], np.float32).reshape(1, 6, 1, 1, 1)
    d = np.array([[1, 0, 0], [-1, 0, 0], [0, 1, 0], [0, -1, 0], [0, 0, 1], [0, 0, -1]], np.float32)
    out = backend.texture(tex, d.reshape(1, 1, 6, 3), boundary_mode="cube")
    assert out.shape == (1, 1, 6, 1)
    assert out.reshape(-1).tolist() == [10, 20, 30, 40, 50, 60]


def test_cube_gradient_picks_one_face(backend):
    # TextureTests.swift:104-113
    tex = np.zeros((1, 6, 1, 1, 1), np.float32)
    d = np.array([0, 1, 0], np.float32).reshape(1, 1, 1, 3)
    d_tex, d_dir, _, _ = backend.texture_bwd(tex, d, np.ones((1, 1, 1, 1), np.float32), boundary_mode="cube")
    assert d_tex.reshape(-1).tolist() == [0, 0, 1, 0, 0, 0]
    assert np.all(d_dir == 0)


@pytest.mark.parametrize("perturb,boundary", [("tex", "wrap"), ("uv", "wrap"), ("tex", "clamp"), ("uv", "zero")])
def test_gradcheck_bilinear(backend, perturb, boundary):
    # TextureTests.swift:117-131, 385-438
    N, Hi, Wi, Ht, Wt, C = 1, 2, 2, 3, 3, 2
    tex = np.random.default_rng(0x7E27).normal(size=(N, Ht, Wt, C)).astype(np.float32)
    uv = np.array([[0.25 + 0.3 * pw, 0.30 + 0.25 * ph] for ph in range(Hi) for pw in range(Wi)],
                  np.float32).reshape(N, Hi, Wi, 2)
    w = np.array([(1 + i % 5) * 0.1 for i in range(N * Hi * Wi * C)], np.float32).reshape(N, Hi, Wi, C)
    d_tex, d_uv, _, _ = backend.texture_bwd(tex, uv, w, boundary_mode=boundary)
    if perturb == "tex":
        num = fd_grad(lambda x: wsum(backend.texture(x, uv, boundary_mode=boundary), w), tex)
        np.testing.assert_allclose(d_tex, num, atol=5e-3)
    else:
        num = fd_grad(lambda x: wsum(backend.texture(tex, x, boundary_mode=boundary), w), uv)
        np.testing.assert_allclose(d_uv, num, atol=5e-3)


def test_construct_mip_shapes(backend):
    # TextureTests.swift:137-151
    tex = np.arange(16, dtype=np.float32).reshape(1, 4, 4, 1)
    lv = backend.construct_mip(tex)
    assert [x.shape for x in lv] == [(1, 4, 4, 1), (1, 2, 2, 1), (1, 1, 1, 1)]
    assert abs(lv[1].reshape(-1)[0] - 2.5) < 1e-6
    assert abs(lv[2].item() - 7.5) < 1e-6


def test_construct_mip_max_level(backend):
    # TextureTests.swift:153-161
    lv = backend.construct_mip(np.zeros((1, 8, 8, 1), np.float32), max_level=2)
    assert [x.shape for x in lv] == [(1, 8, 8, 1), (1, 4, 4, 1), (1, 2, 2, 1)]


def test_construct_mip_odd_dims_stop(backend):
    lv = backend.construct_mip(np.zeros((1, 12, 8, 2), np.float32))
    assert [x.shape[1:3] for x in lv] == [(12, 8), (6, 4), (3, 2)]


TEX42 = (np.arange(32, dtype=np.float32) * 0.05).reshape(1, 4, 4, 2)
UV1 = np.array([0.42, 0.31], np.float32).reshape(1, 1, 1, 2)


def test_trilinear_matches_bilinear_at_lod0(backend):
    # TextureTests.swift:167-182
    da = np.full((1, 1, 1, 4), 1e-6, np.float32)
    b = backend.texture(TEX42, UV1)
    t = backend.texture(TEX42, UV1, da, filter_mode="linear-mipmap-linear")
    np.testing.assert_allclose(b, t, atol=1e-4)


def test_trilinear_at_max_lod_yields_global_mean(backend):
    # TextureTests.swift:187-196
    out = backend.texture(np.ones((1, 4, 4, 1), np.float32), np.array([0.5, 0.5], np.float32).reshape(1, 1, 1, 2),
                          np.full((1, 1, 1, 4), 100.0, np.float32), filter_mode="linear-mipmap-linear")
    assert abs(out.item() - 1) < 1e-6


def _tri_fixture():
    # TextureTests.swift:317-379
    N, Hi, Wi, Ht, Wt, C = 1, 2, 2, 4, 4, 2
    tex = np.random.default_rng(0x71117EAB).normal(size=(N, Ht, Wt, C)).astype(np.float32)
    uv = np.array([[0.32 + 0.27 * pw, 0.41 + 0.23 * ph] for ph in range(Hi) for pw in range(Wi)],
                  np.float32).reshape(N, Hi, Wi, 2)
    da = np.array([0.4 + 0.05 * (i % 3) for i in range(N * Hi * Wi * 4)], np.float32).reshape(N, Hi, Wi, 4)
    w = np.array([(1 + i % 5) * 0.1 for i in range(N * Hi * Wi * C)], np.float32).reshape(N, Hi, Wi, C)
    return tex, uv, da, w


@pytest.mark.parametrize("perturb", ["tex", "uv", "uvDA"])
def test_gradcheck_trilinear(backend, perturb):
    # TextureTests.swift:200-209, tolerance 8e-3 as the reference
    tex, uv, da, w = _tri_fixture()
    f = "linear-mipmap-linear"
    d_tex, d_uv, d_da, _ = backend.texture_bwd(tex, uv, w, da, filter_mode=f)
    if perturb == "tex":
        num = fd_grad(lambda x: wsum(backend.texture(x, uv, da, filter_mode=f), w), tex)
        np.testing.assert_allclose(d_tex, num, atol=8e-3)
    elif perturb == "uv":
        num = fd_grad(lambda x: wsum(backend.texture(tex, x, da, filter_mode=f), w), uv)
        np.testing.assert_allclose(d_uv, num, atol=8e-3)
    else:
        num = fd_grad(lambda x: wsum(backend.texture(tex, uv, x, filter_mode=f), w), da)
        np.testing.assert_allclose(d_da, num, atol=8e-3)


def test_gradcheck_bias_map(backend):
    # The bias map reaches the loss through uvDA * 2^map; its gradient is the
    # adjoint of that multiply (MLX autograd of Texture.swift:110-121).
    tex, uv, da, w = _tri_fixture()
    bmap = np.array([0.1, -0.2, 0.15, -0.05], np.float32).reshape(1, 2, 2)
    f = "linear-mipmap-linear"
    _, _, _, d_map = backend.texture_bwd(tex, uv, w, da, filter_mode=f, bias_map=bmap)
    num = fd_grad(lambda x: wsum(backend.texture(tex, uv, da, filter_mode=f, bias_map=x), w), bmap)
    np.testing.assert_allclose(d_map, num, atol=8e-3)


def test_nearest_exact_texel_lookup(backend):
    # TextureTests.swift:215-225
    out = backend.texture(T22, np.array([0.3, 0.7], np.float32).reshape(1, 1, 1, 2), filter_mode="nearest")
    assert abs(out.item() - 30) < 1e-6


def test_nearest_gradient(backend):
    # TextureTests.swift:228-244
    uv = np.array([0.3, 0.7], np.float32).reshape(1, 1, 1, 2)
    d_tex, d_uv, _, _ = backend.texture_bwd(T22, uv, np.ones((1, 1, 1, 1), np.float32), filter_mode="nearest")
    assert d_tex.reshape(-1).tolist() == [0, 0, 1, 0]
    assert d_uv.reshape(-1).tolist() == [0, 0]


def test_mipmap_nearest_matches_trilinear_at_integer_lod(backend):
    # TextureTests.swift:251-268
    da = np.array([0.5, 0.0, 0.0, 0.5], np.float32).reshape(1, 1, 1, 4)
    t = backend.texture(TEX42, UV1, da, filter_mode="linear-mipmap-linear")
    n = backend.texture(TEX42, UV1, da, filter_mode="linear-mipmap-nearest")
    np.testing.assert_allclose(t, n, atol=1e-5)


def test_per_pixel_bias_map_matches_scaled_uvda(backend):
    # TextureTests.swift:272-293
    uv = np.tile(np.array([0.42, 0.31], np.float32), (1, 2, 2, 1))
    da = np.tile(np.array([0.3, 0.1, 0.1, 0.3], np.float32), (1, 2, 2, 1))
    bmap = np.array([0.5, -0.3, 1.0, -1.0], np.float32).reshape(1, 2, 2)
    b = backend.texture(TEX42, uv, da, filter_mode="linear-mipmap-linear", bias_map=bmap)
    s = backend.texture(TEX42, uv, (da * (2.0 ** bmap)[..., None]).astype(np.float32),
                        filter_mode="linear-mipmap-linear")
    np.testing.assert_allclose(b, s, atol=1e-5)


def test_mip_level_bias_is_equivalent_to_scaled_uvda(backend):
    # TextureTests.swift:298-315
    da = np.array([0.3, 0.1, 0.1, 0.3], np.float32).reshape(1, 1, 1, 4)
    b = backend.texture(TEX42, UV1, da, filter_mode="linear-mipmap-linear", bias=1.0)
    s = backend.texture(TEX42, UV1, da * 2, filter_mode="linear-mipmap-linear")
    np.testing.assert_allclose(b, s, atol=1e-5)


def test_batch1_texture_gradient_sums_over_views(backend):
    g = np.random.default_rng(3)
    tex = g.normal(size=(1, 8, 8, 3)).astype(np.float32)
    uv = g.uniform(0, 1, size=(3, 4, 4, 2)).astype(np.float32)
    d = g.normal(size=(3, 4, 4, 3)).astype(np.float32)
    d1, _, _, _ = backend.texture_bwd(tex, uv, d, boundary_mode="clamp")
    d3, _, _, _ = backend.texture_bwd(np.repeat(tex, 3, 0), uv, d, boundary_mode="clamp")
    np.testing.assert_allclose(d1[0], d3.sum(0), atol=1e-5)


# ---- mip-mapped cube textures (extension: the reference's cube path samples
# level 0 with filterMode .linear only).  The LOD comes from the derivatives of
# the face coordinates, obtained from the direction's screen-space derivatives
# dirDA = [dx/dX, dx/dY, dy/dX, dy/dY, dz/dX, dz/dY] through the cube
# projection u = (sc / ma + 1) / 2.

def _cube_fixture(seed=0xC0BE, Ht=8, C=2):
    g = np.random.default_rng(seed)
    tex = g.normal(size=(1, 6, Ht, Ht, C)).astype(np.float32)
    d = np.array([[0.9, 0.2, -0.3], [-0.8, 0.35, 0.13], [0.15, 1.1, -0.4], [0.3, -0.7, 0.2],
                  [-0.25, 0.3, 0.95], [0.2, -0.1, -1.2]], np.float32).reshape(1, 2, 3, 3)
    dd = g.uniform(0.35, 0.7, size=(1, 2, 3, 6)).astype(np.float32)
    w = np.array([(1 + i % 5) * 0.1 for i in range(6 * C)], np.float32).reshape(1, 2, 3, C)
    return tex, d, dd, w


def test_cube_mip_matches_cube_linear_at_lod0(backend):
    tex, d, _, _ = _cube_fixture()
    dd = np.full((1, 2, 3, 6), 1e-6, np.float32)
    lin = backend.texture(tex, d, boundary_mode="cube")
    for f in ("linear-mipmap-linear", "linear-mipmap-nearest"):
        mip = backend.texture(tex, d, dd, filter_mode=f, boundary_mode="cube")
        assert np.array_equal(lin, mip), f


def test_cube_mip_constant_faces_any_lod(backend):
    tex = np.broadcast_to(np.arange(1, 7, dtype=np.float32).reshape(1, 6, 1, 1, 1), (1, 6, 8, 8, 1)).copy()
    _, d, dd, _ = _cube_fixture()
    for scale in (0.01, 1.0, 100.0):
        out = backend.texture(tex, d, dd * scale, filter_mode="linear-mipmap-linear", boundary_mode="cube")
        np.testing.assert_allclose(out.reshape(-1), [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], rtol=1e-6)


@pytest.mark.parametrize("f", ["linear-mipmap-linear", "linear-mipmap-nearest"])
def test_cube_mip_pz_face_equals_2d_mip(backend, f):
    # On +Z with z = 1 and dz = 0: u = (x + 1) / 2, v = (1 - y) / 2, so the
    # cube sample is the 2D clamp-mode sample of face 4 with
    # uvDA = (dx/dX, dx/dY, -dy/dX, -dy/dY) / 2 — bit for bit.
    tex, _, _, w = _cube_fixture()
    g = np.random.default_rng(5)
    xy = g.uniform(-0.9, 0.9, size=(1, 3, 4, 2)).astype(np.float32)
    d = np.concatenate([xy, np.ones((1, 3, 4, 1), np.float32)], -1)
    dxy = g.uniform(0.05, 0.8, size=(1, 3, 4, 4)).astype(np.float32)
    dd = np.concatenate([dxy, np.zeros((1, 3, 4, 2), np.float32)], -1)
    uv = np.stack([(xy[..., 0] + 1.0) * 0.5, (-xy[..., 1] + 1.0) * 0.5], -1).astype(np.float32)
    uv_da = np.stack([0.5 * dxy[..., 0], 0.5 * dxy[..., 1], -0.5 * dxy[..., 2], -0.5 * dxy[..., 3]],
                     -1).astype(np.float32)
    face = np.ascontiguousarray(tex[:, 4])
    cube = backend.texture(tex, d, dd, filter_mode=f, boundary_mode="cube")
    flat = backend.texture(face, uv, uv_da, filter_mode=f, boundary_mode="clamp")
    assert np.array_equal(cube, flat)
    wc = np.resize(w, cube.shape).astype(np.float32)
    dt_c, d_dir, d_dd, _ = backend.texture_bwd(tex, d, wc, dd, filter_mode=f, boundary_mode="cube")
    dt_f, _, d_uvda, _ = backend.texture_bwd(face, uv, wc, uv_da, filter_mode=f, boundary_mode="clamp")
    np.testing.assert_allclose(dt_c[:, 4], dt_f, rtol=1e-5, atol=1e-6)
    assert np.all(np.delete(dt_c, 4, axis=1) == 0)
    assert np.all(d_dir == 0)
    np.testing.assert_allclose(d_dd[..., 0], 0.5 * d_uvda[..., 0], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(d_dd[..., 1], 0.5 * d_uvda[..., 1], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(d_dd[..., 2], -0.5 * d_uvda[..., 2], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(d_dd[..., 3], -0.5 * d_uvda[..., 3], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("perturb", ["tex", "dirDA"])
def test_gradcheck_cube_trilinear(backend, perturb):
    tex, d, dd, w = _cube_fixture()
    f = "linear-mipmap-linear"
    d_tex, d_dir, d_dd, _ = backend.texture_bwd(tex, d, w, dd, filter_mode=f, boundary_mode="cube")
    assert d_dd.shape == dd.shape and np.all(d_dir == 0)
    if perturb == "tex":
        num = fd_grad(lambda x: wsum(backend.texture(x, d, dd, filter_mode=f, boundary_mode="cube"), w), tex)
        np.testing.assert_allclose(d_tex, num, atol=8e-3)
    else:
        num = fd_grad(lambda x: wsum(backend.texture(tex, d, x, filter_mode=f, boundary_mode="cube"), w), dd)
        assert np.abs(num).max() > 1e-2  # the fixture's LODs are interior
        np.testing.assert_allclose(d_dd, num, atol=8e-3)


def test_gradcheck_cube_bias_map(backend):
    tex, d, dd, w = _cube_fixture()
    bmap = np.array([0.1, -0.2, 0.15, -0.05, 0.3, -0.1], np.float32).reshape(1, 2, 3)
    f = "linear-mipmap-linear"
    _, _, _, d_map = backend.texture_bwd(tex, d, w, dd, filter_mode=f, boundary_mode="cube", bias_map=bmap)
    num = fd_grad(lambda x: wsum(backend.texture(tex, d, dd, filter_mode=f, boundary_mode="cube", bias_map=x),
                                 w), bmap)
    np.testing.assert_allclose(d_map, num, atol=8e-3)


# ---- d_dir through the cube projection (extension: the reference's cube VJP
# returns d_dir = 0, Texture.swift:196-197; opt-in with cube_dir_grad).

@pytest.mark.parametrize("f", ["linear", "linear-mipmap-linear"])
def test_gradcheck_cube_dir(backend, f):
    tex, d, dd, w = _cube_fixture()
    mip = f != "linear"
    da = dd if mip else None
    _, d_dir0, _, _ = backend.texture_bwd(tex, d, w, da, filter_mode=f, boundary_mode="cube")
    assert np.all(d_dir0 == 0)  # the reference's behaviour stays the default
    _, d_dir, _, _ = backend.texture_bwd(tex, d, w, da, filter_mode=f, boundary_mode="cube", cube_dir_grad=True)
    num = fd_grad(lambda x: wsum(backend.texture(tex, x, da, filter_mode=f, boundary_mode="cube"), w), d)
    assert np.abs(num).max() > 1e-1
    np.testing.assert_allclose(d_dir, num, atol=8e-3)


def test_cube_dir_grad_pz_face_matches_uv_grad(backend):
    # On +Z with z = 1: u = (x + 1) / 2, v = (1 - y) / 2, so d_x = d_u / 2,
    # d_y = -d_v / 2 and d_z = -(x d_u - y d_v) / 2 (d_u, d_v from the 2D path).
    tex, _, _, _ = _cube_fixture()
    g = np.random.default_rng(9)
    xy = g.uniform(-0.9, 0.9, size=(1, 3, 4, 2)).astype(np.float32)
    d = np.concatenate([xy, np.ones((1, 3, 4, 1), np.float32)], -1)
    uv = np.stack([(xy[..., 0] + 1.0) * 0.5, (-xy[..., 1] + 1.0) * 0.5], -1).astype(np.float32)
    w = g.normal(size=(1, 3, 4, 2)).astype(np.float32)
    face = np.ascontiguousarray(tex[:, 4])
    _, d_dir, _, _ = backend.texture_bwd(tex, d, w, boundary_mode="cube", cube_dir_grad=True)
    _, d_uv, _, _ = backend.texture_bwd(face, uv, w, boundary_mode="clamp")
    np.testing.assert_allclose(d_dir[..., 0], 0.5 * d_uv[..., 0], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(d_dir[..., 1], -0.5 * d_uv[..., 1], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(d_dir[..., 2], -0.5 * (xy[..., 0] * d_uv[..., 0] - xy[..., 1] * d_uv[..., 1]),
                               rtol=1e-4, atol=1e-5)
