"""Rasterize known-answer tests and gradchecks, restated from the reference's
Tests/MLXDiffRastTests/RasterizeTests.swift, on the oracle and the CUDA path."""
import numpy as np
import pytest

from helpers import fd_grad, wsum

CORNER = np.array([[[-1, 1, 0, 1], [-1, -1, 0, 1], [1, 1, 0, 1]]], np.float32)
TRI1 = np.array([[0, 1, 2]], np.int32)


def test_single_triangle_covers_image(backend):
    # RasterizeTests.swift:11-52
    rast, _ = backend.rasterize(CORNER, TRI1, (2, 2), grad_db=False)
    assert rast.shape == (1, 2, 2, 4)
    f = rast.reshape(-1)
    np.testing.assert_allclose(f[:4], [0.25, 0.25, 0.0, 1.0], atol=1e-5)
    assert f[(0 * 2 + 1) * 4 + 3] == 1.0  # on edge -> inside
    assert f[(1 * 2 + 0) * 4 + 3] == 1.0
    assert f[(1 * 2 + 1) * 4 + 3] == 0.0  # outside -> empty


def test_depth_test_picks_front_triangle(backend):
    # RasterizeTests.swift:54-86
    pos = np.array([[[-1, 1, .5, 1], [-1, -1, .5, 1], [1, 1, .5, 1],
                     [-1, 1, -.5, 1], [-1, -1, -.5, 1], [1, 1, -.5, 1]]], np.float32)
    tri = np.array([[0, 1, 2], [3, 4, 5]], np.int32)
    rast, _ = backend.rasterize(pos, tri, (2, 2), grad_db=False)
    for px in rast.reshape(-1, 4):
        if px[3] == 0:
            continue
        assert abs(px[2] + 0.5) < 1e-5 and px[3] == 2.0


def test_pixels_outside_triangle_are_zero(backend):
    # RasterizeTests.swift:89-106
    pos = np.array([[[-1, 1, 0, 1], [-.5, 1, 0, 1], [-1, .5, 0, 1]]], np.float32)
    rast, _ = backend.rasterize(pos, TRI1, (4, 4), grad_db=False)
    assert np.all(rast[0, 3, 3] == 0)


def test_rast_db_analytic(backend):
    # RasterizeTests.swift:119-146
    _, db = backend.rasterize(CORNER, TRI1, (2, 2))
    f = db.reshape(-1, 4)
    for p in (0, 1, 2):
        np.testing.assert_allclose(f[p], [0.0, 0.5, 0.5, 0.0], atol=1e-5)
    np.testing.assert_allclose(f[3], 0.0, atol=1e-5)


def test_rasterize_into_interpolate_da(backend):
    # RasterizeTests.swift:148-171
    rast, db = backend.rasterize(CORNER, TRI1, (2, 2))
    attr = np.array([[[0.0], [2.0], [4.0]]], np.float32)
    _, oda = backend.interpolate(attr, rast, TRI1, rast_db=db, diff_attrs="all")
    assert oda.shape == (1, 2, 2, 2)
    np.testing.assert_allclose(oda.reshape(-1)[:2], [2.0, 1.0], atol=1e-5)


def _full_cover_pos():
    # RasterizeTests.swift:173-187: edges > 0.5 NDC from every pixel centre.
    return np.array([[[-3, 3, 0.0, 1], [-3, -3, 0.1, 1], [3, 0, -0.1, 1]]], np.float32)


@pytest.mark.parametrize("use_db", [False, True])
def test_gradcheck_rasterize(backend, use_db):
    # RasterizeTests.swift:189-238
    N, H, W = 1, 2, 2
    w_r = np.array([0.0 if i % 4 == 3 else (1 + i % 7) * 0.1 for i in range(N * H * W * 4)],
                   np.float32).reshape(N, H, W, 4)
    w_db = np.array([(2 + i % 5) * 0.05 if use_db else 0.0 for i in range(N * H * W * 4)],
                    np.float32).reshape(N, H, W, 4)
    pos0 = _full_cover_pos()

    def loss(p):
        r, db = backend.rasterize(p, TRI1, (H, W), grad_db=use_db)
        return wsum(r, w_r) + (wsum(db, w_db) if use_db else 0.0)

    analytic = backend.rasterize_bwd(pos0, TRI1, (H, W), w_r, w_db if use_db else None)
    numeric = fd_grad(loss, pos0)
    np.testing.assert_allclose(analytic, numeric, atol=5e-3)


def test_peel_layer_exposes_next_depth(backend):
    # RasterizeTests.swift:253-310
    pos = np.array([[[-2, 2, -.5, 1], [-2, -2, -.5, 1], [2, 2, -.5, 1],
                     [-2, 2, .5, 1], [-2, -2, .5, 1], [2, 2, .5, 1]]], np.float32)
    tri = np.array([[0, 1, 2], [3, 4, 5]], np.int32)
    l0, _ = backend.rasterize(pos, tri, (2, 2), grad_db=False)
    for px in l0.reshape(-1, 4):
        if px[3]:
            assert abs(px[2] + 0.5) < 1e-5 and px[3] == 1.0
    l1, _ = backend.rasterize(pos, tri, (2, 2), grad_db=False, peel=l0)
    for px in l1.reshape(-1, 4):
        if px[3]:
            assert abs(px[2] - 0.5) < 1e-5 and px[3] == 2.0
    l2, _ = backend.rasterize(pos, tri, (2, 2), grad_db=False, peel=l1)
    assert np.all(l2[..., 3] == 0)


def test_range_mode_selects_per_batch_triangles(backend):
    # RasterizeTests.swift:312-362
    pos = np.array([[-1, 1, 0, 1], [-1, -1, 0, 1], [1, 1, 0, 1],
                    [1, 1, .5, 1], [-1, -1, .5, 1], [1, -1, .5, 1]], np.float32)
    tri = np.array([[0, 1, 2], [3, 4, 5]], np.int32)
    ranges = np.array([[0, 1], [1, 1]], np.int32)
    rast, _ = backend.rasterize(pos, tri, (2, 2), grad_db=False, ranges=ranges)
    assert rast.shape == (2, 2, 2, 4)
    assert set(np.unique(rast[0, ..., 3])) <= {0.0, 1.0}
    assert set(np.unique(rast[1, ..., 3])) <= {0.0, 2.0}
    assert (rast[0, ..., 3] == 1).any() and (rast[1, ..., 3] == 2).any()


def test_rasterize_into_interpolate_partition_of_unity(backend):
    # RasterizeTests.swift:364-394
    rast, _ = backend.rasterize(CORNER, TRI1, (2, 2), grad_db=False)
    attr = np.eye(3, dtype=np.float32)[None]
    out, _ = backend.interpolate(attr, rast, TRI1)
    s = out.reshape(-1, 3).sum(1)
    cov = rast.reshape(-1, 4)[:, 3] > 0
    np.testing.assert_allclose(s, np.where(cov, 1.0, 0.0), atol=1e-5)


# ---- edge cases beyond the reference's tests --------------------------------

def test_empty_triangle_list(backend):
    pos = CORNER
    tri = np.zeros((0, 3), np.int32)
    rast, db = backend.rasterize(pos, tri, (5, 7))
    assert rast.shape == (1, 5, 7, 4) and np.all(rast == 0) and np.all(db == 0)


def test_w_nonpositive_and_z_out_of_range_rejected(backend):
    pos = np.array([[[-1, 1, 0, 1], [-1, -1, 0, -1], [1, 1, 0, 1],        # w <= 0 -> culled
                     [-1, 1, 1.5, 1], [-1, -1, 1.5, 1], [1, 1, 1.5, 1]]], np.float32)  # z > 1
    tri = np.array([[0, 1, 2], [3, 4, 5]], np.int32)
    rast, _ = backend.rasterize(pos, tri, (4, 4), grad_db=False)
    assert np.all(rast == 0)


def test_depth_tie_resolves_to_lowest_index(backend):
    # Two identical triangles: the reference's ascending strict-< loop keeps the first.
    pos = np.concatenate([CORNER, CORNER], 1)
    tri = np.array([[3, 4, 5], [0, 1, 2]], np.int32)
    rast, _ = backend.rasterize(pos, tri, (8, 8), grad_db=False)
    ids = rast[..., 3]
    assert set(np.unique(ids)) <= {0.0, 1.0} and (ids == 1).any()


def test_no_triangle_dropped_in_a_dense_tile(backend):
    # 300 nested triangles in one 16x16 tile (the reference's bins keep 128).
    # The front-most one is the LAST in index order and must win.
    n = 300
    verts, tris = [], []
    for i in range(n):
        z = 0.9 - 1.8 * i / n
        verts += [[-0.9, 0.9, z, 1], [-0.9, 0.8, z, 1], [-0.8, 0.9, z, 1]]
        tris.append([3 * i, 3 * i + 1, 3 * i + 2])
    pos = np.array([verts], np.float32)
    tri = np.array(tris, np.int32)
    rast, _ = backend.rasterize(pos, tri, (64, 64), grad_db=False)
    ids = rast[..., 3]
    assert ids.max() == float(n)
    covered = ids > 0
    assert np.all(ids[covered] == n)


def _sliver_scene(sliver_first):
    # A sliver with a finite, non-zero area of 2^-129: 1/area = inf, so at the
    # pixels of row 2 of a 5-row image (centre y = 0 exactly) its barycentrics
    # are inf or 0 * inf = NaN and its depth is NaN.  The reference would store
    # that NaN (every comparison is false) and let its next candidate replace
    # it; this library and its oracle never take a NaN depth, so the full-screen
    # triangle at z = 0.5 wins everywhere whatever the order.
    tiny = np.float32(2.0 ** -130)
    sliver = [[-1, 0, -0.5, 1], [1, 0, -0.5, 1], [1, tiny, -0.5, 1]]
    full = [[-4, -4, 0.5, 1], [4, -4, 0.5, 1], [0, 4, 0.5, 1]]
    verts = sliver + full if sliver_first else full + sliver
    pos = np.array([verts], np.float32)
    tri = np.array([[0, 1, 2], [3, 4, 5]], np.int32)
    return pos, tri, (2.0 if sliver_first else 1.0)


def test_subnormal_area_sliver_never_wins(backend):
    pos, tri, full_id = _sliver_scene(True)
    rast, db = backend.rasterize(pos[:, :3], tri[:1], (5, 8))
    assert np.all(rast == 0) and np.all(db == 0)  # alone: no fragment, no NaN
    for first in (True, False):
        pos, tri, full_id = _sliver_scene(first)
        rast, db = backend.rasterize(pos, tri, (5, 8))
        assert np.all(np.isfinite(rast)) and np.all(np.isfinite(db))
        assert np.all(rast[..., 3] == full_id), first
        assert np.all(rast[..., 2] == np.float32(0.5))
