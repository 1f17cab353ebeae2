"""Interpolate known-answer tests and gradchecks, restated from the reference's
Tests/MLXDiffRastTests/InterpolateTests.swift, on the oracle and the CUDA path.
The reference draws gradcheck inputs from MLXRandom (not reproducible here);
the structure, sizes and tolerances are kept with seeded numpy normals."""
import numpy as np
import pytest

from helpers import fd_grad, wsum

TRI1 = np.array([[0, 1, 2]], np.int32)


def test_forward_constant_barys(backend):
    # InterpolateTests.swift:11-38
    attr = np.array([[[i, i + 1, i + 2] for i in range(3)]], np.float32)
    rast = np.tile(np.array([0.25, 0.5, 0.0, 1.0], np.float32), (1, 2, 2, 1))
    out, oda = backend.interpolate(attr, rast, TRI1)
    assert out.shape == (1, 2, 2, 3) and oda.shape == (1, 2, 2, 0)
    np.testing.assert_allclose(out.reshape(-1, 3), np.tile([1.25, 2.25, 3.25], (4, 1)), atol=1e-5)


def test_empty_pixels_are_zero(backend):
    # InterpolateTests.swift:40-55
    attr = np.ones((1, 3, 2), np.float32)
    rast = np.array([[[[0, 0, 0, 0], [0, 0, 0, 1]]]], np.float32)
    out, _ = backend.interpolate(attr, rast, TRI1)
    assert out.reshape(-1).tolist() == [0, 0, 1, 1]


def test_range_mode_broadcasts_across_batch(backend):
    # InterpolateTests.swift:57-76
    attr2d = np.array([[10, 20], [30, 40], [50, 60]], np.float32)
    rast = np.array([[[[0, 0, 0, 1]]], [[[1, 0, 0, 1]]]], np.float32)
    out, _ = backend.interpolate(attr2d, rast, TRI1)
    assert out.shape == (2, 1, 1, 2)
    assert out.reshape(-1).tolist() == [10, 20, 30, 40]


def test_forward_da_matches_analytic(backend):
    # InterpolateTests.swift:78-104
    attr = np.array([[[1, 2], [4, 5], [7, 8]]], np.float32)
    rast = np.array([[[[0.1, 0.2, 0.0, 1.0]]]], np.float32)
    db = np.array([[[[0.5, -0.25, 0.125, 1.0]]]], np.float32)
    _, oda = backend.interpolate(attr, rast, TRI1, rast_db=db, diff_attrs="all")
    np.testing.assert_allclose(oda.reshape(-1), [2.25, 5.25, 2.25, 5.25], atol=1e-5)


def test_diff_attrs_indices_matches_all_subset(backend):
    # InterpolateTests.swift:106-131
    attr = np.arange(1, 10, dtype=np.float32).reshape(1, 3, 3)
    rast = np.array([[[[0.2, 0.3, 0.0, 1.0]]]], np.float32)
    db = np.array([[[[0.5, 0.1, -0.2, 0.3]]]], np.float32)
    _, da_all = backend.interpolate(attr, rast, TRI1, rast_db=db, diff_attrs="all")
    _, da_idx = backend.interpolate(attr, rast, TRI1, rast_db=db, diff_attrs=[0, 2])
    assert da_all.shape == (1, 1, 1, 6) and da_idx.shape == (1, 1, 1, 4)
    a, i = da_all.reshape(-1), da_idx.reshape(-1)
    np.testing.assert_allclose(i, [a[0], a[1], a[4], a[5]], atol=1e-6)


def _fixture(seed, A, with_da):
    g = np.random.default_rng(seed)
    H = W = 2
    u = g.uniform(0.05, 0.45, H * W)
    v = g.uniform(0.05, 0.45, H * W)
    rast = np.stack([u, v, np.zeros(4), np.ones(4)], 1).astype(np.float32).reshape(1, H, W, 4)
    attr = g.normal(size=(1, 3, A)).astype(np.float32)
    db = g.normal(size=(1, H, W, 4)).astype(np.float32) if with_da else np.zeros((1, H, W, 4), np.float32)
    w_out = g.normal(size=(1, H, W, A)).astype(np.float32)
    return rast, attr, db, w_out, g


@pytest.mark.parametrize("perturb,with_da", [("attr", False), ("rast", False), ("attr", True),
                                             ("rast", True), ("rastDB", True)])
def test_gradcheck(backend, perturb, with_da):
    # InterpolateTests.swift:133-160, 218-314
    A = 2
    rast, attr, db, w_out, g = _fixture(0xD1FFA570BEEF & 0xFFFFFFFF, A, with_da)
    w_da = g.normal(size=(1, 2, 2, 2 * A)).astype(np.float32) if with_da else None
    diff = "all" if with_da else None

    def loss_of(a, r, d):
        o, oda = backend.interpolate(a, r, TRI1, rast_db=d if with_da else None, diff_attrs=diff)
        return wsum(o, w_out) + (wsum(oda, w_da) if with_da else 0.0)

    d_attr, d_rast, d_db = backend.interpolate_bwd(attr, rast, TRI1, w_out, rast_db=db if with_da else None,
                                                   diff_attrs=diff, d_out_da=w_da)
    if perturb == "attr":
        np.testing.assert_allclose(d_attr, fd_grad(lambda x: loss_of(x, rast, db), attr), atol=5e-3)
    elif perturb == "rast":
        skip = lambda i: i % 4 in (2, 3)  # noqa: E731  tri-id and z channels: not differentiable
        num = fd_grad(lambda x: loss_of(attr, x, db), rast, skip=skip)
        flat = d_rast.reshape(-1)
        for i in range(flat.size):
            if skip(i):
                assert abs(flat[i]) < 1e-5
            else:
                assert abs(flat[i] - num.reshape(-1)[i]) < 5e-3
    else:
        np.testing.assert_allclose(d_db, fd_grad(lambda x: loss_of(attr, rast, x), db), atol=5e-3)


@pytest.mark.parametrize("perturb", ["attr", "rastDB"])
def test_diff_attrs_indices_gradcheck(backend, perturb):
    # InterpolateTests.swift:137-196 (.indices([1, 3]), A = 4)
    A, idx = 4, [1, 3]
    rast, attr, db, w_out, g = _fixture(0x1D7E50A2, A, True)
    w_da = g.normal(size=(1, 2, 2, 2 * len(idx))).astype(np.float32)

    def loss_of(a, d):
        o, oda = backend.interpolate(a, rast, TRI1, rast_db=d, diff_attrs=idx)
        return wsum(o, w_out) + wsum(oda, w_da)

    d_attr, _, d_db = backend.interpolate_bwd(attr, rast, TRI1, w_out, rast_db=db, diff_attrs=idx,
                                              d_out_da=w_da)
    if perturb == "attr":
        np.testing.assert_allclose(d_attr, fd_grad(lambda x: loss_of(x, db), attr), atol=5e-3)
    else:
        np.testing.assert_allclose(d_db, fd_grad(lambda x: loss_of(attr, x), db), atol=5e-3)


def test_shared_attr_gradient_sums_over_views(backend):
    # [V, A] attr broadcast over N views: its gradient is the sum over views
    # (MLX broadcast-backward, Interpolate.swift:67-73).
    g = np.random.default_rng(5)
    attr2d = g.normal(size=(3, 3)).astype(np.float32)
    rast = np.stack([np.tile(np.array([0.2, 0.3, 0, 1], np.float32), (2, 2, 1)),
                     np.tile(np.array([0.6, 0.1, 0, 1], np.float32), (2, 2, 1))])
    d_out = g.normal(size=(2, 2, 2, 3)).astype(np.float32)
    d_shared, _, _ = backend.interpolate_bwd(attr2d, rast, TRI1, d_out)
    d_full, _, _ = backend.interpolate_bwd(np.stack([attr2d, attr2d]), rast, TRI1, d_out)
    assert d_shared.shape == (3, 3)
    np.testing.assert_allclose(d_shared, d_full.sum(0), atol=1e-5)
