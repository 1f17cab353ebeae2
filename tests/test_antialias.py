"""Antialias / topology-hash known-answer tests and gradchecks, restated from the
reference's Tests/MLXDiffRastTests/AntialiasTests.swift, on the oracle and the
CUDA path."""
import numpy as np

from helpers import fd_grad, wsum

TRI1 = np.array([[0, 1, 2]], np.int32)


def test_topology_hash_two_triangles_shared_edge(backend):
    # AntialiasTests.swift:11-36
    h = backend.topology_hash(np.array([[0, 1, 2], [1, 2, 3]], np.int32))
    assert h.shape == (2, 3)
    assert h.reshape(-1).tolist() == [1, -1, -1, -1, -1, 0]


def test_topology_hash_single_triangle_all_boundary(backend):
    # AntialiasTests.swift:38-42
    assert backend.topology_hash(TRI1).reshape(-1).tolist() == [-1, -1, -1]


def test_topology_hash_non_manifold_edge_marked(backend):
    # AntialiasTests.swift:47-71
    h = backend.topology_hash(np.array([[0, 1, 2], [0, 1, 3], [0, 1, 4]], np.int32))
    for t in range(3):
        assert h[t, 2] == -2 and h[t, 0] == -1 and h[t, 1] == -1


def test_topology_hash_matches_sort_reference_on_random_mesh(backend):
    # Degenerate and repeated edges included: the GPU hash must equal the
    # reference's sort-and-run construction bit for bit.
    import oracle
    g = np.random.default_rng(7)
    tri = g.integers(0, 40, size=(500, 3)).astype(np.int32)
    assert np.array_equal(backend.topology_hash(tri), oracle.topology_hash(tri))


def test_no_silhouette_is_identity(backend):
    # AntialiasTests.swift:78-87
    color = np.arange(18, dtype=np.float32).reshape(1, 3, 3, 2)
    out = backend.antialias(color, np.zeros((1, 3, 3, 4), np.float32), np.zeros((1, 3, 4), np.float32), TRI1)
    assert np.array_equal(out, color)


def test_fully_covered_is_identity(backend):
    # AntialiasTests.swift:91-107
    color = np.array([1, 2, 3, 4], np.float32).reshape(1, 2, 2, 1)
    pos = np.array([[[-3, 3, 0, 1], [-3, -3, 0, 1], [3, 0, 0, 1]]], np.float32)
    rast, _ = backend.rasterize(pos, TRI1, (2, 2), grad_db=False)
    assert np.array_equal(backend.antialias(color, rast, pos, TRI1), color)


TILTED = np.array([[[-3, 3, 0, 1], [-3, -2.7, 0, 1], [2.7, 3, 0, 1]]], np.float32)


def test_silhouette_blends_covered_and_empty_pixels(backend):
    # AntialiasTests.swift:112-173
    H = W = 4
    rast, _ = backend.rasterize(TILTED, TRI1, (H, W), grad_db=False)
    color = (10.0 * (1 + np.arange(16, dtype=np.float32))).reshape(1, H, W, 1)
    out = backend.antialias(color, rast, TILTED, TRI1)
    cov = rast[0, ..., 3] > 0
    found = False
    for h in range(H):
        for w in range(W):
            nbrs = [(h, w + 1), (h + 1, w), (h, w - 1), (h - 1, w)]
            mixed = any(0 <= a < H and 0 <= b < W and cov[a, b] != cov[h, w] for a, b in nbrs)
            if mixed and abs(out[0, h, w, 0] - color[0, h, w, 0]) > 1e-4:
                found = True
    assert found
    ids = rast[0, ..., 3]
    for h in range(1, H - 1):
        for w in range(1, W - 1):
            if np.all(ids[h - 1:h + 2, w - 1:w + 2] == ids[h, w]):
                assert abs(out[0, h, w, 0] - color[0, h, w, 0]) < 1e-5


def test_gradcheck_color(backend):
    # AntialiasTests.swift:176-213
    H = W = 4
    C = 2
    rast, _ = backend.rasterize(TILTED, TRI1, (H, W), grad_db=False)
    topo = backend.topology_hash(TRI1)
    color = (np.arange(H * W * C, dtype=np.float32) * 0.3 + 1).reshape(1, H, W, C)
    w = np.array([(1 + i % 7) * 0.1 for i in range(H * W * C)], np.float32).reshape(1, H, W, C)
    d_color, _ = backend.antialias_bwd(color, rast, TILTED, TRI1, w, topo)
    num = fd_grad(lambda x: wsum(backend.antialias(x, rast, TILTED, TRI1, topo), w), color)
    np.testing.assert_allclose(d_color, num, atol=5e-3)


QUAD_POS = np.array([[[-0.45, 0.55, 0, 1], [0.55, 0.55, 0, 1], [0.55, -0.45, 0, 1], [-0.45, -0.45, 0, 1]]],
                    np.float32)
QUAD_TRI = np.array([[0, 1, 2], [0, 2, 3]], np.int32)


def test_gradcheck_pos(backend):
    # AntialiasTests.swift:223-279 (rast frozen outside the loss)
    H = W = 4
    C = 2
    topo = backend.topology_hash(QUAD_TRI)
    rast, _ = backend.rasterize(QUAD_POS, QUAD_TRI, (H, W), grad_db=False)
    color = (np.arange(H * W * C, dtype=np.float32) * 0.3 + 1).reshape(1, H, W, C)
    w = np.array([(1 + i % 5) * 0.1 for i in range(H * W * C)], np.float32).reshape(1, H, W, C)
    _, d_pos = backend.antialias_bwd(color, rast, QUAD_POS, QUAD_TRI, w, topo)
    num = fd_grad(lambda p: wsum(backend.antialias(color, rast, p, QUAD_TRI, topo), w), QUAD_POS)
    np.testing.assert_allclose(d_pos, num, atol=5e-3)


def test_pos_gradient_is_non_trivial(backend):
    # AntialiasTests.swift:283-297
    H = W = 4
    rast, _ = backend.rasterize(QUAD_POS, QUAD_TRI, (H, W), grad_db=False)
    color = np.arange(16, dtype=np.float32).reshape(1, H, W, 1)
    _, d_pos = backend.antialias_bwd(color, rast, QUAD_POS, QUAD_TRI, np.ones_like(color))
    assert np.any(np.abs(d_pos) > 1e-5)
