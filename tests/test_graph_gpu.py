"""Graph-safe binning (fixed tile-list capacity, no host readback) and CUDA
graph capture of a whole training step.

With a fixed capacity, tiles whose list would run past the buffer test every
triangle of their view; every result must stay bit-identical to the exact
(read-back) path, with ample and with tiny capacities, in every raster mode
(one layer, a peeled layer, two layers in one pass, with and without rast_db)
and in the unbinned mode used for very large views."""
import numpy as np
import pytest

from diffrast import scenes

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def soup():
    base, tri = scenes.triangle_soup(20000, 1000, 10, seed=21)
    M = scenes.similarity_matrices(3, seed=22)
    pos = np.einsum("nij,vj->nvi", M, base).astype(np.float32)
    return pos, tri


def _capped(pairs):
    import diffrast

    class _C:
        def __enter__(self):
            diffrast.raster_overflow()  # reset the count
            diffrast.set_raster_list_capacity(pairs)
            return self

        def __exit__(self, *a):
            diffrast.set_raster_list_capacity(0)
    return _C()


def _layers(pos, tri, res, n, db):
    import torch

    import diffrast
    out = diffrast.rasterize_layers(torch.from_numpy(pos).cuda(), torch.from_numpy(tri).cuda(), res, n, grad_db=db)
    torch.cuda.synchronize()
    return [(r.cpu().numpy(), d.cpu().numpy() if d is not None else None) for r, d in out]


@pytest.mark.parametrize("pairs", [1 << 24, 4096, 1])
@pytest.mark.parametrize("layers,db", [(1, False), (2, True), (3, True)])
def test_capped_lists_bit_exact(soup, pairs, layers, db):
    import diffrast
    pos, tri = soup
    res = (320, 288)
    ref = _layers(pos, tri, res, layers, db)
    with _capped(pairs):
        got = _layers(pos, tri, res, layers, db)
        over = diffrast.raster_overflow()
    for (ra, da), (rb, dbb) in zip(got, ref):
        assert np.array_equal(ra, rb)
        if db:
            assert np.array_equal(da, dbb)
    if pairs >= 1 << 24:
        assert over == 0
    else:
        assert over > 0  # the small buffers force the full-scan path


def test_capped_lists_unbinned_views(soup):
    # 3328^2 views have more tiles than the binned setup's shared histogram:
    # the unbinned setup / scatter with a capacity.
    import diffrast
    pos, tri = soup
    pos, tri = pos[:1], np.ascontiguousarray(tri[:2000])
    ref = _layers(pos, tri, (3328, 3328), 1, False)
    with _capped(1000):
        got = _layers(pos, tri, (3328, 3328), 1, False)
        over = diffrast.raster_overflow()
    assert np.array_equal(got[0][0], ref[0][0]) and over > 0


def test_cuda_graph_captures_a_training_step():
    # Rasterize -> interpolate -> antialias -> MSE and every VJP, captured once
    # and replayed: the same loss and gradients as the eager step.
    import torch

    import diffrast
    from diffrast import chains
    dev = torch.device("cuda", 0)
    c = chains.Cfg2(dev)
    with _capped(1 << 22):
        for p in c.params():
            p.grad = None
        ref_loss = float(c.step().detach())
        ref = [p.grad.detach().clone() for p in c.params()]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                for p in c.params():
                    p.grad = None
                c.step()
        torch.cuda.current_stream().wait_stream(s)
        for p in c.params():
            p.grad = None
        g = torch.cuda.CUDAGraph()
        n0 = diffrast.launch_count(0)
        with torch.cuda.graph(g):
            loss = c.step()
        captured = diffrast.launch_count(0) - n0
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        assert diffrast.raster_overflow() == 0
        assert captured > 10
        assert abs(float(loss.detach()) - ref_loss) <= 1e-6 * max(1.0, abs(ref_loss))
        for a, b in zip(c.params(), ref):
            ga, gb = a.grad.double(), b.double()
            assert float((ga - gb).norm() / gb.norm().clamp_min(1e-30)) < 1e-5
        del g


def test_capped_scan_all_batches_with_itemless_candidates():
    # Every tile scans the whole triangle list (capacity 1).  In tile (0, 0)
    # the staged batch of 256 candidates holds covering triangles interleaved
    # with triangles elsewhere (no items in that tile), and its last 56
    # candidates own no item at all: the walk must skip item-less candidates
    # in the middle and never step past the batch's last item.
    import oracle as O
    import diffrast
    res = (64, 64)
    g = np.random.default_rng(5)
    verts, tris = [], []
    for i in range(256):
        in_tile0 = i < 200 and i % 3 != 1
        cx, cy = ((-0.85, 0.85) if in_tile0 else (0.6, -0.6))
        cx += g.uniform(-0.1, 0.1); cy += g.uniform(-0.1, 0.1)
        z = g.uniform(-0.9, 0.9)
        r = g.uniform(0.05, 0.3)
        a = g.uniform(0, 2 * np.pi)
        for k in range(3):
            verts.append([cx + r * np.cos(a + 2.1 * k), cy + r * np.sin(a + 2.1 * k), z, 1.0])
        tris.append([3 * i, 3 * i + 1, 3 * i + 2])
    pos = np.array([verts], np.float32)
    tri = np.array(tris, np.int32)
    ref = _layers(pos, tri, res, 2, True)
    with _capped(1):
        got = _layers(pos, tri, res, 2, True)
        over = diffrast.raster_overflow()
    assert over > 0
    r_prev = None
    for l in range(2):
        assert np.array_equal(got[l][0], ref[l][0]) and np.array_equal(got[l][1], ref[l][1])
        r_o, d_o = O.rasterize(pos, tri, res, peel_layer=r_prev)
        assert np.array_equal(got[l][0], r_o) and np.array_equal(got[l][1], d_o)
        r_prev = r_o
    assert (got[0][0][0, :16, :16, 3] > 0).mean() > 0.5  # tile (0, 0) is mostly covered
