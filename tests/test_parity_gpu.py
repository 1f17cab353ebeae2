"""CUDA library vs CPU oracle on seeded synthetic scenes (the configurations'
meshes at sizes the oracle finishes in seconds, plus full-resolution views of
the 1M-triangle soup).  Tolerances:
  tri_id / coverage / topology: bit-exact
  barycentrics, z, rast_db, interpolated values, textures: <= 1e-5 relative
  (in practice bit-exact where no atomics are involved)
  gradients with atomic accumulation: <= 1e-4 relative L2
"""
import numpy as np
import pytest

import backends
from diffrast import scenes
from helpers import rel_l2

pytestmark = pytest.mark.gpu

O = backends.OracleBackend()


@pytest.fixture(scope="module")
def cu():
    return backends.CudaBackend()


def _rel_max(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-6)) if a.size else 0.0


@pytest.fixture(scope="module")
def ico():
    return scenes.scene_icosphere_views(4, 256)


@pytest.fixture(scope="module")
def soup():
    base, tri = scenes.triangle_soup(20000, 1000, 10, seed=21)
    M = scenes.similarity_matrices(3, seed=22)
    pos = np.einsum("nij,vj->nvi", M, base).astype(np.float32)
    return pos, tri


def test_rasterize_bit_exact_icosphere(cu, ico):
    for db in (False, True):
        r_c, d_c = cu.rasterize(ico["pos"], ico["tri"], ico["res"], grad_db=db)
        r_o, d_o = O.rasterize(ico["pos"], ico["tri"], ico["res"], grad_db=db)
        assert np.array_equal(r_c, r_o)
        if db:
            assert np.array_equal(d_c, d_o)


def test_rasterize_bit_exact_soup_with_peel(cu, soup):
    pos, tri = soup
    r0c, d0c = cu.rasterize(pos, tri, (320, 288))
    r0o, d0o = O.rasterize(pos, tri, (320, 288))
    assert np.array_equal(r0c, r0o) and np.array_equal(d0c, d0o)
    r1c, _ = cu.rasterize(pos, tri, (320, 288), peel=r0o)
    r1o, _ = O.rasterize(pos, tri, (320, 288), peel=r0o)
    assert np.array_equal(r1c, r1o)
    assert (r1c[..., 3] > 0).sum() > 0  # the second layer is not empty


def test_rasterize_range_mode_bit_exact(cu, soup):
    pos, tri = soup
    T = tri.shape[0]
    ranges = np.array([[0, T // 2], [T // 3, T // 2], [0, T]], np.int32)
    r_c, _ = cu.rasterize(pos[0], tri, (128, 200), ranges=ranges)
    r_o, _ = O.rasterize(pos[0], tri, (128, 200), ranges=ranges)
    assert np.array_equal(r_c, r_o)


def test_rasterize_full_size_soup_views_bit_exact(cu):
    # Two full 1024^2 views of the 1M-triangle cfg4 soup (depth complexity ~13).
    s = scenes.scene_cfg4(n_views=2)
    pos = np.einsum("nij,vj->nvi", s["sim"], s["base"]).astype(np.float32)
    r_c, d_c = cu.rasterize(pos, s["tri"], s["res"])
    r_o, d_o = O.rasterize(pos, s["tri"], s["res"])
    assert np.array_equal(r_c[..., 3], r_o[..., 3])
    assert np.array_equal(r_c, r_o) and np.array_equal(d_c, d_o)


def test_rasterize_bwd_matches_oracle(cu, ico):
    g = np.random.default_rng(1)
    N, (H, W) = ico["pos"].shape[0], ico["res"]
    d_r = g.normal(size=(N, H, W, 4)).astype(np.float32)
    d_db = g.normal(size=(N, H, W, 4)).astype(np.float32)
    for db in (None, d_db):
        a = cu.rasterize_bwd(ico["pos"], ico["tri"], ico["res"], d_r, db)
        b = O.rasterize_bwd(ico["pos"], ico["tri"], ico["res"], d_r, db)
        assert rel_l2(a, b) < 1e-4


def test_rasterize_bwd_range_mode(cu, soup):
    pos, tri = soup
    T = tri.shape[0]
    ranges = np.array([[0, T], [T // 4, T // 2]], np.int32)
    d_r = np.random.default_rng(2).normal(size=(2, 96, 96, 4)).astype(np.float32)
    a = cu.rasterize_bwd(pos[0], tri, (96, 96), d_r, ranges=ranges)
    b = O.rasterize_bwd(pos[0], tri, (96, 96), d_r, ranges=ranges)
    assert a.shape == pos[0].shape and rel_l2(a, b) < 1e-4


@pytest.mark.parametrize("A,diff", [(3, None), (8, "all"), (5, [4, 0, 2]), (2, "all")])
@pytest.mark.parametrize("shared", [True, False])
def test_interpolate_matches_oracle(cu, ico, A, diff, shared):
    rast, db = O.rasterize(ico["pos"], ico["tri"], ico["res"])
    N, V = ico["pos"].shape[:2]
    g = np.random.default_rng(A)
    attr = g.normal(size=((V, A) if shared else (N, V, A))).astype(np.float32)
    o_c, oda_c = cu.interpolate(attr, rast, ico["tri"], db, diff)
    o_o, oda_o = O.interpolate(attr, rast, ico["tri"], db, diff)
    assert _rel_max(o_c, o_o) <= 1e-5 and _rel_max(oda_c, oda_o) <= 1e-5
    K = 0 if diff is None else (A if diff == "all" else len(diff))
    d_out = g.normal(size=o_o.shape).astype(np.float32)
    d_da = g.normal(size=(N,) + ico["res"] + (2 * K,)).astype(np.float32) if K else None
    ga = cu.interpolate_bwd(attr, rast, ico["tri"], d_out, db, diff, d_da)
    gb = O.interpolate_bwd(attr, rast, ico["tri"], d_out, db, diff, d_da)
    assert rel_l2(ga[0], gb[0]) < 1e-4
    np.testing.assert_allclose(ga[1], gb[1], rtol=1e-5, atol=1e-6)
    if K:
        np.testing.assert_allclose(ga[2], gb[2], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("C", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("boundary", ["wrap", "clamp", "zero"])
@pytest.mark.parametrize("filt", ["nearest", "linear", "linear-mipmap-nearest", "linear-mipmap-linear"])
def test_texture_matches_oracle(cu, filt, boundary, C):
    # C = 4 takes the float4 texel path, C <= 4 the vector-atomic scatter
    # (float2 pairs for C = 2, 3), C = 5 the per-channel fallback.
    g = np.random.default_rng(11)
    tex = g.random((1, 64, 128, C)).astype(np.float32)
    uv = g.uniform(-0.3, 1.3, size=(2, 48, 40, 2)).astype(np.float32)
    da = (g.normal(size=(2, 48, 40, 4)) * 0.02).astype(np.float32)
    bmap = g.uniform(-1, 1, size=(2, 48, 40)).astype(np.float32)
    mip = filt.startswith("linear-mipmap")
    kw = dict(uv_da=da if mip else None, filter_mode=filt, boundary_mode=boundary,
              bias=0.5 if mip else 0.0, bias_map=bmap if mip else None)
    a = cu.texture(tex, uv, **kw)
    b = O.texture(tex, uv, **kw)
    assert _rel_max(a, b) <= 1e-5
    d_out = g.normal(size=a.shape).astype(np.float32)
    ga = cu.texture_bwd(tex, uv, d_out, **kw)
    gb = O.texture_bwd(tex, uv, d_out, **kw)
    assert rel_l2(ga[0], gb[0]) < 1e-4
    assert rel_l2(ga[1], gb[1]) < 1e-4 if np.any(gb[1]) else np.all(ga[1] == 0)
    if mip:
        assert rel_l2(ga[2], gb[2]) < 1e-4
        assert rel_l2(ga[3], gb[3]) < 1e-4


def test_texture_cube_matches_oracle(cu):
    g = np.random.default_rng(12)
    tex = g.random((2, 6, 32, 32, 3)).astype(np.float32)
    d = g.normal(size=(2, 40, 24, 3)).astype(np.float32)
    a = cu.texture(tex, d, boundary_mode="cube")
    b = O.texture(tex, d, boundary_mode="cube")
    assert _rel_max(a, b) <= 1e-5
    d_out = g.normal(size=a.shape).astype(np.float32)
    ga = cu.texture_bwd(tex, d, d_out, boundary_mode="cube")
    gb = O.texture_bwd(tex, d, d_out, boundary_mode="cube")
    assert rel_l2(ga[0], gb[0]) < 1e-4 and np.all(ga[1] == 0)
    # d_dir through the projection (extension, opt-in)
    ga = cu.texture_bwd(tex, d, d_out, boundary_mode="cube", cube_dir_grad=True)
    gb = O.texture_bwd(tex, d, d_out, boundary_mode="cube", cube_dir_grad=True)
    assert rel_l2(ga[0], gb[0]) < 1e-4 and rel_l2(ga[1], gb[1]) < 1e-4


@pytest.mark.parametrize("C", [1, 3, 4])
@pytest.mark.parametrize("nt", [1, 2])
@pytest.mark.parametrize("filt", ["linear-mipmap-nearest", "linear-mipmap-linear"])
def test_texture_cube_mip_matches_oracle(cu, filt, nt, C):
    # Mip-mapped cube (extension): LOD from the direction derivatives through
    # the cube projection, per-face pyramids, bias and bias map.
    g = np.random.default_rng(21)
    tex = g.random((nt, 6, 64, 64, C)).astype(np.float32)
    d = g.normal(size=(2, 40, 24, 3)).astype(np.float32)
    dd = (np.exp(g.uniform(-7, 0, size=(2, 40, 24, 1))) * g.normal(size=(2, 40, 24, 6))).astype(np.float32)
    bmap = g.uniform(-1, 1, size=(2, 40, 24)).astype(np.float32)
    kw = dict(uv_da=dd, filter_mode=filt, boundary_mode="cube", bias=0.25, bias_map=bmap)
    a = cu.texture(tex, d, **kw)
    b = O.texture(tex, d, **kw)
    assert _rel_max(a, b) <= 1e-5
    d_out = g.normal(size=a.shape).astype(np.float32)
    ga = cu.texture_bwd(tex, d, d_out, **kw)
    gb = O.texture_bwd(tex, d, d_out, **kw)
    assert rel_l2(ga[0], gb[0]) < 1e-4 and np.all(ga[1] == 0)
    assert ga[2].shape == dd.shape and rel_l2(ga[2], gb[2]) < 1e-4
    assert rel_l2(ga[3], gb[3]) < 1e-4
    ga = cu.texture_bwd(tex, d, d_out, cube_dir_grad=True, **kw)
    gb = O.texture_bwd(tex, d, d_out, cube_dir_grad=True, **kw)
    assert rel_l2(ga[1], gb[1]) < 1e-4 and rel_l2(ga[2], gb[2]) < 1e-4


@pytest.mark.parametrize("C", [1, 3, 4, 5])
@pytest.mark.parametrize("filt", ["linear-mipmap-nearest", "linear-mipmap-linear"])
def test_texture_bwd_small_levels_reduced_in_shared_memory(cu, filt, C):
    # A bias of +6 sends most LODs to the pyramid's top levels (4x4 .. 1x1 of
    # a 256^2 texture), which the VJP accumulates in shared memory per CTA and
    # adds to the pyramid gradient once per CTA: many pixels per texel.
    g = np.random.default_rng(31)
    tex = g.random((1, 256, 256, C)).astype(np.float32)
    uv = g.uniform(0, 1, size=(3, 96, 80, 2)).astype(np.float32)
    da = (g.normal(size=(3, 96, 80, 4)) * 0.01).astype(np.float32)
    bmap = g.uniform(-1, 1, size=(3, 96, 80)).astype(np.float32)
    kw = dict(uv_da=da, filter_mode=filt, boundary_mode="wrap", bias=6.0, bias_map=bmap)
    a = cu.texture(tex, uv, **kw)
    b = O.texture(tex, uv, **kw)
    assert _rel_max(a, b) <= 1e-5
    d_out = g.normal(size=a.shape).astype(np.float32)
    ga = cu.texture_bwd(tex, uv, d_out, **kw)
    gb = O.texture_bwd(tex, uv, d_out, **kw)
    for x, y in zip(ga, gb):
        assert rel_l2(x, y) < 1e-4


def test_texture_mip_large_pyramid(cu):
    # A 1024^2 x 4 texture (11 levels) sampled at mixed LODs.
    g = np.random.default_rng(13)
    tex = scenes.value_noise(1024, 1024, 4, seed=8)[None]
    uv = g.uniform(0, 1, size=(1, 64, 64, 2)).astype(np.float32)
    da = (np.exp(g.uniform(-9, 0, size=(1, 64, 64, 1))) * g.normal(size=(1, 64, 64, 4))).astype(np.float32)
    kw = dict(uv_da=da, filter_mode="linear-mipmap-linear", boundary_mode="wrap")
    a = cu.texture(tex, uv, **kw)
    b = O.texture(tex, uv, **kw)
    assert _rel_max(a, b) <= 1e-5
    d_out = g.normal(size=a.shape).astype(np.float32)
    ga, gb = cu.texture_bwd(tex, uv, d_out, **kw), O.texture_bwd(tex, uv, d_out, **kw)
    assert rel_l2(ga[0], gb[0]) < 1e-4 and rel_l2(ga[1], gb[1]) < 1e-4 and rel_l2(ga[2], gb[2]) < 1e-4


@pytest.mark.parametrize("C", [3, 4])
def test_construct_mip_matches_oracle(cu, C):
    # C = 4 builds with one float4 per texel; both bit-exact.
    tex = np.random.default_rng(14).random((2, 256, 128, C)).astype(np.float32)
    for a, b in zip(cu.construct_mip(tex), O.construct_mip(tex)):
        assert np.array_equal(a, b)


def test_topology_hash_bit_exact_on_scenes(cu, ico, soup):
    for tri in (ico["tri"], soup[1]):
        assert np.array_equal(cu.topology_hash(tri), O.topology_hash(tri))


def test_antialias_matches_oracle(cu, ico):
    rast, _ = O.rasterize(ico["pos"], ico["tri"], ico["res"], grad_db=False)
    g = np.random.default_rng(15)
    N, (H, W) = ico["pos"].shape[0], ico["res"]
    color = g.random((N, H, W, 3)).astype(np.float32)
    topo = O.topology_hash(ico["tri"])
    a = cu.antialias(color, rast, ico["pos"], ico["tri"], topo)
    b = O.antialias(color, rast, ico["pos"], ico["tri"], topo)
    assert _rel_max(a, b) <= 1e-5
    assert np.any(a != color)
    d_out = g.normal(size=a.shape).astype(np.float32)
    ga = cu.antialias_bwd(color, rast, ico["pos"], ico["tri"], d_out, topo)
    gb = O.antialias_bwd(color, rast, ico["pos"], ico["tri"], d_out, topo)
    assert rel_l2(ga[0], gb[0]) < 1e-5
    assert rel_l2(ga[1], gb[1]) < 1e-4


def test_antialias_soup_with_strips(cu, soup):
    pos, tri = soup
    rast, _ = O.rasterize(pos, tri, (256, 256), grad_db=False)
    g = np.random.default_rng(16)
    color = g.normal(size=(pos.shape[0], 256, 256, 8)).astype(np.float32)
    topo = O.topology_hash(tri)
    a = cu.antialias(color, rast, pos, tri, topo)
    b = O.antialias(color, rast, pos, tri, topo)
    assert _rel_max(a, b) <= 1e-5
    d_out = g.normal(size=a.shape).astype(np.float32)
    ga = cu.antialias_bwd(color, rast, pos, tri, d_out, topo)
    gb = O.antialias_bwd(color, rast, pos, tri, d_out, topo)
    assert rel_l2(ga[0], gb[0]) < 1e-5 and rel_l2(ga[1], gb[1]) < 1e-4


def test_rasterize_layers_equals_chained_peeling(cu, soup):
    import torch

    import diffrast
    pos, tri = soup
    p = torch.from_numpy(pos).cuda().requires_grad_(True)
    t = torch.from_numpy(tri).cuda()
    layers = diffrast.rasterize_layers(p, t, (200, 256), 3)
    r_prev = None
    for l, (r, db) in enumerate(layers):
        rc, dc = diffrast.rasterize(p.detach(), t, (200, 256), peel_layer=r_prev)
        assert torch.equal(r, rc) and torch.equal(db, dc), l
        r_prev = rc
    # VJP of the layered call == sum of the per-layer VJPs
    g = np.random.default_rng(3)
    w = [torch.from_numpy(g.normal(size=(3, 200, 256, 4)).astype(np.float32)).cuda() for _ in range(6)]
    loss = sum((r * w[2 * l]).sum() + (db * w[2 * l + 1]).sum() for l, (r, db) in enumerate(layers))
    loss.backward()
    import oracle
    ref = np.zeros_like(pos)
    r_prev = None
    for l in range(3):
        r_o, _ = oracle.rasterize(pos, tri, (200, 256), peel_layer=r_prev)
        ref += oracle.rasterize_bwd(pos, tri, r_o, w[2 * l].cpu().numpy(), w[2 * l + 1].cpu().numpy())
        r_prev = r_o
    assert rel_l2(p.grad.cpu().numpy(), ref) < 1e-4


@pytest.mark.parametrize("diff", [None, "all"])
def test_interpolate_bwd_soup_short_runs(cu, soup, diff):
    # Tiny triangles: pixel runs of equal triangle are short, exercising the
    # warp-aggregated d_attr path with many heads per warp.
    pos, tri = soup
    rast, db = O.rasterize(pos, tri, (256, 256))
    V = pos.shape[1]
    g = np.random.default_rng(17)
    attr = g.normal(size=(V, 8)).astype(np.float32)
    d_out = g.normal(size=(3, 256, 256, 8)).astype(np.float32)
    d_da = g.normal(size=(3, 256, 256, 16)).astype(np.float32) if diff else None
    ga = cu.interpolate_bwd(attr, rast, tri, d_out, db, diff, d_da)
    gb = O.interpolate_bwd(attr, rast, tri, d_out, db, diff, d_da)
    assert rel_l2(ga[0], gb[0]) < 1e-4
    np.testing.assert_allclose(ga[1], gb[1], rtol=1e-5, atol=1e-5)
    if diff:
        np.testing.assert_allclose(ga[2], gb[2], rtol=1e-5, atol=1e-5)


def test_xf_mode_matches_instanced_on_transformed_positions(cu, soup):
    # Per-view transform entry points: identical rasterization to instanced mode
    # on the positions the transform defines; d_verts = sum_n M_n^T d_pos_n.
    import torch

    import diffrast
    import oracle
    base, tri = scenes.triangle_soup(20000, 1000, 10, seed=21)
    M = scenes.similarity_matrices(3, seed=22).astype(np.float32)
    M[1, 3, 2] = 0.01  # a non-affine row, so w depends on z
    pos = oracle.xf_positions(base, M)
    vb = torch.from_numpy(base).cuda().requires_grad_(True)
    xf = torch.from_numpy(M).cuda()
    t = torch.from_numpy(tri).cuda()
    layers = diffrast.rasterize_layers(vb, t, (160, 192), 2, xform=xf)
    r0o, d0o = O.rasterize(pos, tri, (160, 192))
    r1o, d1o = O.rasterize(pos, tri, (160, 192), peel=r0o)
    assert np.array_equal(layers[0][0].detach().cpu().numpy(), r0o)
    assert np.array_equal(layers[0][1].detach().cpu().numpy(), d0o)
    assert np.array_equal(layers[1][0].detach().cpu().numpy(), r1o)
    assert np.array_equal(layers[1][1].detach().cpu().numpy(), d1o)
    g = np.random.default_rng(4)
    w = [g.normal(size=(3, 160, 192, 4)).astype(np.float32) for _ in range(4)]
    col = torch.from_numpy(g.normal(size=(3, 160, 192, 3)).astype(np.float32)).cuda()
    wa = g.normal(size=(3, 160, 192, 3)).astype(np.float32)
    aa = diffrast.antialias(col, layers[0][0], vb, t, xform=xf)
    topo = oracle.topology_hash(tri)
    np.testing.assert_allclose(aa.detach().cpu().numpy(), oracle.antialias(col.cpu().numpy(), r0o, pos, tri, topo), rtol=1e-5,
                               atol=1e-6)
    loss = sum((layers[l][0] * torch.from_numpy(w[2 * l]).cuda()).sum()
               + (layers[l][1] * torch.from_numpy(w[2 * l + 1]).cuda()).sum() for l in range(2))
    loss = loss + (aa * torch.from_numpy(wa).cuda()).sum()
    loss.backward()
    d_pos = (oracle.rasterize_bwd(pos, tri, r0o, w[0], w[1]) + oracle.rasterize_bwd(pos, tri, r1o, w[2], w[3])
             + oracle.antialias_bwd(col.cpu().numpy(), r0o, pos, tri, wa, topo)[1])
    ref = oracle.xf_vertex_grad(d_pos, M)
    assert rel_l2(vb.grad.cpu().numpy(), ref) < 1e-4


def test_layers_fused_pass_depth_ties(cu, soup):
    # Every triangle appears three times: twice at its own depth (an exact z
    # tie, broken by the lower index) and once pushed back.  Layer 1 must skip
    # the tied copy (z <= layer-0 z is peeled) and find the pushed-back one or a
    # deeper triangle — the z == z(k0) branch of the fused two-layer pass.
    import torch

    import diffrast
    pos, tri = soup
    pos = pos[:, :, :].copy()
    V = pos.shape[1]
    back = pos.copy()
    back[..., 2] += 0.05 * back[..., 3]
    p = np.concatenate([pos, back], axis=1)
    t = np.concatenate([tri, tri, tri + V]).astype(np.int32)
    layers = diffrast.rasterize_layers(torch.from_numpy(p).cuda(), torch.from_numpy(t).cuda(), (192, 160), 3)
    r_prev = None
    for l in range(3):
        r_o, d_o = O.rasterize(p, t, (192, 160), peel=r_prev)
        assert np.array_equal(layers[l][0].cpu().numpy(), r_o), l
        assert np.array_equal(layers[l][1].cpu().numpy(), d_o), l
        r_prev = r_o
    ids0 = layers[0][0][..., 3].cpu().numpy()
    assert ids0.max() <= tri.shape[0]  # ties resolve to the first copy


def test_subnormal_area_slivers_bit_exact(cu, soup):
    # Slivers of area 2^-129 (1/area = inf, NaN depth along the row y = 0)
    # spliced into the soup before and after full-screen triangles: CUDA and the
    # oracle agree bit for bit in one layer, in the fused two-layer pass and in
    # a peeled third layer.
    import torch

    import diffrast
    pos, tri = soup
    V = pos.shape[1]
    N = pos.shape[0]
    tiny = np.float32(2.0 ** -130)
    extra = np.array([[-1, 0, -0.5, 1], [1, 0, -0.5, 1], [1, tiny, -0.5, 1],
                      [-4, -4, 0.95, 1], [4, -4, 0.95, 1], [0, 4, 0.95, 1],
                      [-0.5, 0, -0.9, 1], [0.7, 0, -0.9, 1], [0.7, tiny, -0.9, 1]], np.float32)
    p = np.concatenate([pos, np.broadcast_to(extra, (N,) + extra.shape)], axis=1).copy()
    e = np.arange(9, dtype=np.int32).reshape(3, 3) + V
    t = np.concatenate([e[:1], tri[: len(tri) // 2], e[1:2], tri[len(tri) // 2:], e[2:]]).astype(np.int32)
    res = (161, 144)  # odd height: the centre row is y = 0 exactly
    r_c, d_c = cu.rasterize(p, t, res)
    r_o, d_o = O.rasterize(p, t, res)
    assert np.array_equal(r_c, r_o) and np.array_equal(d_c, d_o)
    assert np.all(np.isfinite(r_c)) and np.all(np.isfinite(d_c))
    layers = diffrast.rasterize_layers(torch.from_numpy(p).cuda(), torch.from_numpy(t).cuda(), res, 3)
    r_prev = None
    for l in range(3):
        r_o, d_o = O.rasterize(p, t, res, peel=r_prev)
        assert np.array_equal(layers[l][0].cpu().numpy(), r_o), l
        assert np.array_equal(layers[l][1].cpu().numpy(), d_o), l
        r_prev = r_o


def test_layers_full_size_soup_two_views(cu):
    # Both depth layers of two full 1024^2 cfg4 views from the fused pass.
    import torch

    import diffrast
    s = scenes.scene_cfg4(n_views=2)
    pos = np.einsum("nij,vj->nvi", s["sim"], s["base"]).astype(np.float32)
    layers = diffrast.rasterize_layers(torch.from_numpy(pos).cuda(), torch.from_numpy(s["tri"]).cuda(), s["res"], 2)
    r0o, d0o = O.rasterize(pos, s["tri"], s["res"])
    r1o, d1o = O.rasterize(pos, s["tri"], s["res"], peel=r0o)
    assert np.array_equal(layers[0][0].cpu().numpy(), r0o) and np.array_equal(layers[0][1].cpu().numpy(), d0o)
    assert np.array_equal(layers[1][0].cpu().numpy(), r1o) and np.array_equal(layers[1][1].cpu().numpy(), d1o)


@pytest.mark.parametrize("xf", [False, True])
def test_antialias_vjp_from_forward_record_equals_search(cu, soup, xf):
    # The VJP with the forward's per-pixel record (aa_work) and the VJP that
    # searches the silhouettes again give the same d_color bit for bit and the
    # same d_pos up to float atomic order.
    import ctypes

    import torch

    from diffrast import _lib as L
    pos, tri = soup
    N, H, W, C = pos.shape[0], 256, 224, 8
    base, Ms = None, None
    if xf:
        import oracle
        base, _ = scenes.triangle_soup(20000, 1000, 10, seed=21)
        Ms = scenes.similarity_matrices(N, seed=22).astype(np.float32)
        pos = oracle.xf_positions(base, Ms)
    rast, _ = O.rasterize(pos, tri, (H, W), grad_db=False)
    g = np.random.default_rng(23)
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    color, d_out = t(g.normal(size=(N, H, W, C)).astype(np.float32)), t(g.normal(size=(N, H, W, C)).astype(np.float32))
    r, tr = t(rast), t(tri)
    topo = t(O.topology_hash(tri))
    from diffrast import ops
    lib = L.lib()
    c = ops._ctx(color)
    V = (base if xf else pos).shape[-2]
    p = t(base) if xf else t(pos)
    xfm = t(Ms) if xf else None
    work = torch.empty(lib.dr_antialias_work_bytes(N, H, W), dtype=torch.uint8, device=dev)
    outs = []
    for w in (None, work):
        out = torch.empty_like(color)
        dc, dp = torch.empty_like(color), torch.empty_like(p)
        P = lambda x: None if x is None else x.data_ptr()
        if xf:
            L.check(lib.dr_antialias_xf_fwd(c, P(color), N, H, W, C, P(r), P(p), V, P(xfm), P(tr), tri.shape[0],
                                            P(topo), P(out), P(w)), c, "aa_xf_fwd")
            L.check(lib.dr_antialias_xf_bwd(c, P(color), N, H, W, C, P(r), P(p), V, P(xfm), P(tr), tri.shape[0],
                                            P(topo), P(d_out), P(dc), P(dp), P(w)), c, "aa_xf_bwd")
        else:
            L.check(lib.dr_antialias_fwd(c, P(color), N, H, W, C, P(r), P(p), V, P(tr), tri.shape[0], P(topo),
                                         P(out), P(w)), c, "aa_fwd")
            L.check(lib.dr_antialias_bwd(c, P(color), N, H, W, C, P(r), P(p), V, P(tr), tri.shape[0], P(topo),
                                         P(d_out), P(dc), P(dp), P(w)), c, "aa_bwd")
        torch.cuda.synchronize()
        outs.append((out.cpu().numpy(), dc.cpu().numpy(), dp.cpu().numpy()))
    (o0, c0, p0), (o1, c1, p1) = outs
    assert np.array_equal(o0, o1) and np.array_equal(c0, c1)
    assert rel_l2(p1, p0) < 1e-5
    wb = work[: N * H * W * 16].view(torch.float32).view(N, H, W, 4).cpu().numpy()
    assert (wb > 0).any() and (wb <= 0.5).all()
    # and against the oracle's VJP
    gb = O.antialias_bwd(color.cpu().numpy(), rast, pos, tri, d_out.cpu().numpy(), topo.cpu().numpy())
    assert rel_l2(c1, gb[0]) < 1e-5
    ref_p = oracle_vertex_grad(gb[1], Ms) if xf else gb[1]
    assert rel_l2(p1, ref_p) < 1e-4


def oracle_vertex_grad(d_pos, Ms):
    import oracle
    return oracle.xf_vertex_grad(d_pos, Ms)


def test_rasterize_unbinned_setup_at_large_resolution(cu, ico):
    # 3328 x 3328 has 43,264 tiles per view, more than the binned setup's
    # shared histogram holds, so tile lists are built by the per-triangle
    # global-atomic setup; the result is the same bit for bit.
    pos, tri = ico["pos"][:1], ico["tri"]
    r_c, d_c = cu.rasterize(pos, tri, (3328, 3328))
    r_o, d_o = O.rasterize(pos, tri, (3328, 3328))
    assert np.array_equal(r_c, r_o) and np.array_equal(d_c, d_o)


def test_mse_loss_and_scaled_vjp_match_torch():
    # Loss in the forward, gradient in the backward scaled by the incoming
    # cotangent on the device: compare with torch's fp32 MSE under a weight.
    import torch

    import diffrast
    g = torch.Generator().manual_seed(31)
    p = torch.randn(3, 37, 41, 5, generator=g).cuda().requires_grad_(True)
    t = torch.randn(3, 37, 41, 5, generator=g).cuda()
    p2 = p.detach().clone().requires_grad_(True)
    loss = diffrast.mse_loss(p, t)
    (loss * 3.5).backward()
    ref = torch.mean((p2 - t) ** 2)
    (ref * 3.5).backward()
    assert abs(float(loss.detach()) - float(ref.detach())) <= 1e-5 * abs(float(ref.detach()))
    assert torch.allclose(p.grad, p2.grad, rtol=1e-5, atol=1e-8)


def test_unused_outputs_get_no_materialised_cotangent(cu, soup):
    # out_da and rast_db off the loss path: the VJPs see None and give the
    # same gradients as the calls without those outputs.
    import torch

    import diffrast
    pos, tri = soup
    p1 = torch.from_numpy(pos).cuda().requires_grad_(True)
    p2 = torch.from_numpy(pos).cuda().requires_grad_(True)
    t = torch.from_numpy(tri).cuda()
    attr = torch.randn(pos.shape[1], 4, generator=torch.Generator().manual_seed(3)).cuda()
    r1, db1 = diffrast.rasterize(p1, t, (96, 128))
    o1, _ = diffrast.interpolate(attr, r1, t, rast_db=db1, diff_attrs="all")
    r2, _ = diffrast.rasterize(p2, t, (96, 128), grad_db=False)
    o2, _ = diffrast.interpolate(attr, r2, t)
    w = torch.randn(o1.shape, generator=torch.Generator().manual_seed(4)).cuda()
    (o1 * w).sum().backward()
    (o2 * w).sum().backward()
    assert torch.equal(r1, r2) and torch.equal(o1, o2)
    assert rel_l2(p1.grad.cpu().numpy(), p2.grad.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("C", [1, 4, 5])
@pytest.mark.parametrize("filt", ["linear", "linear-mipmap-linear", "cube"])
def test_texture_bwd_hot_texels_and_runs(cu, filt, C):
    # Whole warps sampling one texel (the constant-uv "background" block),
    # long runs of neighbours sharing texels (a magnified texture) and random
    # samples, with C = 1, 4 (the per-CTA hot-texel cache) and 5 (above it),
    # on a pixel count that is not a multiple of the block size.
    g = np.random.default_rng(40 + C)
    N, H, W = 2, 67, 93
    if filt == "cube":
        tex = g.random((1, 6, 16, 16, C)).astype(np.float32)
        d = g.normal(size=(N, H, W, 3)).astype(np.float32)
        d[:, :30] = np.array([0.2, -0.1, 1.0], np.float32)            # one texel of the +z face
        d[:, 30:50, :, 0] = np.linspace(-1, 1, W, dtype=np.float32)  # slow sweep: long runs
        d[:, 30:50, :, 1:] = np.array([0.1, 1.0], np.float32)
        kw = dict(boundary_mode="cube")
        uv = d
    else:
        tex = g.random((1, 32, 48, C)).astype(np.float32)
        uv = g.uniform(0, 1, size=(N, H, W, 2)).astype(np.float32)
        uv[:, :30] = 0.0                                              # background: one sample point
        uv[:, 30:50, :, 0] = np.linspace(0.2, 0.3, W, dtype=np.float32)  # magnified: runs of 20+ pixels
        uv[:, 30:50, :, 1] = 0.6
        mip = filt.startswith("linear-mipmap")
        da = (g.normal(size=(N, H, W, 4)) * 0.01).astype(np.float32)
        kw = dict(uv_da=da if mip else None, filter_mode=filt, boundary_mode="wrap")
    d_out = g.normal(size=(N, H, W, C)).astype(np.float32)
    ga = cu.texture_bwd(tex, uv, d_out, **kw)
    gb = O.texture_bwd(tex, uv, d_out, **kw)
    assert rel_l2(ga[0], gb[0]) < 1e-4


def test_antialias_ragged_pixel_count(cu, soup):
    # P = 3 * 37 * 53 is not a multiple of the block size: the last block's
    # lanes past the end take part in the warp-aggregated list appends without
    # adding entries.
    pos, tri = soup
    rast, _ = O.rasterize(pos, tri, (37, 53), grad_db=False)
    g = np.random.default_rng(41)
    color = g.normal(size=(3, 37, 53, 3)).astype(np.float32)
    topo = O.topology_hash(tri)
    a = cu.antialias(color, rast, pos, tri, topo)
    b = O.antialias(color, rast, pos, tri, topo)
    assert _rel_max(a, b) <= 1e-5
    d_out = g.normal(size=a.shape).astype(np.float32)
    ga = cu.antialias_bwd(color, rast, pos, tri, d_out, topo)
    gb = O.antialias_bwd(color, rast, pos, tri, d_out, topo)
    assert rel_l2(ga[0], gb[0]) < 1e-5 and rel_l2(ga[1], gb[1]) < 1e-4
