"""Parity against the reference's golden vectors: the nvdiffrast fixture
(Tests/MLXDiffRastTests/Fixtures/diffrast_fixtures.safetensors, restated in this
library's conventions by tests/golden/make_golden.py).  Runs on the oracle
(pinning it) and on the CUDA path."""
import numpy as np

from helpers import rel_l2


def test_rasterize_matches_nvdiffrast(backend, golden):
    g = golden
    rast, db = backend.rasterize(g["pos"], g["tri"], (16, 16))
    assert np.array_equal(rast[..., 3], g["rast"][..., 3])          # tri_id exact
    np.testing.assert_allclose(rast[..., :3], g["rast"][..., :3], atol=3e-7)
    np.testing.assert_allclose(db, g["rast_db"], atol=3e-7)


def test_rasterize_vjp_xy_matches_nvdiffrast(backend, golden):
    g = golden
    d_pos = backend.rasterize_bwd(g["pos"], g["tri"], (16, 16), g["co_rast"], g["co_rast_db"])
    assert rel_l2(d_pos[..., :2], g["d_pos_xy_from_rast"]) < 1e-5


def test_interpolate_matches_nvdiffrast(backend, golden):
    g = golden
    out, oda = backend.interpolate(g["attr"], g["rast"], g["tri"], rast_db=g["rast_db"], diff_attrs="all")
    np.testing.assert_allclose(out, g["interp_out"], atol=3e-7)
    np.testing.assert_allclose(oda, g["interp_out_da"], atol=3e-7)
    d_attr, d_rast, d_db = backend.interpolate_bwd(g["attr"], g["rast"], g["tri"], g["co_interp_out"],
                                                   rast_db=g["rast_db"], diff_attrs="all",
                                                   d_out_da=g["co_interp_out_da"])
    assert rel_l2(d_attr, g["d_attr_from_interp"]) < 1e-6
    np.testing.assert_allclose(d_rast, g["d_rast_from_interp"], atol=1e-6)
    np.testing.assert_allclose(d_db, g["d_rast_db_from_interp"], atol=1e-6)


def test_texture_bilinear_matches_nvdiffrast(backend, golden):
    # ParityTests.swift:92-100 (<= 1e-5); gradients to float noise.
    g = golden
    out = backend.texture(g["tex"], g["uv"], filter_mode="linear", boundary_mode="clamp")
    np.testing.assert_allclose(out, g["tex_bilinear"], atol=1e-6)
    d_tex, d_uv, _, _ = backend.texture_bwd(g["tex"], g["uv"], g["co_tex"], filter_mode="linear",
                                            boundary_mode="clamp")
    assert rel_l2(d_tex, g["d_tex_from_bilinear"]) < 1e-6
    np.testing.assert_allclose(d_uv, g["d_uv_from_bilinear"], atol=1e-6)


def test_texture_trilinear_matches_nvdiffrast(backend, golden):
    # ParityTests.swift:102-111 (<= 1e-4).  The fixture's LODs are all <= 0, so
    # it pins level 0 only (and a zero uvDA gradient).
    g = golden
    f = "linear-mipmap-linear"
    out = backend.texture(g["tex"], g["uv"], g["uv_da"], filter_mode=f, boundary_mode="clamp")
    np.testing.assert_allclose(out, g["tex_trilinear"], atol=1e-6)
    d_tex, d_uv, d_da, _ = backend.texture_bwd(g["tex"], g["uv"], g["co_tex"], g["uv_da"], filter_mode=f,
                                               boundary_mode="clamp")
    assert rel_l2(d_tex, g["d_tex_from_trilinear"]) < 1e-6
    np.testing.assert_allclose(d_uv, g["d_uv_from_trilinear"], atol=1e-6)
    np.testing.assert_allclose(d_da, g["d_uvDA_from_trilinear"], atol=1e-7)


def test_antialias_constant_colour_matches_nvdiffrast(backend, golden):
    g = golden
    rast, _ = backend.rasterize(g["pos"], g["tri"], (16, 16), grad_db=False)
    out = backend.antialias(g["aa_color"], rast, g["pos"], g["tri"])
    np.testing.assert_allclose(out, g["antialias_out"], atol=1e-7)
    _, d_pos = backend.antialias_bwd(g["aa_color"], rast, g["pos"], g["tri"], g["co_antialias"])
    np.testing.assert_allclose(d_pos, g["d_pos_from_antialias"], atol=1e-7)
