"""Regenerate tests/golden/nvdiffrast_fixture.npz from the reference's fixture.

The reference ships ``Tests/MLXDiffRastTests/Fixtures/diffrast_fixtures.safetensors``,
produced by real nvdiffrast on CUDA by ``scripts/diffrast_fixtures.py`` (16x16
image, 2 triangles, an 8x8x3 ramp texture).  nvdiffrast differs from
mlx-swift-diffrast in two documented conventions (CONVENTIONS.md:17-46 of the
reference): image y is flipped, and rast stores (w0, w1) instead of (w1, w2).
This script restates the fixture in this library's conventions so the tests can
compare directly, and writes a small .npz that travels with the repository (the
reference checkout is not present on GPU machines).

Remaps (our = this library, nv = nvdiffrast; all image tensors flipped on H):
  rast:     our.u = nv.v, our.v = 1 - nv.u - nv.v (0 on empty pixels),
            z and tri_id+1 unchanged
  rast_db:  (nv.dv/dx, -nv.dv/dy, -(nv.du/dx + nv.dv/dx), nv.du/dy + nv.dv/dy)
  interp_out:    flip only;  interp_out_da: flip, negate the d/dy channels
  d_rast (from interpolate): our = (G_v - G_u, -G_u) of nv's (G_u, G_v)
  d_rast_db (from interpolate): our = (G2 - G0, G1 - G3, -G0, G1)
  cotangents fed to our VJPs are the chain-rule images of nv's cotangents.
  d_pos_from_rast: only the x, y columns are comparable, with the z cotangent
  dropped (nvdiffrast does not differentiate through z, and its w column uses
  perspective-correct barycentrics while the reference's are screen-linear).
  antialias: the fixture's colour is constant, so out == colour and d_pos == 0
  in both libraries; d_color differs by algorithm and is not used.
  texture: convention-free (same uv input), stored unchanged.

Usage (the fixture is the reference checkout's
Tests/MLXDiffRastTests/Fixtures/diffrast_fixtures.safetensors):
    python tests/golden/make_golden.py path/to/diffrast_fixtures.safetensors
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def fixture_inputs():
    """Inputs rebuilt exactly as scripts/diffrast_fixtures.py:23-54 builds them."""
    pos = np.array([[[-0.7, 0.8, 0.0, 1.0], [0.8, 0.7, 0.1, 1.0],
                     [0.7, -0.8, 0.2, 1.0], [-0.8, -0.7, 0.0, 1.0]]], np.float32)
    tri = np.array([[0, 1, 2], [0, 2, 3]], np.int32)
    attr = np.array([[[1, 0, 0], [0, 1, 0], [0, 0, 1], [1, 1, 0]]], np.float32)
    Ht = Wt = 8
    tex = np.zeros((1, Ht, Wt, 3), np.float32)
    for y in range(Ht):
        for x in range(Wt):
            tex[0, y, x, 0] = np.float32(x / (Wt - 1))
            tex[0, y, x, 1] = np.float32(y / (Ht - 1))
            tex[0, y, x, 2] = np.float32((x + y) / (Wt + Ht - 2))
    return pos, tri, attr, tex


def flip(a):
    return np.ascontiguousarray(a[:, ::-1])


def convert(src):
    from safetensors.numpy import load_file

    d = load_file(src)
    pos, tri, attr, tex = fixture_inputs()
    g = {"pos": pos, "tri": tri, "attr": attr, "tex": tex}

    nv = flip(d["rast"])
    covered = nv[..., 3] > 0
    g["rast"] = np.stack([np.where(covered, nv[..., 1], 0.0),
                          np.where(covered, 1.0 - nv[..., 0] - nv[..., 1], 0.0),
                          nv[..., 2], nv[..., 3]], -1).astype(np.float32)
    ndb = flip(d["rast_db"])
    g["rast_db"] = np.stack([ndb[..., 2], -ndb[..., 3], -(ndb[..., 0] + ndb[..., 2]),
                             ndb[..., 1] + ndb[..., 3]], -1).astype(np.float32)

    # rasterize VJP goldens: cotangents mapped to our channels, z dropped.
    co = flip(d["co_rast"])
    g["co_rast"] = np.stack([co[..., 1] - co[..., 0], -co[..., 0], np.zeros_like(co[..., 2]),
                             np.zeros_like(co[..., 3])], -1).astype(np.float32)
    C = flip(d["co_rast_db"])
    g["co_rast_db"] = np.stack([C[..., 2] - C[..., 0], C[..., 1] - C[..., 3], -C[..., 0],
                                C[..., 1]], -1).astype(np.float32)
    g["d_pos_xy_from_rast"] = d["d_pos_from_rast"][..., :2].copy()

    # interpolate goldens
    g["interp_out"] = flip(d["interp_out"])
    oda = flip(d["interp_out_da"]).copy()
    oda[..., 1::2] *= -1.0
    g["interp_out_da"] = oda
    g["co_interp_out"] = flip(d["co_interp_out"])
    coda = flip(d["co_interp_out_da"]).copy()
    coda[..., 1::2] *= -1.0
    g["co_interp_out_da"] = coda
    g["d_attr_from_interp"] = d["d_attr_from_interp"].copy()
    G = flip(d["d_rast_from_interp"])
    g["d_rast_from_interp"] = np.stack([G[..., 1] - G[..., 0], -G[..., 0],
                                        np.zeros_like(G[..., 0]), np.zeros_like(G[..., 0])],
                                       -1).astype(np.float32)
    G = flip(d["d_rast_db_from_interp"])
    g["d_rast_db_from_interp"] = np.stack([G[..., 2] - G[..., 0], G[..., 1] - G[..., 3],
                                           -G[..., 0], G[..., 1]], -1).astype(np.float32)

    # texture goldens: convention-free
    for k in ["uv", "uv_da", "co_tex", "tex_bilinear", "d_tex_from_bilinear",
              "d_uv_from_bilinear", "tex_trilinear", "d_tex_from_trilinear",
              "d_uv_from_trilinear", "d_uvDA_from_trilinear"]:
        g[k] = d[k].copy()

    # antialias goldens (trivial: constant colour)
    g["aa_color"] = np.full((1, 16, 16, 3), 0.7, np.float32)
    g["co_antialias"] = flip(d["co_antialias"])
    g["antialias_out"] = flip(d["antialias_out"])
    g["d_pos_from_antialias"] = d["d_pos_from_antialias"].copy()
    return {k: np.ascontiguousarray(v) for k, v in g.items()}


def main():
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py path/to/diffrast_fixtures.safetensors")
    src = sys.argv[1]
    g = convert(src)
    out = os.path.join(HERE, "nvdiffrast_fixture.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out}: {len(g)} arrays")


if __name__ == "__main__":
    main()
