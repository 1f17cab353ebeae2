"""Full-chain forward+backward on the CPU oracle — TEST INFRASTRUCTURE ONLY.

The same chains as diffrast.chains (one per benchmark configuration), composed
from the oracle's restatement of the reference kernels, with the VJPs applied
explicitly in reverse order (what MLX's autograd does over the reference's
CustomFunctions).  Used as the parity checker of whole steps and as the timed
CPU baseline (a bounded sample of views).  Returns (loss, {name: gradient}).
"""
from __future__ import annotations

import numpy as np

from . import (antialias, antialias_bwd, interpolate, interpolate_bwd, mse_fwd_bwd, rasterize,
               rasterize_bwd, texture, texture_bwd, topology_hash)


def _mse(pred, target, nthreads):
    loss, d = mse_fwd_bwd(pred, target, 1.0 / pred.size, nthreads)
    return loss, d


def cfg1(pos, tri, rgb, target, res, topo=None, nthreads=0):
    topo = topology_hash(tri) if topo is None else topo
    rast, _ = rasterize(pos, tri, res, grad_db=False, nthreads=nthreads)
    col, _ = interpolate(rgb, rast, tri, nthreads=nthreads)
    aa = antialias(col, rast, pos, tri, topo, nthreads=nthreads)
    loss, d_aa = _mse(aa, target, nthreads)
    d_col, d_pos_aa = antialias_bwd(col, rast, pos, tri, d_aa, topo, nthreads=nthreads)
    d_rgb, d_rast, _ = interpolate_bwd(rgb, rast, tri, d_col, nthreads=nthreads)
    d_pos = rasterize_bwd(pos, tri, rast, d_rast, nthreads=nthreads) + d_pos_aa
    return loss, {"pos": d_pos, "rgb": d_rgb}


def cfg2(pos, tri, rgb_attr, uv_attr, tex, target, res, topo=None, nthreads=0):
    topo = topology_hash(tri) if topo is None else topo
    rast, _ = rasterize(pos, tri, res, grad_db=False, nthreads=nthreads)
    rgb, _ = interpolate(rgb_attr, rast, tri, nthreads=nthreads)
    uv, _ = interpolate(uv_attr, rast, tri, nthreads=nthreads)
    tc = texture(tex, uv, filter_mode="linear", boundary_mode="clamp", nthreads=nthreads)
    shade = (rgb * tc).astype(np.float32)
    aa = antialias(shade, rast, pos, tri, topo, nthreads=nthreads)
    loss, d_aa = _mse(aa, target, nthreads)
    d_shade, d_pos_aa = antialias_bwd(shade, rast, pos, tri, d_aa, topo, nthreads=nthreads)
    d_rgb_img = (d_shade * tc).astype(np.float32)
    d_tc = (d_shade * rgb).astype(np.float32)
    d_tex, d_uv, _, _ = texture_bwd(tex, uv, d_tc, filter_mode="linear", boundary_mode="clamp",
                                    nthreads=nthreads)
    d_uvattr, d_rast_uv, _ = interpolate_bwd(uv_attr, rast, tri, d_uv, nthreads=nthreads)
    d_rgb, d_rast_rgb, _ = interpolate_bwd(rgb_attr, rast, tri, d_rgb_img, nthreads=nthreads)
    d_pos = rasterize_bwd(pos, tri, rast, d_rast_uv + d_rast_rgb, nthreads=nthreads) + d_pos_aa
    return loss, {"pos": d_pos, "rgb": d_rgb, "uv": d_uvattr, "tex": d_tex}


def cfg3(pos, tri, uv_attr, tex, bias_map, target, res, nthreads=0):
    rast, db = rasterize(pos, tri, res, grad_db=True, nthreads=nthreads)
    uv, uvda = interpolate(uv_attr, rast, tri, rast_db=db, diff_attrs="all", nthreads=nthreads)
    f = "linear-mipmap-linear"
    col = texture(tex, uv, uvda, f, "wrap", 0.0, bias_map, nthreads=nthreads)
    loss, d_col = _mse(col, target, nthreads)
    d_tex, d_uv, d_uvda, _ = texture_bwd(tex, uv, d_col, uvda, f, "wrap", 0.0, bias_map, nthreads=nthreads)
    d_uvattr, d_rast, d_db = interpolate_bwd(uv_attr, rast, tri, d_uv, rast_db=db, diff_attrs="all",
                                             d_out_da=d_uvda, nthreads=nthreads)
    d_pos = rasterize_bwd(pos, tri, rast, d_rast, d_db, nthreads=nthreads)
    return loss, {"pos": d_pos, "uv": d_uvattr, "tex": d_tex}


def cfg4(pos, tri, attr, tgt0, tgt1, res, topo=None, nthreads=0):
    """pos [n, V, 4] (already transformed per view); returns d_pos per view."""
    topo = topology_hash(tri) if topo is None else topo
    rast0, db0 = rasterize(pos, tri, res, grad_db=True, nthreads=nthreads)
    rast1, db1 = rasterize(pos, tri, res, grad_db=True, peel_layer=rast0, nthreads=nthreads)
    out0, _ = interpolate(attr, rast0, tri, rast_db=db0, diff_attrs="all", nthreads=nthreads)
    out1, _ = interpolate(attr, rast1, tri, rast_db=db1, diff_attrs="all", nthreads=nthreads)
    aa0 = antialias(out0, rast0, pos, tri, topo, nthreads=nthreads)
    l0, d_aa0 = _mse(aa0, tgt0, nthreads)
    l1, d_out1 = _mse(out1, tgt1, nthreads)
    d_out0, d_pos_aa = antialias_bwd(out0, rast0, pos, tri, d_aa0, topo, nthreads=nthreads)
    zero_da = np.zeros(out0.shape[:3] + (2 * attr.shape[-1],), np.float32)
    d_attr0, d_rast0, d_db0 = interpolate_bwd(attr, rast0, tri, d_out0, rast_db=db0, diff_attrs="all",
                                              d_out_da=zero_da, nthreads=nthreads)
    d_attr1, d_rast1, d_db1 = interpolate_bwd(attr, rast1, tri, d_out1, rast_db=db1, diff_attrs="all",
                                              d_out_da=zero_da, nthreads=nthreads)
    d_pos = (rasterize_bwd(pos, tri, rast0, d_rast0, d_db0, nthreads=nthreads)
             + rasterize_bwd(pos, tri, rast1, d_rast1, d_db1, nthreads=nthreads) + d_pos_aa)
    return l0 + l1, {"pos": d_pos, "attr": d_attr0 + d_attr1}


def cfg5(pos, tri, nrm, cube, target, res, topo=None, nthreads=0, filter_mode="linear-mipmap-linear"):
    """filter_mode "linear" is the reference's cube mode; the mipmap filters
    take the normals' screen-space derivatives (rast_db, diff_attrs all)."""
    topo = topology_hash(tri) if topo is None else topo
    mip = filter_mode != "linear"
    rast, db = rasterize(pos, tri, res, grad_db=mip, nthreads=nthreads)
    d, dda = interpolate(nrm, rast, tri, rast_db=db if mip else None, diff_attrs="all" if mip else None,
                         nthreads=nthreads)
    # background pixels have a zero normal: look them up along +z
    d = (d + (rast[..., 3:] == 0).astype(np.float32) * np.array([0, 0, 1], np.float32)).astype(np.float32)
    col = texture(cube, d, dda if mip else None, filter_mode, "cube", nthreads=nthreads)
    aa = antialias(col, rast, pos, tri, topo, nthreads=nthreads)
    loss, d_aa = _mse(aa, target, nthreads)
    d_col, d_pos_aa = antialias_bwd(col, rast, pos, tri, d_aa, topo, nthreads=nthreads)
    d_cube, d_dir, d_dda, _ = texture_bwd(cube, d, d_col, dda if mip else None, filter_mode, "cube",
                                          nthreads=nthreads)
    if mip:
        d_nrm, d_rast, d_db = interpolate_bwd(nrm, rast, tri, d_dir, rast_db=db, diff_attrs="all", d_out_da=d_dda,
                                              nthreads=nthreads)
        d_pos = rasterize_bwd(pos, tri, rast, d_rast, d_db, nthreads=nthreads) + d_pos_aa
    else:
        d_nrm, d_rast, _ = interpolate_bwd(nrm, rast, tri, d_dir, nthreads=nthreads)
        d_pos = rasterize_bwd(pos, tri, rast, d_rast, nthreads=nthreads) + d_pos_aa
    return loss, {"pos": d_pos, "cube": d_cube}
