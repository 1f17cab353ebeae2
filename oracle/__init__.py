"""CPU parity oracle for the diffrast chain — TEST INFRASTRUCTURE ONLY.

numpy front end over ``libdiffrast_oracle.so`` (diffrast_oracle.cpp), the C++
restatement of mlx-swift-diffrast's Metal kernel arithmetic.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module; the CUDA library never calls it and has no CPU fallback.

Every function takes and returns C-contiguous numpy arrays (float32 / int32)
and mirrors one ``dr_*`` entry point of ``include/diffrast.h``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libdiffrast_oracle.so")
_lib = None

FILTERS = {"nearest": 0, "linear": 1, "linear-mipmap-nearest": 2, "linear-mipmap-linear": 3}
BOUNDARIES = {"wrap": 0, "clamp": 1, "zero": 2, "cube": 3}


def build() -> str:
    """Compile the oracle with its Makefile (idempotent); returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.orc_mse_fwd_bwd.restype = ctypes.c_double
    return _lib


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.int32)


def _nt(nthreads):
    return int(nthreads if nthreads else (os.cpu_count() or 1))


def _check(rc, name):
    if rc != 0:
        raise ValueError(f"oracle {name} rejected its arguments (rc={rc})")


# ---------------------------------------------------------------- rasterize

def rasterize(pos, tri, resolution, grad_db=True, ranges=None, peel_layer=None, nthreads=0):
    pos, tri, ranges, peel_layer = _f32(pos), _i32(tri), _i32(ranges), _f32(peel_layer)
    H, W = resolution
    if ranges is not None:
        N, V = ranges.shape[0], pos.shape[0]
    else:
        N, V = pos.shape[0], pos.shape[1]
    T = tri.shape[0]
    rast = np.zeros((N, H, W, 4), np.float32)
    db = np.zeros((N, H, W, 4), np.float32) if grad_db else None
    rc = lib().orc_rasterize_fwd(_p(pos), V, _p(tri), T, _p(ranges), N, H, W, _p(peel_layer),
                                 _p(rast), _p(db), _nt(nthreads))
    _check(rc, "rasterize_fwd")
    return rast, (db if grad_db else np.zeros((N, H, W, 0), np.float32))


def rasterize_bwd(pos, tri, rast, d_rast, d_rast_db=None, ranges=None, nthreads=0):
    pos, tri, ranges = _f32(pos), _i32(tri), _i32(ranges)
    rast, d_rast, d_rast_db = _f32(rast), _f32(d_rast), _f32(d_rast_db)
    N, H, W = rast.shape[:3]
    V = pos.shape[0] if ranges is not None else pos.shape[1]
    d_pos = np.zeros(pos.shape, np.float32)
    rc = lib().orc_rasterize_bwd(_p(pos), V, _p(tri), tri.shape[0], _p(ranges), N, H, W,
                                 _p(rast), _p(d_rast), _p(d_rast_db), _p(d_pos), _nt(nthreads))
    _check(rc, "rasterize_bwd")
    return d_pos


# -------------------------------------------------------------- interpolate

def _attr3(attr):
    attr = _f32(attr)
    return attr[None] if attr.ndim == 2 else attr


def _diff(diff_attrs, A):
    if diff_attrs is None:
        return None, 0
    if isinstance(diff_attrs, str) and diff_attrs == "all":
        return None, A
    idx = _i32(np.asarray(diff_attrs))
    return idx, int(idx.shape[0])


def interpolate(attr, rast, tri, rast_db=None, diff_attrs=None, nthreads=0):
    a3 = _attr3(attr)
    rast, tri, rast_db = _f32(rast), _i32(tri), _f32(rast_db)
    N, H, W = rast.shape[:3]
    Na, V, A = a3.shape
    idx, K = _diff(diff_attrs, A)
    out = np.zeros((N, H, W, A), np.float32)
    out_da = np.zeros((N, H, W, 2 * K), np.float32)
    rc = lib().orc_interpolate_fwd(_p(a3), Na, V, A, _p(rast), N, H, W, _p(tri), tri.shape[0],
                                   _p(rast_db), _p(idx), K, _p(out), _p(out_da) if K else None,
                                   _nt(nthreads))
    _check(rc, "interpolate_fwd")
    return out, out_da


def interpolate_bwd(attr, rast, tri, d_out, rast_db=None, diff_attrs=None, d_out_da=None,
                    nthreads=0):
    a3 = _attr3(attr)
    rast, tri, rast_db = _f32(rast), _i32(tri), _f32(rast_db)
    d_out, d_out_da = _f32(d_out), _f32(d_out_da)
    N, H, W = rast.shape[:3]
    Na, V, A = a3.shape
    idx, K = _diff(diff_attrs, A)
    d_attr = np.zeros(a3.shape, np.float32)
    d_rast = np.zeros((N, H, W, 4), np.float32)
    d_rast_db = np.zeros((N, H, W, 4), np.float32) if K else None
    rc = lib().orc_interpolate_bwd(_p(a3), Na, V, A, _p(rast), N, H, W, _p(tri), tri.shape[0],
                                   _p(rast_db), _p(idx), K, _p(d_out), _p(d_out_da), _p(d_attr),
                                   _p(d_rast), _p(d_rast_db), _nt(nthreads))
    _check(rc, "interpolate_bwd")
    d_attr = d_attr.reshape(np.shape(attr)) if np.ndim(attr) == 2 else d_attr
    return d_attr, d_rast, d_rast_db


# ------------------------------------------------------------------ texture

def mip_layout(Nt, Ht, Wt, C, max_level=-1):
    L = ctypes.c_int()
    off = (ctypes.c_int64 * 64)()
    hh = (ctypes.c_int * 64)()
    ww = (ctypes.c_int * 64)()
    tot = ctypes.c_int64()
    lib().orc_texture_mip_layout(Nt, Ht, Wt, C, max_level, ctypes.byref(L), off, hh, ww,
                                 ctypes.byref(tot))
    n = L.value
    return n, list(off[:n]), list(hh[:n]), list(ww[:n]), tot.value


def texture_construct_mip(tex, max_level=None, nthreads=0):
    tex = _f32(tex)
    Nt, Ht, Wt, C = tex.shape
    ml = -1 if max_level is None else int(max_level)
    L, off, hh, ww, tot = mip_layout(Nt, Ht, Wt, C, ml)
    pyr = np.zeros(max(tot, 1), np.float32)
    lib().orc_texture_construct_mip(_p(tex), Nt, Ht, Wt, C, ml, _p(pyr), _nt(nthreads))
    levels = [tex]
    for k in range(1, L):
        n = Nt * hh[k] * ww[k] * C
        levels.append(pyr[off[k]:off[k] + n].reshape(Nt, hh[k], ww[k], C))
    return levels


def _tex_dims(tex, boundary):
    if boundary == "cube":
        Nt, _, Ht, Wt, C = tex.shape
    else:
        Nt, Ht, Wt, C = tex.shape
    return Nt, Ht, Wt, C


def texture(tex, uv, uv_da=None, filter_mode="linear", boundary_mode="wrap",
            mip_level_bias=0.0, mip_level_bias_map=None, max_level=-1, nthreads=0):
    tex, uv, uv_da, bmap = _f32(tex), _f32(uv), _f32(uv_da), _f32(mip_level_bias_map)
    Nt, Ht, Wt, C = _tex_dims(tex, boundary_mode)
    N, Hi, Wi = uv.shape[:3]
    out = np.zeros((N, Hi, Wi, C), np.float32)
    rc = lib().orc_texture_fwd(FILTERS[filter_mode], BOUNDARIES[boundary_mode], _p(tex), Nt, Ht,
                               Wt, C, max_level, _p(uv), _p(uv_da), ctypes.c_float(mip_level_bias),
                               _p(bmap), N, Hi, Wi, _p(out), _nt(nthreads))
    _check(rc, "texture_fwd")
    return out


def texture_bwd(tex, uv, d_out, uv_da=None, filter_mode="linear", boundary_mode="wrap",
                mip_level_bias=0.0, mip_level_bias_map=None, max_level=-1, nthreads=0, cube_dir_grad=False):
    """cube_dir_grad: the d_dir chain rule through the cube projection
    (extension, flag bit 0x100 of the boundary code; the reference returns 0)."""
    tex, uv, uv_da, bmap, d_out = _f32(tex), _f32(uv), _f32(uv_da), _f32(mip_level_bias_map), _f32(d_out)
    Nt, Ht, Wt, C = _tex_dims(tex, boundary_mode)
    N, Hi, Wi = uv.shape[:3]
    d_tex = np.zeros(tex.shape, np.float32)
    d_uv = np.zeros(uv.shape, np.float32)
    mip = filter_mode.startswith("linear-mipmap")
    d_uv_da = np.zeros((N, Hi, Wi, 6 if boundary_mode == "cube" else 4), np.float32) if mip else None
    d_map = np.zeros((N, Hi, Wi), np.float32) if mip else None
    rc = lib().orc_texture_bwd(FILTERS[filter_mode], BOUNDARIES[boundary_mode] | (0x100 if cube_dir_grad else 0),
                               _p(tex), Nt, Ht,
                               Wt, C, max_level, _p(uv), _p(uv_da), ctypes.c_float(mip_level_bias),
                               _p(bmap), N, Hi, Wi, _p(d_out), _p(d_tex), _p(d_uv), _p(d_uv_da),
                               _p(d_map), _nt(nthreads))
    _check(rc, "texture_bwd")
    return d_tex, d_uv, d_uv_da, d_map


# ---------------------------------------------------------------- antialias

def topology_hash(tri):
    tri = _i32(tri)
    topo = np.zeros(tri.shape, np.int32)
    lib().orc_topology_hash(_p(tri), tri.shape[0], _p(topo))
    return topo


def antialias(color, rast, pos, tri, topology_hash_=None, nthreads=0):
    color, rast, pos, tri = _f32(color), _f32(rast), _f32(pos), _i32(tri)
    topo = topology_hash(tri) if topology_hash_ is None else _i32(topology_hash_)
    N, H, W, C = color.shape
    out = np.zeros(color.shape, np.float32)
    rc = lib().orc_antialias_fwd(_p(color), N, H, W, C, _p(rast), _p(pos), pos.shape[1], _p(tri),
                                 tri.shape[0], _p(topo), _p(out), _nt(nthreads))
    _check(rc, "antialias_fwd")
    return out


def antialias_bwd(color, rast, pos, tri, d_out, topology_hash_=None, nthreads=0):
    color, rast, pos, tri, d_out = _f32(color), _f32(rast), _f32(pos), _i32(tri), _f32(d_out)
    topo = topology_hash(tri) if topology_hash_ is None else _i32(topology_hash_)
    N, H, W, C = color.shape
    d_color = np.zeros(color.shape, np.float32)
    d_pos = np.zeros(pos.shape, np.float32)
    rc = lib().orc_antialias_bwd(_p(color), N, H, W, C, _p(rast), _p(pos), pos.shape[1], _p(tri),
                                 tri.shape[0], _p(topo), _p(d_out), _p(d_color), _p(d_pos),
                                 _nt(nthreads))
    _check(rc, "antialias_bwd")
    return d_color, d_pos


def mse_fwd_bwd(pred, target, scale, nthreads=0):
    pred, target = _f32(pred), _f32(target)
    d = np.zeros(pred.shape, np.float32)
    loss = lib().orc_mse_fwd_bwd(_p(pred), _p(target), ctypes.c_int64(pred.size),
                                 ctypes.c_float(scale), _p(d),
                                 _nt(nthreads))
    return loss, d


# ------------------------------------------------- per-view vertex transforms

def xf_positions(verts, xform):
    """Clip positions of the "xf" entry points: pos[n, v, r] =
    ((M[n,r,0] x + M[n,r,1] y) + M[n,r,2] z) + M[n,r,3] w, every product and
    sum rounded to float32 (the order include/diffrast.h specifies)."""
    v = np.ascontiguousarray(verts, np.float32)
    M = np.ascontiguousarray(xform, np.float32)
    out = np.empty((M.shape[0], v.shape[0], 4), np.float32)
    for r in range(4):
        acc = M[:, None, r, 0] * v[None, :, 0]
        acc = acc + M[:, None, r, 1] * v[None, :, 1]
        acc = acc + M[:, None, r, 2] * v[None, :, 2]
        acc = acc + M[:, None, r, 3] * v[None, :, 3]
        out[..., r] = acc
    return out


def xf_vertex_grad(d_pos, xform):
    """Gradient of the shared vertices from per-view clip gradients:
    d_verts[v] = sum_n M_n^T d_pos[n, v] (float64 accumulation)."""
    return np.einsum("nri,nvr->vi", np.asarray(xform, np.float64),
                     np.asarray(d_pos, np.float64)).astype(np.float32)


# ------------------------------------------------------- optimizer (examples)

def adam_step(param, grad, m, v, t, lr, beta1=0.9, beta2=0.999, eps=1e-8, mask=None):
    """Adam.swift:36-43 in float32, one IEEE operation at a time in the
    reference's order: returns (param, m, v) after step t (t >= 1).  `mask`
    multiplies the gradient first, as the PoseFit / MeshFit examples do."""
    f = np.float32
    g = np.asarray(grad, f)
    if mask is not None:
        g = (g * np.asarray(mask, f)).astype(f)
    b1, b2, lr, eps = f(beta1), f(beta2), f(lr), f(eps)
    m = (b1 * np.asarray(m, f) + (f(1) - b1) * g).astype(f)
    v = (b2 * np.asarray(v, f) + (f(1) - b2) * (g * g)).astype(f)
    c1 = f(1) - np.power(b1, f(t))
    c2 = f(1) - np.power(b2, f(t))
    m_hat = (m / c1).astype(f)
    v_hat = (v / c2).astype(f)
    p = (np.asarray(param, f) - (lr * m_hat) / (np.sqrt(v_hat) + eps)).astype(f)
    return p, m, v
