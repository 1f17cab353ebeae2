"""The DiffRast operator surface over libdiffrast's C ABI, for torch tensors.

Each op mirrors the Swift `DiffRast.*` function of mlx-swift-diffrast
(Sources/MLXDiffRast/*.swift): same argument names and meaning, same layouts
and conventions, same `precondition` checks (raised here as ValueError /
DiffRastError).  Forward and VJP are the explicit dr_*_fwd / dr_*_bwd pairs of
include/diffrast.h, bound into torch.autograd.Function; torch provides device
memory and the stream, every FLOP runs in the CUDA library.

Two small differences from the reference's host glue, both about avoiding work:
  * rasterize's VJP reuses the forward's rast instead of re-rasterizing
    (Rasterize.swift:109-116 re-runs the forward because MLX does not cache it);
  * broadcast inputs (attr [V,A] / [1,V,A], a batch-1 texture, range-mode pos)
    are read and accumulated in place instead of materialising N copies.
"""
from __future__ import annotations

import contextlib
import enum
from typing import Optional, Sequence, Union

import torch

from . import _lib as L


class BoundaryMode(enum.IntEnum):
    """DiffRast.BoundaryMode (Texture.swift:8-17)."""
    wrap = 0
    clamp = 1
    zero = 2
    cube = 3


# Flag bit of the boundary argument of dr_texture_bwd (DR_TEXTURE_CUBE_DIR_GRAD).
CUBE_DIR_GRAD = 0x100


class FilterMode(enum.IntEnum):
    """DiffRast.FilterMode (Texture.swift:35-40)."""
    nearest = 0
    linear = 1
    linearMipmapNearest = 2
    linearMipmapLinear = 3


class DiffAttrs:
    """DiffRast.DiffAttrs (Interpolate.swift:15-18): `.all` or `.indices([...])`."""

    def __init__(self, indices: Optional[Sequence[int]] = None):
        self._indices = None if indices is None else [int(i) for i in indices]

    @classmethod
    def indices(cls, idx: Sequence[int]) -> "DiffAttrs":
        return cls(list(idx))

    @property
    def is_all(self) -> bool:
        return self._indices is None

    def resolve(self, A: int):
        if self._indices is None:
            return None, A
        if len(self._indices) == 0:
            raise ValueError("interpolate: diffAttrs.indices must be non-empty")
        if not all(0 <= i < A for i in self._indices):
            raise ValueError(f"interpolate: diffAttrs.indices values must be in [0, A) (A={A})")
        return list(self._indices), len(self._indices)

    def __eq__(self, o):
        return isinstance(o, DiffAttrs) and self._indices == o._indices

    def __repr__(self):
        return "DiffAttrs.all" if self._indices is None else f"DiffAttrs.indices({self._indices})"


DiffAttrs.all = DiffAttrs(None)


def _as_diff(d) -> Optional[DiffAttrs]:
    if d is None or isinstance(d, DiffAttrs):
        return d
    if isinstance(d, str):
        if d == "all":
            return DiffAttrs.all
        raise ValueError(f"unknown diffAttrs {d!r}")
    return DiffAttrs.indices(d)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the library has no CPU path)")
    t = t.detach() if t.requires_grad else t
    if t.dtype != torch.float32:
        t = t.float()
    return t.contiguous()


def _i32(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the library has no CPU path)")
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t.contiguous()


def _ctx(t: torch.Tensor):
    dev = t.device.index if t.device.index is not None else torch.cuda.current_device()
    c = L.ctx_for(dev)
    L.lib().dr_ctx_set_stream(c, torch.cuda.current_stream(dev).cuda_stream)
    return c


# -------------------------------------------------------------- tile order
#
# No counterpart in the reference.  Interpolate gathers attribute rows by
# vertex and its VJP adds into a gradient table of the same shape; every view
# of a batch shows about the same triangles, so in image order each view
# sweeps both tables once, missing L2 on them again when they do not fit it
# together.  A tile order groups the batch's 32 x 8 tiles by the world region
# they show (a few regions, the views in order inside each), so one region's
# slice of the tables stays in L2 while every view passes over it.  Outputs
# do not depend on the order.

_TILE_ORDERS = {}  # device index -> (order tensor, (N, H, W)) the context holds


def tile_order(rast: torch.Tensor, pos: torch.Tensor, tri: torch.Tensor) -> torch.Tensor:
    """Processing order of rast's [N, H, W] batch of 32 x 8 pixel tiles grouped
    by the world region each shows (dr_tile_order): int32 [count], a
    permutation of the tile indices.  pos: [V, 4] vertices in one frame shared
    by all views (the per-view transform mode's shared vertices, or one view's
    clip-space positions); tri: [T, 3]."""
    rast_c = _f32(rast, "rast")
    pos_c = _f32(pos, "pos")
    tri_c = _i32(tri, "tri")
    if rast_c.dim() != 4 or rast_c.shape[3] != 4:
        raise ValueError(f"tile_order: rast must be [N, H, W, 4] (got {tuple(rast_c.shape)})")
    if pos_c.dim() != 2 or pos_c.shape[1] != 4:
        raise ValueError(f"tile_order: pos must be [V, 4] (got {tuple(pos_c.shape)})")
    N, H, W, _ = rast_c.shape
    order = torch.empty(int(L.lib().dr_tile_count(N, H, W)), dtype=torch.int32, device=rast_c.device)
    c = _ctx(rast_c)
    L.check(L.lib().dr_tile_order(c, _ptr(rast_c), N, H, W, _ptr(tri_c), tri_c.shape[0], _ptr(pos_c),
                                  pos_c.shape[0], _ptr(order)), c, "tile_order")
    return order


def set_tile_order(order: Optional[torch.Tensor], shape=None, device=None):
    """Make interpolate (forward and VJP, the _mse forms included) process
    batches of exactly shape = (N, H, W) pixels tile by tile in `order` (from
    tile_order); order=None restores image order on `device` (default: the
    current device).  The tensor is kept alive while it is set."""
    if order is None:
        dev = device if device is not None else torch.cuda.current_device()
        dev = dev.index if isinstance(dev, torch.device) else int(dev)
        c = L.ctx_for(dev)
        L.check(L.lib().dr_ctx_set_tile_order(c, None, 0, 0, 0), c, "set_tile_order")
        _TILE_ORDERS.pop(dev, None)
        return
    if shape is None or len(shape) != 3:
        raise ValueError("set_tile_order: shape must be (N, H, W)")
    N, H, W = (int(x) for x in shape)
    if order.dtype != torch.int32 or not order.is_cuda or not order.is_contiguous():
        raise ValueError("set_tile_order: order must be a contiguous int32 CUDA tensor from tile_order")
    if order.numel() != int(L.lib().dr_tile_count(N, H, W)):
        raise ValueError(f"set_tile_order: order has {order.numel()} entries, the batch has "
                         f"{int(L.lib().dr_tile_count(N, H, W))} tiles")
    c = _ctx(order)
    L.check(L.lib().dr_ctx_set_tile_order(c, _ptr(order), N, H, W), c, "set_tile_order")
    _TILE_ORDERS[order.device.index] = (order, (N, H, W))


@contextlib.contextmanager
def tile_order_scope(order: torch.Tensor, shape):
    """set_tile_order(order, shape) for the body of a with-statement (the
    backward passes run inside it too), image order again after it."""
    set_tile_order(order, shape)
    try:
        yield
    finally:
        set_tile_order(None, device=order.device)


# --------------------------------------------------------------- rasterize

class _Rasterize(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pos, tri, ranges, peel, H, W, grad_db):
        ctx.set_materialize_grads(False)  # outputs off the loss path get None, not zeros
        posc = _f32(pos, "pos")
        if ranges is not None:
            N, V = ranges.shape[0], posc.shape[0]
        else:
            N, V = posc.shape[0], posc.shape[1]
        T = tri.shape[0]
        rast = torch.empty((N, H, W, 4), device=posc.device, dtype=torch.float32)
        db = torch.empty((N, H, W, 4), device=posc.device, dtype=torch.float32) if grad_db else None
        c = _ctx(posc)
        L.check(L.lib().dr_rasterize_fwd(c, _ptr(posc), V, _ptr(tri), T, _ptr(ranges), N, H, W,
                                         _ptr(peel), _ptr(rast), _ptr(db)), c, "rasterize")
        ctx.save_for_backward(posc, tri, ranges, rast)
        ctx.dims = (N, V, T, H, W, grad_db)
        if db is None:
            db = torch.zeros((N, H, W, 0), device=posc.device, dtype=torch.float32)
        return rast, db

    @staticmethod
    def backward(ctx, d_rast, d_db):
        posc, tri, ranges, rast = ctx.saved_tensors
        N, V, T, H, W, grad_db = ctx.dims
        if d_rast is None and (d_db is None or not grad_db):
            return None, None, None, None, None, None, None
        if d_rast is None:
            d_rast = torch.zeros_like(rast)
        d_rast = d_rast.contiguous().float()
        d_db = d_db.contiguous().float() if (grad_db and d_db is not None) else None
        d_pos = torch.empty_like(posc)
        c = _ctx(posc)
        L.check(L.lib().dr_rasterize_bwd(c, _ptr(posc), V, _ptr(tri), T, _ptr(ranges), N, H, W,
                                         _ptr(rast), _ptr(d_rast), _ptr(d_db), _ptr(d_pos)),
                c, "rasterize_bwd")
        return d_pos, None, None, None, None, None, None


def rasterize(pos: torch.Tensor, tri: torch.Tensor, resolution, grad_db: bool = True,
              ranges: Optional[torch.Tensor] = None, peel_layer: Optional[torch.Tensor] = None):
    """DiffRast.rasterize (Rasterize.swift:44-144) -> (rast, rast_db).

    Instanced mode: pos [N, V, 4].  Range mode: pos [V, 4] and ranges [N, 2]
    int32 (start, count).  rast_db is [N, H, W, 0] when grad_db is False.
    """
    if tri.dim() != 2 or tri.shape[1] != 3:
        raise ValueError(f"rasterize: tri must be [T, 3] (got {tuple(tri.shape)})")
    H, W = int(resolution[0]), int(resolution[1])
    if ranges is not None:
        if pos.dim() != 2 or pos.shape[1] != 4:
            raise ValueError(f"rasterize: with `ranges`, pos must be [V, 4] (got {tuple(pos.shape)})")
        if ranges.dim() != 2 or ranges.shape[1] != 2:
            raise ValueError(f"rasterize: ranges must be [N, 2] (got {tuple(ranges.shape)})")
        ranges = _i32(ranges, "ranges")
        N = ranges.shape[0]
    else:
        if pos.dim() != 3 or pos.shape[2] != 4:
            raise ValueError(f"rasterize: pos must be [N, V, 4] (got {tuple(pos.shape)})")
        N = pos.shape[0]
    if peel_layer is not None:
        if tuple(peel_layer.shape) != (N, H, W, 4):
            raise ValueError("rasterize: peelLayer must match rast shape [N, H, W, 4] "
                             f"(got {tuple(peel_layer.shape)})")
        peel_layer = _f32(peel_layer, "peel_layer")
    return _Rasterize.apply(pos, _i32(tri, "tri"), ranges, peel_layer, H, W, bool(grad_db))


class _RasterizeLayers(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pos, xform, tri, ranges, H, W, grad_db, nl):
        ctx.set_materialize_grads(False)  # outputs off the loss path get None, not zeros
        import ctypes
        posc = _f32(pos, "pos")
        xf = _f32(xform, "xform") if xform is not None else None
        if xf is not None:
            N, V = xf.shape[0], posc.shape[0]
        elif ranges is not None:
            N, V = ranges.shape[0], posc.shape[0]
        else:
            N, V = posc.shape[0], posc.shape[1]
        T = tri.shape[0]
        rasts = [torch.empty((N, H, W, 4), device=posc.device, dtype=torch.float32) for _ in range(nl)]
        dbs = ([torch.empty((N, H, W, 4), device=posc.device, dtype=torch.float32) for _ in range(nl)]
               if grad_db else None)
        rp = (ctypes.c_void_p * nl)(*[r.data_ptr() for r in rasts])
        dp = (ctypes.c_void_p * nl)(*[d.data_ptr() for d in dbs]) if grad_db else None
        rpp = ctypes.cast(rp, ctypes.c_void_p)
        dpp = ctypes.cast(dp, ctypes.c_void_p) if dp is not None else None
        c = _ctx(posc)
        if xf is not None:
            L.check(L.lib().dr_rasterize_xf_fwd(c, _ptr(posc), V, _ptr(xf), _ptr(tri), T, N, H, W, nl, rpp, dpp),
                    c, "rasterize_xf")
        else:
            L.check(L.lib().dr_rasterize_layers_fwd(c, _ptr(posc), V, _ptr(tri), T, _ptr(ranges), N, H, W, nl,
                                                    rpp, dpp), c, "rasterize_layers")
        ctx.save_for_backward(posc, xf, tri, ranges, *rasts)
        ctx.dims = (N, V, T, H, W, grad_db, nl)
        if not grad_db:
            dbs = [torch.zeros((N, H, W, 0), device=posc.device, dtype=torch.float32) for _ in range(nl)]
        out = []
        for r, d in zip(rasts, dbs):
            out += [r, d]
        return tuple(out)

    @staticmethod
    def backward(ctx, *grads):
        import ctypes
        posc, xf, tri, ranges, *rasts = ctx.saved_tensors
        N, V, T, H, W, grad_db, nl = ctx.dims
        d_r = [g.contiguous().float() if g is not None else None for g in grads[0::2]]
        d_d = [g.contiguous().float() if (grad_db and g is not None) else None for g in grads[1::2]]
        # A layer whose rast_db reaches the loss but whose rast does not still
        # needs a (zero) rast cotangent; a layer reaching it by neither is skipped.
        d_r = [torch.zeros_like(rasts[l]) if (d_r[l] is None and d_d[l] is not None) else d_r[l]
               for l in range(nl)]
        if all(g is None for g in d_r):
            return None, None, None, None, None, None, None, None
        d_pos = torch.empty_like(posc)
        rp = ctypes.cast((ctypes.c_void_p * nl)(*[r.data_ptr() for r in rasts]), ctypes.c_void_p)
        gp = ctypes.cast((ctypes.c_void_p * nl)(*[(g.data_ptr() if g is not None else None) for g in d_r]),
                         ctypes.c_void_p)
        dp = ctypes.cast((ctypes.c_void_p * nl)(*[(g.data_ptr() if g is not None else None) for g in d_d]),
                         ctypes.c_void_p)
        c = _ctx(posc)
        if xf is not None:
            L.check(L.lib().dr_rasterize_xf_bwd(c, _ptr(posc), V, _ptr(xf), _ptr(tri), T, N, H, W, nl, rp, gp, dp,
                                                _ptr(d_pos)), c, "rasterize_xf_bwd")
        else:
            L.check(L.lib().dr_rasterize_layers_bwd(c, _ptr(posc), V, _ptr(tri), T, _ptr(ranges), N, H, W, nl,
                                                    rp, gp, dp, _ptr(d_pos)), c, "rasterize_layers_bwd")
        return d_pos, None, None, None, None, None, None, None


def rasterize_layers(pos: torch.Tensor, tri: torch.Tensor, resolution, num_layers: int, grad_db: bool = True,
                     ranges: Optional[torch.Tensor] = None, xform: Optional[torch.Tensor] = None):
    """Depth peeling of `num_layers` layers in one call: the same results as
    rasterize(...) followed by rasterize(..., peel_layer=previous) calls, with
    triangle setup and tile binning done once.  Returns [(rast, rast_db), ...].

    With `xform` [N, 4, 4], `pos` is a shared vertex buffer [V, 4] and view n
    rasterizes M_n @ pos (no [N, V, 4] tensor is materialised); the gradient
    flows to the shared vertices."""
    if tri.dim() != 2 or tri.shape[1] != 3:
        raise ValueError(f"rasterize: tri must be [T, 3] (got {tuple(tri.shape)})")
    if int(num_layers) < 1:
        raise ValueError("rasterize_layers: num_layers must be >= 1")
    H, W = int(resolution[0]), int(resolution[1])
    if xform is not None:
        if pos.dim() != 2 or pos.shape[1] != 4 or xform.dim() != 3 or tuple(xform.shape[1:]) != (4, 4):
            raise ValueError("rasterize: with `xform` [N, 4, 4], pos must be [V, 4]")
        if ranges is not None:
            raise ValueError("rasterize: `xform` and `ranges` are exclusive")
    elif ranges is not None:
        if pos.dim() != 2 or pos.shape[1] != 4:
            raise ValueError(f"rasterize: with `ranges`, pos must be [V, 4] (got {tuple(pos.shape)})")
        ranges = _i32(ranges, "ranges")
    elif pos.dim() != 3 or pos.shape[2] != 4:
        raise ValueError(f"rasterize: pos must be [N, V, 4] (got {tuple(pos.shape)})")
    outs = _RasterizeLayers.apply(pos, xform, _i32(tri, "tri"), ranges, H, W, bool(grad_db), int(num_layers))
    return [(outs[2 * l], outs[2 * l + 1]) for l in range(int(num_layers))]


# ------------------------------------------------------------- interpolate

class _Interpolate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, attr, rast, rast_db, tri, idx, K):
        ctx.set_materialize_grads(False)  # outputs off the loss path get None, not zeros
        attr_c = _f32(attr, "attr")
        a3 = attr_c if attr_c.dim() == 3 else attr_c.unsqueeze(0)
        rast_c = _f32(rast, "rast")
        db_c = _f32(rast_db, "rast_db") if K > 0 else None
        N, H, W = rast_c.shape[:3]
        Na, V, A = a3.shape
        out = torch.empty((N, H, W, A), device=rast_c.device, dtype=torch.float32)
        out_da = torch.empty((N, H, W, 2 * K), device=rast_c.device, dtype=torch.float32)
        arr = (ctypes_int_array(idx) if idx is not None else None)
        c = _ctx(rast_c)
        L.check(L.lib().dr_interpolate_fwd(c, _ptr(a3), Na, V, A, _ptr(rast_c), N, H, W, _ptr(tri),
                                           tri.shape[0], _ptr(db_c), arr, K, _ptr(out),
                                           _ptr(out_da) if K > 0 else None), c, "interpolate")
        ctx.save_for_backward(a3, rast_c, db_c, tri)
        ctx.meta = (idx, K, tuple(attr.shape))
        return out, out_da

    @staticmethod
    def backward(ctx, d_out, d_out_da):
        a3, rast_c, db_c, tri = ctx.saved_tensors
        idx, K, attr_shape = ctx.meta
        N, H, W = rast_c.shape[:3]
        Na, V, A = a3.shape
        if d_out is None and (d_out_da is None or K == 0):
            return None, None, None, None, None, None
        d_out = torch.zeros((N, H, W, A), device=rast_c.device) if d_out is None else d_out.contiguous().float()
        if K > 0 and d_out_da is None:
            # out_da did not reach the loss: its cotangent is zero, so the DA
            # terms of every gradient vanish; run the plain VJP.
            K, idx = 0, None
        d_out_da = d_out_da.contiguous().float() if K > 0 else None
        d_attr = torch.empty_like(a3)
        d_rast = torch.empty_like(rast_c)
        d_db = torch.empty_like(rast_c) if K > 0 else None
        arr = (ctypes_int_array(idx) if idx is not None else None)
        c = _ctx(rast_c)
        L.check(L.lib().dr_interpolate_bwd(c, _ptr(a3), Na, V, A, _ptr(rast_c), N, H, W, _ptr(tri),
                                           tri.shape[0], _ptr(db_c), arr, K, _ptr(d_out),
                                           _ptr(d_out_da), _ptr(d_attr), _ptr(d_rast), _ptr(d_db)),
                c, "interpolate_bwd")
        return d_attr.reshape(attr_shape), d_rast, d_db, None, None, None


def ctypes_int_array(values):
    import ctypes
    arr = (ctypes.c_int * len(values))(*values)
    return ctypes.cast(arr, ctypes.c_void_p)


def interpolate(attr: torch.Tensor, rast: torch.Tensor, tri: torch.Tensor,
                rast_db: Optional[torch.Tensor] = None,
                diff_attrs: Union[None, DiffAttrs, str, Sequence[int]] = None):
    """DiffRast.interpolate (Interpolate.swift:43-132) -> (out, out_da)."""
    if rast.dim() != 4 or rast.shape[3] != 4:
        raise ValueError(f"interpolate: rast must be [N, H, W, 4] (got {tuple(rast.shape)})")
    if tri.dim() != 2 or tri.shape[1] != 3:
        raise ValueError(f"interpolate: tri must be [T, 3] (got {tuple(tri.shape)})")
    if attr.dim() not in (2, 3):
        raise ValueError(f"interpolate: attr must be [V, A] or [N, V, A] (got {tuple(attr.shape)})")
    diff = _as_diff(diff_attrs)
    N = rast.shape[0]
    Na = 1 if attr.dim() == 2 else attr.shape[0]
    if Na != 1 and Na != N:
        raise ValueError(f"interpolate: attr batch dim {Na} incompatible with rast batch {N}")
    A = attr.shape[-1]
    if diff is not None:
        if rast_db is None:
            raise ValueError("interpolate: rastDB is required when diffAttrs is set")
        if tuple(rast_db.shape) != tuple(rast.shape):
            raise ValueError(f"interpolate: rastDB must match rast shape (got {tuple(rast_db.shape)} "
                             f"vs {tuple(rast.shape)})")
        idx, K = diff.resolve(A)
    else:
        idx, K, rast_db = None, 0, None
    return _Interpolate.apply(attr, rast, rast_db, _i32(tri, "tri"), idx, K)


# ----------------------------------------------------------------- texture

def _mip_layout(Nt, Ht, Wt, C, max_level):
    import ctypes
    n = ctypes.c_int()
    off = (ctypes.c_int64 * 32)()
    hh = (ctypes.c_int * 32)()
    ww = (ctypes.c_int * 32)()
    tot = ctypes.c_int64()
    st = L.lib().dr_texture_mip_layout(Nt, Ht, Wt, C, max_level, ctypes.byref(n), off, hh, ww,
                                       ctypes.byref(tot))
    if st != L.DR_OK:
        raise ValueError("textureConstructMip: bad texture shape")
    k = n.value
    return k, list(off[:k]), list(hh[:k]), list(ww[:k]), tot.value


def _build_pyramid(tex_c: torch.Tensor, max_level: int):
    Nt, Ht, Wt, C = tex_c.shape
    n, off, hh, ww, tot = _mip_layout(Nt, Ht, Wt, C, max_level)
    pyr = torch.empty(max(tot, 1), device=tex_c.device, dtype=torch.float32)
    c = _ctx(tex_c)
    L.check(L.lib().dr_texture_construct_mip(c, _ptr(tex_c), Nt, Ht, Wt, C, max_level, _ptr(pyr)),
            c, "textureConstructMip")
    return pyr, (n, off, hh, ww)


class _Texture(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tex, uv, uv_da, bias_map, filt, bnd, bias, dir_grad=False):
        ctx.set_materialize_grads(False)  # outputs off the loss path get None, not zeros
        tex_c = _f32(tex, "tex")
        uv_c = _f32(uv, "uv")
        da_c = _f32(uv_da, "uvDA") if uv_da is not None else None
        map_c = _f32(bias_map, "mipLevelBiasMap") if bias_map is not None else None
        cube = bnd == BoundaryMode.cube
        if cube:
            Nt, _, Ht, Wt, C = tex_c.shape
        else:
            Nt, Ht, Wt, C = tex_c.shape
        N, Hi, Wi = uv_c.shape[:3]
        mip = filt in (FilterMode.linearMipmapNearest, FilterMode.linearMipmapLinear)
        pyr = None
        if mip:  # a cube's pyramid is that of its Nt * 6 faces
            pyr, _ = _build_pyramid(tex_c.view(-1, Ht, Wt, C) if cube else tex_c, -1)
        out = torch.empty((N, Hi, Wi, C), device=uv_c.device, dtype=torch.float32)
        c = _ctx(uv_c)
        L.check(L.lib().dr_texture_fwd(c, int(filt), int(bnd), _ptr(tex_c), Nt, Ht, Wt, C, _ptr(pyr), -1,
                                       _ptr(uv_c), _ptr(da_c), float(bias), _ptr(map_c), N, Hi, Wi,
                                       _ptr(out)), c, "texture")
        ctx.save_for_backward(tex_c, uv_c, da_c, map_c, pyr)
        ctx.meta = (int(filt), int(bnd) | (CUBE_DIR_GRAD if dir_grad else 0), float(bias), (Nt, Ht, Wt, C, N, Hi, Wi),
                    tuple(map_c.shape) if map_c is not None else None)
        return out

    @staticmethod
    def backward(ctx, d_out):
        tex_c, uv_c, da_c, map_c, pyr = ctx.saved_tensors
        filt, bnd, bias, (Nt, Ht, Wt, C, N, Hi, Wi), map_shape = ctx.meta
        if d_out is None:
            return None, None, None, None, None, None, None, None
        d_out = d_out.contiguous().float()
        d_tex = torch.empty_like(tex_c)
        d_uv = torch.empty_like(uv_c)
        mip = filt in (FilterMode.linearMipmapNearest, FilterMode.linearMipmapLinear)
        d_da = torch.empty_like(da_c) if (mip and ctx.needs_input_grad[2]) else None
        d_map = (torch.empty((N, Hi, Wi), device=uv_c.device, dtype=torch.float32)
                 if (mip and map_c is not None and ctx.needs_input_grad[3]) else None)
        c = _ctx(uv_c)
        L.check(L.lib().dr_texture_bwd(c, filt, bnd, _ptr(tex_c), Nt, Ht, Wt, C, _ptr(pyr), -1, _ptr(uv_c),
                                       _ptr(da_c), float(bias), _ptr(map_c), N, Hi, Wi, _ptr(d_out),
                                       _ptr(d_tex), _ptr(d_uv), _ptr(d_da), _ptr(d_map)),
                c, "texture_bwd")
        if d_map is not None:
            d_map = d_map.reshape(map_shape)
        return d_tex, d_uv, d_da, d_map, None, None, None, None


def texture(tex: torch.Tensor, uv: torch.Tensor, uv_da: Optional[torch.Tensor] = None,
            filter_mode: FilterMode = FilterMode.linear, boundary_mode: BoundaryMode = BoundaryMode.wrap,
            mip_level_bias: float = 0.0, mip_level_bias_map: Optional[torch.Tensor] = None, *,
            cube_dir_grad: bool = False):
    """DiffRast.texture (Texture.swift:62-131).

    cube_dir_grad (extension, cube textures only): the direction receives the
    chain rule through the face projection (and, for the mipmap filters, the
    LOD) instead of the reference's zero gradient (Texture.swift:196-197).
    """
    filt, bnd = FilterMode(filter_mode), BoundaryMode(boundary_mode)
    if cube_dir_grad and bnd != BoundaryMode.cube:
        raise ValueError("texture: cube_dir_grad applies to cube textures only")
    if bnd == BoundaryMode.cube:
        # .linear as the reference; the mipmap filters are an extension that
        # takes the direction's derivatives dirDA [N, H_img, W_img, 6]
        # (interpolate's diff_attrs layout for a 3-component direction).
        if filt == FilterMode.nearest:
            raise ValueError("texture: cube textures support the linear and mipmap filterModes")
        if tex.dim() != 5 or tex.shape[1] != 6:
            raise ValueError(f"texture: cube tex must be [N, 6, H, W, C] (got {tuple(tex.shape)})")
        if uv.dim() != 4 or uv.shape[3] != 3:
            raise ValueError("texture: cube uv must be [N, H_img, W_img, 3] direction vector "
                             f"(got {tuple(uv.shape)})")
        if tex.shape[0] not in (1, uv.shape[0]):
            raise ValueError("texture: tex batch dim incompatible with uv batch")
        if filt == FilterMode.linear:
            return _Texture.apply(tex, uv, None, None, filt, bnd, 0.0, cube_dir_grad)
        if uv_da is None:
            raise ValueError("texture: mipmap filterModes require uvDA")
        if tuple(uv_da.shape) != tuple(uv.shape[:3]) + (6,):
            raise ValueError(f"texture: cube uvDA must be [N, H_img, W_img, 6] (got {tuple(uv_da.shape)})")
        _check_bias_map(mip_level_bias_map, uv)
        return _Texture.apply(tex, uv, uv_da, mip_level_bias_map, filt, bnd, float(mip_level_bias), cube_dir_grad)
    if tex.dim() != 4:
        raise ValueError(f"texture: tex must be [N, H_tex, W_tex, C] (got {tuple(tex.shape)})")
    if uv.dim() != 4 or uv.shape[3] != 2:
        raise ValueError(f"texture: uv must be [N, H_img, W_img, 2] (got {tuple(uv.shape)})")
    if tex.shape[0] != 1 and tex.shape[0] != uv.shape[0]:
        raise ValueError(f"texture: tex batch dim {tex.shape[0]} incompatible with uv batch {uv.shape[0]}")
    if filt in (FilterMode.nearest, FilterMode.linear):
        return _Texture.apply(tex, uv, None, None, filt, bnd, 0.0)
    if uv_da is None:
        raise ValueError("texture: mipmap filterModes require uvDA")
    if tuple(uv_da.shape) != tuple(uv.shape[:3]) + (4,):
        raise ValueError(f"texture: uvDA must be [N, H_img, W_img, 4] (got {tuple(uv_da.shape)})")
    _check_bias_map(mip_level_bias_map, uv)
    return _Texture.apply(tex, uv, uv_da, mip_level_bias_map, filt, bnd, float(mip_level_bias))


def _check_bias_map(m, uv):
    if m is not None:
        if tuple(m.shape[:3]) != tuple(uv.shape[:3]) or not (m.dim() == 3 or (m.dim() == 4 and m.shape[3] == 1)):
            raise ValueError("texture: mipLevelBiasMap must be [N, H_img, W_img] or [N, H_img, W_img, 1] "
                             f"(got {tuple(m.shape)})")


def texture_construct_mip(tex: torch.Tensor, max_level: Optional[int] = None):
    """DiffRast.textureConstructMip (Texture.swift:144-161): [level0 = tex, level1, ...].

    Forward only (the levels are views of one pyramid buffer); gradients of
    mipmapped sampling flow through `texture`, which folds them into the texture.
    """
    if tex.dim() != 4:
        raise ValueError(f"textureConstructMip: tex must be [N, H, W, C] (got {tuple(tex.shape)})")
    tex_c = _f32(tex, "tex")
    ml = -1 if max_level is None else int(max_level)
    pyr, (n, off, hh, ww) = _build_pyramid(tex_c, ml)
    Nt, _, _, C = tex_c.shape
    levels = [tex]
    for k in range(1, n):
        cnt = Nt * hh[k] * ww[k] * C
        levels.append(pyr[off[k]:off[k] + cnt].view(Nt, hh[k], ww[k], C))
    return levels


# --------------------------------------------------------------- antialias

def antialias_construct_topology_hash(tri: torch.Tensor) -> torch.Tensor:
    """DiffRast.antialiasConstructTopologyHash (Antialias.swift:19-66), on the GPU."""
    if tri.dim() != 2 or tri.shape[1] != 3:
        raise ValueError(f"antialiasConstructTopologyHash: tri must be [T, 3] (got {tuple(tri.shape)})")
    tri_c = _i32(tri, "tri")
    topo = torch.empty_like(tri_c)
    c = _ctx(tri_c)
    L.check(L.lib().dr_antialias_construct_topology_hash(c, _ptr(tri_c), tri_c.shape[0], _ptr(topo)),
            c, "antialiasConstructTopologyHash")
    return topo


class _Antialias(torch.autograd.Function):
    @staticmethod
    def forward(ctx, color, pos, xform, rast, tri, topo):
        ctx.set_materialize_grads(False)  # outputs off the loss path get None, not zeros
        color_c = _f32(color, "color")
        pos_c = _f32(pos, "pos")
        xf = _f32(xform, "xform") if xform is not None else None
        rast_c = _f32(rast, "rast")
        N, H, W, C = color_c.shape
        V, T = (pos_c.shape[0] if xf is not None else pos_c.shape[1]), tri.shape[0]
        out = torch.empty_like(color_c)
        c = _ctx(color_c)
        # The forward records each pixel's silhouettes for the VJP (17 B/px)
        # when a gradient will be asked for; the VJP then skips the search.
        work = None
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
            work = torch.empty(L.lib().dr_antialias_work_bytes(N, H, W), dtype=torch.uint8, device=color_c.device)
        if xf is not None:
            L.check(L.lib().dr_antialias_xf_fwd(c, _ptr(color_c), N, H, W, C, _ptr(rast_c), _ptr(pos_c), V, _ptr(xf),
                                                _ptr(tri), T, _ptr(topo), _ptr(out), _ptr(work)), c, "antialias_xf")
        else:
            L.check(L.lib().dr_antialias_fwd(c, _ptr(color_c), N, H, W, C, _ptr(rast_c), _ptr(pos_c), V, _ptr(tri),
                                             T, _ptr(topo), _ptr(out), _ptr(work)), c, "antialias")
        ctx.save_for_backward(color_c, pos_c, xf, rast_c, tri, topo, work)
        return out

    @staticmethod
    def backward(ctx, d_out):
        color_c, pos_c, xf, rast_c, tri, topo, work = ctx.saved_tensors
        if d_out is None:
            return None, None, None, None, None, None
        N, H, W, C = color_c.shape
        V, T = (pos_c.shape[0] if xf is not None else pos_c.shape[1]), tri.shape[0]
        d_out = d_out.contiguous().float()
        d_color = torch.empty_like(color_c)
        d_pos = torch.empty_like(pos_c)
        c = _ctx(color_c)
        if xf is not None:
            L.check(L.lib().dr_antialias_xf_bwd(c, _ptr(color_c), N, H, W, C, _ptr(rast_c), _ptr(pos_c), V, _ptr(xf),
                                                _ptr(tri), T, _ptr(topo), _ptr(d_out), _ptr(d_color), _ptr(d_pos),
                                                _ptr(work)), c, "antialias_xf_bwd")
        else:
            L.check(L.lib().dr_antialias_bwd(c, _ptr(color_c), N, H, W, C, _ptr(rast_c), _ptr(pos_c), V, _ptr(tri),
                                             T, _ptr(topo), _ptr(d_out), _ptr(d_color), _ptr(d_pos), _ptr(work)),
                    c, "antialias_bwd")
        return d_color, d_pos, None, None, None, None


def antialias(color: torch.Tensor, rast: torch.Tensor, pos: torch.Tensor, tri: torch.Tensor,
              topology_hash: Optional[torch.Tensor] = None, xform: Optional[torch.Tensor] = None) -> torch.Tensor:
    """DiffRast.antialias (Antialias.swift:90-131); differentiable w.r.t. color and pos.

    With `xform` [N, 4, 4], `pos` is the shared vertex buffer [V, 4] and view n
    uses M_n @ pos (as rasterize_layers(xform=...))."""
    if color.dim() != 4:
        raise ValueError(f"antialias: color must be [N, H, W, C] (got {tuple(color.shape)})")
    if rast.dim() != 4 or rast.shape[3] != 4 or tuple(rast.shape[:3]) != tuple(color.shape[:3]):
        raise ValueError("antialias: rast must match color in [N, H, W] and have 4 channels")
    if xform is not None:
        if pos.dim() != 2 or pos.shape[1] != 4 or tuple(xform.shape) != (color.shape[0], 4, 4):
            raise ValueError("antialias: with `xform` [N, 4, 4], pos must be [V, 4]")
    else:
        if pos.dim() != 3 or pos.shape[2] != 4:
            raise ValueError(f"antialias: pos must be [N, V, 4] (got {tuple(pos.shape)})")
        if pos.shape[0] != color.shape[0]:
            raise ValueError("antialias: pos batch must match color batch")
    if tri.dim() != 2 or tri.shape[1] != 3:
        raise ValueError(f"antialias: tri must be [T, 3] (got {tuple(tri.shape)})")
    tri_c = _i32(tri, "tri")
    topo = antialias_construct_topology_hash(tri_c) if topology_hash is None else _i32(topology_hash, "topologyHash")
    return _Antialias.apply(color, pos, xform, rast.detach(), tri_c, topo)


# -------------------------------------------------------------------- loss

class _MSE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target):
        p = _f32(pred, "pred")
        t = _f32(target, "target")
        n = p.numel()
        loss = torch.empty((), device=p.device, dtype=torch.float32)
        c = _ctx(p)
        # Loss only; the gradient is formed in backward, scaled there by the
        # incoming cotangent read on the device (no extra pass over d_pred).
        L.check(L.lib().dr_mse_fwd_bwd(c, _ptr(p), _ptr(t), n, 1.0 / max(n, 1), None, _ptr(loss), 1), c, "mse")
        ctx.save_for_backward(p, t)
        return loss

    @staticmethod
    def backward(ctx, g):
        p, t = ctx.saved_tensors
        if g is None:
            return None, None
        g = g.contiguous().float()
        d = torch.empty_like(p)
        c = _ctx(p)
        L.check(L.lib().dr_mse_bwd(c, _ptr(p), _ptr(t), p.numel(), 1.0 / max(p.numel(), 1), _ptr(g), _ptr(d)),
                c, "mse_bwd")
        return d, None


def mse_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """mean((pred - target)^2) with its gradient computed in the same kernel."""
    return _MSE.apply(pred, target)


# ------------------------------------------------- ops fused with the loss
#
# The reference's examples render and then take mean((image - target)^2)
# (ColorFitExample/main.swift:57-60).  When an op's output feeds only that
# loss, the *_mse ops compute it in the op's own kernels: the forward adds the
# loss while it writes the output, and the VJP forms the output's cotangent
# 2 (out - target) / numel * d_loss where it reads it, so neither a separate
# loss pass nor a materialised d_out runs.  The output is returned for
# inspection and is not differentiable: gradients flow through the loss only.

def _check_target(target: torch.Tensor, like: torch.Tensor, name: str) -> torch.Tensor:
    if tuple(target.shape) != tuple(like.shape):
        raise ValueError(f"{name}: target must have the output's shape {tuple(like.shape)} "
                         f"(got {tuple(target.shape)})")
    return _f32(target, "target")


class _AntialiasMSE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, color, pos, xform, rast, tri, topo, target):
        ctx.set_materialize_grads(False)
        color_c = _f32(color, "color")
        pos_c = _f32(pos, "pos")
        xf = _f32(xform, "xform") if xform is not None else None
        rast_c = _f32(rast, "rast")
        tgt = _check_target(target, color_c, "antialias_mse")
        N, H, W, C = color_c.shape
        V, T = (pos_c.shape[0] if xf is not None else pos_c.shape[1]), tri.shape[0]
        out = torch.empty_like(color_c)
        loss = torch.empty((), device=color_c.device, dtype=torch.float32)
        scale = 1.0 / max(out.numel(), 1)
        c = _ctx(color_c)
        work = None
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
            work = torch.empty(L.lib().dr_antialias_work_bytes(N, H, W), dtype=torch.uint8, device=color_c.device)
        if xf is not None:
            L.check(L.lib().dr_antialias_xf_fwd_mse(c, _ptr(color_c), N, H, W, C, _ptr(rast_c), _ptr(pos_c), V,
                                                    _ptr(xf), _ptr(tri), T, _ptr(topo), _ptr(out), _ptr(work),
                                                    _ptr(tgt), scale, _ptr(loss)), c, "antialias_xf_mse")
        else:
            L.check(L.lib().dr_antialias_fwd_mse(c, _ptr(color_c), N, H, W, C, _ptr(rast_c), _ptr(pos_c), V,
                                                 _ptr(tri), T, _ptr(topo), _ptr(out), _ptr(work), _ptr(tgt), scale,
                                                 _ptr(loss)), c, "antialias_mse")
        ctx.save_for_backward(color_c, pos_c, xf, rast_c, tri, topo, work, out, tgt)
        ctx.scale = scale
        ctx.mark_non_differentiable(out)
        return loss, out

    @staticmethod
    def backward(ctx, d_loss, _d_out):
        color_c, pos_c, xf, rast_c, tri, topo, work, out, tgt = ctx.saved_tensors
        if d_loss is None:
            return None, None, None, None, None, None, None
        N, H, W, C = color_c.shape
        V, T = (pos_c.shape[0] if xf is not None else pos_c.shape[1]), tri.shape[0]
        g = d_loss.contiguous().float()
        d_color = torch.empty_like(color_c)
        d_pos = torch.empty_like(pos_c)
        c = _ctx(color_c)
        if xf is not None:
            L.check(L.lib().dr_antialias_xf_bwd_mse(c, _ptr(color_c), N, H, W, C, _ptr(rast_c), _ptr(pos_c), V,
                                                    _ptr(xf), _ptr(tri), T, _ptr(topo), _ptr(out), _ptr(tgt),
                                                    ctx.scale, _ptr(g), _ptr(d_color), _ptr(d_pos), _ptr(work)),
                    c, "antialias_xf_bwd_mse")
        else:
            L.check(L.lib().dr_antialias_bwd_mse(c, _ptr(color_c), N, H, W, C, _ptr(rast_c), _ptr(pos_c), V,
                                                 _ptr(tri), T, _ptr(topo), _ptr(out), _ptr(tgt), ctx.scale, _ptr(g),
                                                 _ptr(d_color), _ptr(d_pos), _ptr(work)), c, "antialias_bwd_mse")
        return d_color, d_pos, None, None, None, None, None


def antialias_mse(color: torch.Tensor, rast: torch.Tensor, pos: torch.Tensor, tri: torch.Tensor,
                  target: torch.Tensor, topology_hash: Optional[torch.Tensor] = None,
                  xform: Optional[torch.Tensor] = None):
    """mean((antialias(color, rast, pos, tri) - target)^2) computed inside the
    antialias kernels -> (loss, out).  Arguments as antialias(); the loss is
    differentiable w.r.t. color and pos, out is not."""
    if color.dim() != 4:
        raise ValueError(f"antialias: color must be [N, H, W, C] (got {tuple(color.shape)})")
    if rast.dim() != 4 or rast.shape[3] != 4 or tuple(rast.shape[:3]) != tuple(color.shape[:3]):
        raise ValueError("antialias: rast must match color in [N, H, W] and have 4 channels")
    if xform is not None:
        if pos.dim() != 2 or pos.shape[1] != 4 or tuple(xform.shape) != (color.shape[0], 4, 4):
            raise ValueError("antialias: with `xform` [N, 4, 4], pos must be [V, 4]")
    elif pos.dim() != 3 or pos.shape[2] != 4 or pos.shape[0] != color.shape[0]:
        raise ValueError(f"antialias: pos must be [N, V, 4] (got {tuple(pos.shape)})")
    if tri.dim() != 2 or tri.shape[1] != 3:
        raise ValueError(f"antialias: tri must be [T, 3] (got {tuple(tri.shape)})")
    tri_c = _i32(tri, "tri")
    topo = antialias_construct_topology_hash(tri_c) if topology_hash is None else _i32(topology_hash, "topologyHash")
    return _AntialiasMSE.apply(color, pos, xform, rast.detach(), tri_c, topo, target)


class _InterpolateMSE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, attr, rast, rast_db, tri, idx, K, target):
        ctx.set_materialize_grads(False)
        attr_c = _f32(attr, "attr")
        a3 = attr_c if attr_c.dim() == 3 else attr_c.unsqueeze(0)
        rast_c = _f32(rast, "rast")
        db_c = _f32(rast_db, "rast_db") if K > 0 else None
        N, H, W = rast_c.shape[:3]
        Na, V, A = a3.shape
        out = torch.empty((N, H, W, A), device=rast_c.device, dtype=torch.float32)
        out_da = torch.empty((N, H, W, 2 * K), device=rast_c.device, dtype=torch.float32)
        tgt = _check_target(target, out, "interpolate_mse")
        loss = torch.empty((), device=rast_c.device, dtype=torch.float32)
        scale = 1.0 / max(out.numel(), 1)
        arr = (ctypes_int_array(idx) if idx is not None else None)
        c = _ctx(rast_c)
        L.check(L.lib().dr_interpolate_fwd_mse(c, _ptr(a3), Na, V, A, _ptr(rast_c), N, H, W, _ptr(tri),
                                               tri.shape[0], _ptr(db_c), arr, K, _ptr(out),
                                               _ptr(out_da) if K > 0 else None, _ptr(tgt), scale, _ptr(loss)),
                c, "interpolate_mse")
        ctx.save_for_backward(a3, rast_c, db_c, tri, out, tgt)
        ctx.meta = (idx, K, tuple(attr.shape), scale)
        ctx.mark_non_differentiable(out)
        return loss, out, out_da

    @staticmethod
    def backward(ctx, d_loss, _d_out, d_out_da):
        a3, rast_c, db_c, tri, out, tgt = ctx.saved_tensors
        idx, K, attr_shape, scale = ctx.meta
        N, H, W = rast_c.shape[:3]
        Na, V, A = a3.shape
        if d_loss is None and (d_out_da is None or K == 0):
            return None, None, None, None, None, None, None
        g = torch.zeros((), device=rast_c.device) if d_loss is None else d_loss.contiguous().float()
        if K > 0 and d_out_da is None:
            K, idx = 0, None  # out_da is off the loss path: no DA terms
        d_out_da = d_out_da.contiguous().float() if K > 0 else None
        d_attr = torch.empty_like(a3)
        d_rast = torch.empty_like(rast_c)
        d_db = torch.empty_like(rast_c) if K > 0 else None
        arr = (ctypes_int_array(idx) if idx is not None else None)
        c = _ctx(rast_c)
        L.check(L.lib().dr_interpolate_bwd_mse(c, _ptr(a3), Na, V, A, _ptr(rast_c), N, H, W, _ptr(tri),
                                               tri.shape[0], _ptr(db_c), arr, K, _ptr(out), _ptr(tgt), scale,
                                               _ptr(g), _ptr(d_out_da), _ptr(d_attr), _ptr(d_rast), _ptr(d_db)),
                c, "interpolate_bwd_mse")
        return d_attr.reshape(attr_shape), d_rast, d_db, None, None, None, None


def interpolate_mse(attr: torch.Tensor, rast: torch.Tensor, tri: torch.Tensor, target: torch.Tensor,
                    rast_db: Optional[torch.Tensor] = None,
                    diff_attrs: Union[None, DiffAttrs, str, Sequence[int]] = None):
    """mean((interpolate(attr, rast, tri, ...).out - target)^2) computed inside
    the interpolate kernels -> (loss, out, out_da).  Arguments as
    interpolate(); the loss and out_da are differentiable, out is not."""
    if rast.dim() != 4 or rast.shape[3] != 4:
        raise ValueError(f"interpolate: rast must be [N, H, W, 4] (got {tuple(rast.shape)})")
    if tri.dim() != 2 or tri.shape[1] != 3:
        raise ValueError(f"interpolate: tri must be [T, 3] (got {tuple(tri.shape)})")
    if attr.dim() not in (2, 3):
        raise ValueError(f"interpolate: attr must be [V, A] or [N, V, A] (got {tuple(attr.shape)})")
    diff = _as_diff(diff_attrs)
    N = rast.shape[0]
    Na = 1 if attr.dim() == 2 else attr.shape[0]
    if Na != 1 and Na != N:
        raise ValueError(f"interpolate: attr batch dim {Na} incompatible with rast batch {N}")
    A = attr.shape[-1]
    if diff is not None:
        if rast_db is None:
            raise ValueError("interpolate: rastDB is required when diffAttrs is set")
        idx, K = diff.resolve(A)
    else:
        idx, K, rast_db = None, 0, None
    return _InterpolateMSE.apply(attr, rast, rast_db, _i32(tri, "tri"), idx, K, target)


# ------------------------------------ rasterize + interpolate, fused forward
#
# No counterpart in the reference (rasterize and interpolate are separate
# operators there).  Two depth layers of the per-view transform mode with
# interpolate (.all derivatives) run in one pass: the rasterizer interpolates
# each pixel's winner as it writes it, so rast is not read back by a second
# kernel.  The outputs equal rasterize_layers(...) followed by interpolate /
# interpolate_mse on each layer, bit for bit.  When only out reaches the loss
# (directly or through its fused loss), the VJP is one pass for both layers'
# interpolate and rasterize VJPs (dr_rasterize_xf_interp_bwd); otherwise the
# separate VJP kernels.

# False runs the separate VJPs in every case (to compare the two).
FUSED_LAYERS_VJP = True


def _ptr_pair(ts):
    """A C array of two device pointers (NULL for None)."""
    import ctypes
    return ctypes.cast((ctypes.c_void_p * 2)(*[(t.data_ptr() if t is not None else None) for t in ts]),
                       ctypes.c_void_p)


class _RasterizeInterpolateLayers(torch.autograd.Function):
    @staticmethod
    def forward(ctx, verts, attr, xform, tri, H, W, tgt0, tgt1):
        ctx.set_materialize_grads(False)
        import ctypes
        vc = _f32(verts, "verts")
        xf = _f32(xform, "xform")
        attr_c = _f32(attr, "attr")
        a3 = attr_c if attr_c.dim() == 3 else attr_c.unsqueeze(0)
        N, V, T = xf.shape[0], vc.shape[0], tri.shape[0]
        Na, Va, A = a3.shape
        dev = vc.device
        rasts = [torch.empty((N, H, W, 4), device=dev, dtype=torch.float32) for _ in range(2)]
        dbs = [torch.empty((N, H, W, 4), device=dev, dtype=torch.float32) for _ in range(2)]
        outs = [torch.empty((N, H, W, A), device=dev, dtype=torch.float32) for _ in range(2)]
        odas = [torch.empty((N, H, W, 2 * A), device=dev, dtype=torch.float32) for _ in range(2)]
        tgts = [_check_target(t, outs[l], "rasterize_interpolate_layers") if t is not None else None
                for l, t in enumerate((tgt0, tgt1))]
        losses = [torch.zeros((), device=dev, dtype=torch.float32) for _ in range(2)]
        scale = 1.0 / max(outs[0].numel(), 1)

        def arr(ts):
            return ctypes.cast((ctypes.c_void_p * 2)(*[(t.data_ptr() if t is not None else None) for t in ts]),
                               ctypes.c_void_p)
        any_t = any(t is not None for t in tgts)
        c = _ctx(vc)
        L.check(L.lib().dr_rasterize_xf_interp_fwd(
            c, _ptr(vc), V, _ptr(xf), _ptr(tri), T, N, H, W, _ptr(a3), Na, A, arr(rasts), arr(dbs), arr(outs),
            arr(odas), arr(tgts) if any_t else None, scale,
            arr([losses[l] if tgts[l] is not None else None for l in range(2)]) if any_t else None),
            c, "rasterize_interpolate_layers")
        ctx.save_for_backward(vc, xf, tri, a3, *rasts, *dbs, *outs,
                              *[t if t is not None else torch.empty(0, device=dev) for t in tgts])
        ctx.meta = (N, V, T, H, W, A, tuple(attr.shape), scale, [t is not None for t in tgts])
        # A layer's out feeds its fused loss when it has a target; it is then
        # not differentiable (as interpolate_mse's), and a loss without a
        # target is a constant zero.
        for l in range(2):
            if tgts[l] is not None:
                ctx.mark_non_differentiable(outs[l])
            else:
                ctx.mark_non_differentiable(losses[l])
        return (rasts[0], dbs[0], outs[0], odas[0], rasts[1], dbs[1], outs[1], odas[1], losses[0], losses[1])

    @staticmethod
    def backward(ctx, g_r0, g_db0, g_o0, g_oda0, g_r1, g_db1, g_o1, g_oda1, g_l0, g_l1):
        import ctypes
        vc, xf, tri, a3, r0, r1, db0, db1, o0, o1, t0, t1 = ctx.saved_tensors
        N, V, T, H, W, A, attr_shape, scale, has_t = ctx.meta
        Na = a3.shape[0]
        rasts, dbs, outs, tgts = (r0, r1), (db0, db1), (o0, o1), (t0, t1)
        g_r, g_db, g_o, g_oda, g_l = (g_r0, g_r1), (g_db0, g_db1), (g_o0, g_o1), (g_oda0, g_oda1), (g_l0, g_l1)
        c = _ctx(vc)
        if FUSED_LAYERS_VJP and all(g is None for g in g_r + g_db + g_oda):
            # Only out reaches the loss (directly or through its fused loss):
            # both VJPs of both layers in one pass.
            d_out, o_p, t_p, dl_p = [None, None], [None, None], [None, None], [None, None]
            for l in range(2):
                if has_t[l] and g_l[l] is not None:
                    o_p[l], t_p[l], dl_p[l] = outs[l], tgts[l], g_l[l].contiguous().float()
                elif not has_t[l] and g_o[l] is not None:
                    d_out[l] = g_o[l].contiguous().float()
            if all(x is None for x in d_out + o_p):
                return (None,) * 8
            d_attr = torch.empty_like(a3)
            d_verts = torch.empty_like(vc)
            L.check(L.lib().dr_rasterize_xf_interp_bwd(
                c, _ptr(vc), V, _ptr(xf), _ptr(tri), T, N, H, W, _ptr(a3), Na, A, _ptr_pair(rasts),
                _ptr_pair(d_out), _ptr_pair(o_p), _ptr_pair(t_p), scale, _ptr_pair(dl_p), _ptr(d_attr),
                _ptr(d_verts)), c, "rasterize_interpolate_layers_bwd")
            return (d_verts, d_attr.reshape(attr_shape), None, None, None, None, None, None)
        d_attr = None
        d_rast, d_db = [None, None], [None, None]
        for l in range(2):
            mse = has_t[l] and g_l[l] is not None
            plain = (not has_t[l]) and g_o[l] is not None
            K = A if g_oda[l] is not None else 0
            if not (mse or plain or K):
                continue
            da = torch.empty_like(a3)
            dr_ = torch.empty_like(rasts[l])
            ddb = torch.empty_like(rasts[l]) if K else None
            oda = g_oda[l].contiguous().float() if K else None
            if mse:
                L.check(L.lib().dr_interpolate_bwd_mse(
                    c, _ptr(a3), Na, V, A, _ptr(rasts[l]), N, H, W, _ptr(tri), T, _ptr(dbs[l]), None, K,
                    _ptr(outs[l]), _ptr(tgts[l]), scale, _ptr(g_l[l].contiguous().float()), _ptr(oda), _ptr(da),
                    _ptr(dr_), _ptr(ddb)), c, "interpolate_bwd_mse")
            else:
                d_out = (g_o[l].contiguous().float() if plain
                         else torch.zeros((N, H, W, A), device=vc.device, dtype=torch.float32))
                L.check(L.lib().dr_interpolate_bwd(
                    c, _ptr(a3), Na, V, A, _ptr(rasts[l]), N, H, W, _ptr(tri), T, _ptr(dbs[l]), None, K,
                    _ptr(d_out), _ptr(oda), _ptr(da), _ptr(dr_), _ptr(ddb)), c, "interpolate_bwd")
            d_attr = da if d_attr is None else d_attr + da
            d_rast[l], d_db[l] = dr_, ddb
        for l in range(2):
            if g_r[l] is not None:
                d_rast[l] = g_r[l].float() if d_rast[l] is None else d_rast[l] + g_r[l]
            if g_db[l] is not None:
                d_db[l] = g_db[l].float() if d_db[l] is None else d_db[l] + g_db[l]
            if d_rast[l] is None and d_db[l] is not None:
                d_rast[l] = torch.zeros_like(rasts[l])
        d_verts = None
        if any(g is not None for g in d_rast):
            d_verts = torch.empty_like(vc)
            d_rast = [g.contiguous() if g is not None else None for g in d_rast]
            d_db = [g.contiguous() if g is not None else None for g in d_db]

            def arr(ts):
                return ctypes.cast((ctypes.c_void_p * 2)(*[(t.data_ptr() if t is not None else None) for t in ts]),
                                   ctypes.c_void_p)
            L.check(L.lib().dr_rasterize_xf_bwd(c, _ptr(vc), V, _ptr(xf), _ptr(tri), T, N, H, W, 2, arr(rasts),
                                                arr(d_rast), arr(d_db), _ptr(d_verts)), c, "rasterize_xf_bwd")
        return (d_verts, d_attr.reshape(attr_shape) if d_attr is not None else None, None, None, None, None, None,
                None)


def rasterize_interpolate_layers(verts: torch.Tensor, tri: torch.Tensor, resolution, attr: torch.Tensor,
                                 xform: torch.Tensor, targets=(None, None)):
    """Two depth layers of the per-view transform mode (verts [V, 4], xform
    [N, 4, 4]) with interpolate of attr ([V, A] or [N, V, A], A a multiple of
    4; diffAttrs .all) fused into the rasterizer's pass.  targets: per layer
    None or an [N, H, W, A] target of a fused mean-squared-error loss.
    Returns [(rast, rast_db, out, out_da, loss), ...] for layers 0 and 1, the
    same values as rasterize_layers(verts, tri, resolution, 2, xform=xform)
    followed by interpolate(attr, rast, tri, rast_db, "all") (or
    interpolate_mse with the layer's target); a layer's loss is a zero
    constant when it has no target, and its out is not differentiable when it
    has one."""
    if tri.dim() != 2 or tri.shape[1] != 3:
        raise ValueError(f"rasterize: tri must be [T, 3] (got {tuple(tri.shape)})")
    if verts.dim() != 2 or verts.shape[1] != 4 or xform.dim() != 3 or tuple(xform.shape[1:]) != (4, 4):
        raise ValueError("rasterize_interpolate_layers: verts must be [V, 4] and xform [N, 4, 4]")
    if attr.dim() not in (2, 3) or attr.shape[-2] != verts.shape[0] or attr.shape[-1] % 4 != 0:
        raise ValueError("rasterize_interpolate_layers: attr must be [V, A] or [N, V, A] with verts' V and A a "
                         f"multiple of 4 (got {tuple(attr.shape)})")
    if attr.dim() == 3 and attr.shape[0] not in (1, xform.shape[0]):
        raise ValueError(f"interpolate: attr batch dim {attr.shape[0]} incompatible with rast batch {xform.shape[0]}")
    H, W = int(resolution[0]), int(resolution[1])
    t0, t1 = targets
    o = _RasterizeInterpolateLayers.apply(verts, attr, xform, _i32(tri, "tri"), H, W, t0, t1)
    return [(o[0], o[1], o[2], o[3], o[8]), (o[4], o[5], o[6], o[7], o[9])]


# Swift-style aliases of the reference's names.
textureConstructMip = texture_construct_mip
antialiasConstructTopologyHash = antialias_construct_topology_hash
