"""Full-chain forward+backward steps for the benchmark configurations.

A chain owns its scene tensors on one device and exposes `step()`, which runs
the configuration's render chain (rasterize -> interpolate -> texture ->
antialias -> MSE), the backward to every learnable tensor, and returns the loss
(a device scalar).  Views can be sharded across ranks: each rank builds only its
own views (`view_lo:view_hi`) and `shared_grads()` lists the tensors whose
gradients are summed across ranks (mesh, attributes, texture).

Per-step pixels = views * H * W (a second depth-peel layer is not counted twice).
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from . import ops, scenes


@dataclass
class ChainInfo:
    name: str
    n_views: int          # views this rank renders per step
    res: tuple
    pixels: int           # pixels per step on this rank
    kernels: Dict[str, float] = field(default_factory=dict)  # algorithmic bytes per launch


def _t(a, dev, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    if grad:
        t.requires_grad_(True)
    return t


class Chain:
    info: ChainInfo
    # Set by a multi-rank driver to its dist.GradSync: chains that run several
    # backward calls per step tell it which one is the last.
    grad_sync = None

    def backward(self, loss: torch.Tensor, last: bool = True) -> None:
        if self.grad_sync is not None:
            self.grad_sync.arm(last)
        loss.backward()

    def params(self) -> List[torch.Tensor]:
        raise NotImplementedError

    def shared_params(self) -> List[torch.Tensor]:
        """Parameters every rank holds a replica of (their gradients are summed
        across ranks)."""
        return self.params()

    def shared_grads(self) -> List[torch.Tensor]:
        return [p.grad for p in self.shared_params() if p.grad is not None]

    def zero_grad(self):
        for p in self.params():
            p.grad = None

    def step(self) -> torch.Tensor:
        raise NotImplementedError


# ------------------------------------------------------------------- cfg1

class Cfg1(Chain):
    """Tier-1 colour fit: one fixed triangle, 256^2, rasterize -> interpolate(RGB)
    -> antialias -> MSE; backward to the vertex colours and positions."""

    def __init__(self, dev, view_lo=0, view_hi=1):
        s = scenes.scene_cfg1()
        self.pos = _t(s["pos"], dev, True)
        self.tri = _t(s["tri"], dev)
        self.rgb = _t(s["attr"], dev, True)
        self.target = _t(s["target"], dev)
        self.topo = ops.antialias_construct_topology_hash(self.tri)
        H, W = s["res"]
        self.res = (H, W)
        P = H * W
        self.info = ChainInfo("cfg1", 1, (H, W), P)

    def params(self):
        return [self.pos, self.rgb]

    def step(self):
        rast, _ = ops.rasterize(self.pos, self.tri, self.res, grad_db=False)
        col, _ = ops.interpolate(self.rgb, rast, self.tri)
        loss, _ = ops.antialias_mse(col, rast, self.pos, self.tri, self.target, self.topo)
        loss.backward()
        return loss


# ------------------------------------------------------------------- cfg2

class Cfg2(Chain):
    """Icosphere L4, 8 views at 512^2: RGB and spherical-UV interpolation, bilinear
    clamp texture 512^2x3, shade = rgb * tex, antialias, MSE; d_pos, d_attr, d_tex."""

    def __init__(self, dev, view_lo=0, view_hi=8, res=512, tex=512):
        s = scenes.scene_cfg2(n_views=view_hi, res=res, tex=tex)
        self.pos = _t(s["pos"][view_lo:view_hi], dev, True)
        self.tri = _t(s["tri"], dev)
        self.rgb = _t(s["rgb"], dev, True)
        self.uv = _t(s["uv"], dev, True)
        self.tex = _t(s["tex"], dev, True)
        self.target = _t(s["target"][view_lo:view_hi], dev)
        self.topo = ops.antialias_construct_topology_hash(self.tri)
        self.res = s["res"]
        n = view_hi - view_lo
        self.info = ChainInfo("cfg2", n, self.res, n * self.res[0] * self.res[1])

    def params(self):
        return [self.pos, self.rgb, self.uv, self.tex]

    def shared_params(self):
        return [self.rgb, self.uv, self.tex]

    def step(self):
        rast, _ = ops.rasterize(self.pos, self.tri, self.res, grad_db=False)
        rgb, _ = ops.interpolate(self.rgb, rast, self.tri)
        uv, _ = ops.interpolate(self.uv, rast, self.tri)
        tc = ops.texture(self.tex, uv, filter_mode=ops.FilterMode.linear, boundary_mode=ops.BoundaryMode.clamp)
        loss, _ = ops.antialias_mse(rgb * tc, rast, self.pos, self.tri, self.target, self.topo)
        loss.backward()
        return loss


# ------------------------------------------------------------------- cfg3

class Cfg3(Chain):
    """Icosphere L4, 16 views at 1024^2 with rast_db; UV with diffAttrs=.all;
    trilinear 2048^2x4 noise texture, wrap, per-pixel mip bias ~U[-1,1]; MSE;
    backward d_tex (all levels folded), d_uv, d_uvDA -> d_rast/d_rast_db -> d_pos."""

    def __init__(self, dev, view_lo=0, view_hi=16, res=1024, tex=2048):
        s = scenes.scene_cfg3(n_views=view_hi, res=res, tex=tex)
        self.pos = _t(s["pos"][view_lo:view_hi], dev, True)
        self.tri = _t(s["tri"], dev)
        self.uv = _t(s["uv"], dev, True)
        self.tex = _t(s["tex"], dev, True)
        self.bias = _t(s["bias_map"][view_lo:view_hi], dev)
        self.target = _t(s["target"][view_lo:view_hi], dev)
        self.res = s["res"]
        n = view_hi - view_lo
        self.info = ChainInfo("cfg3", n, self.res, n * self.res[0] * self.res[1])

    def params(self):
        return [self.pos, self.uv, self.tex]

    def shared_params(self):
        return [self.uv, self.tex]

    def step(self):
        rast, db = ops.rasterize(self.pos, self.tri, self.res, grad_db=True)
        uv, uvda = ops.interpolate(self.uv, rast, self.tri, db, ops.DiffAttrs.all)
        col = ops.texture(self.tex, uv, uvda, ops.FilterMode.linearMipmapLinear, ops.BoundaryMode.wrap,
                          mip_level_bias_map=self.bias)
        loss = ops.mse_loss(col, self.target)
        loss.backward()
        return loss


# ------------------------------------------------------------------- cfg4

class Cfg4(Chain):
    """1M-triangle soup (20% in edge-sharing strips), 32 views at 1024^2: two depth
    layers with rast_db (the second peels the first), interpolate 8 channels with
    diffAttrs=.all on both, antialias (topology hash) on layer 0; loss =
    MSE(aa0) + MSE(interp1); backward to the soup vertices and attributes.

    The views are per-view 2-D similarity transforms M_n of the shared soup in
    clip space (pos_n = M_n @ base), evaluated inside the rasterize and antialias
    kernels (the library's per-view transform mode), so no [N, V, 4] tensor is
    materialised and every view's gradient lands on the shared [V, 4] buffer."""

    def __init__(self, dev, view_lo=0, view_hi=32, total_views=32, res=1024, n_isolated=800_000,
                 n_strips=20_000, use_tile_order=True, fused=True):
        self.use_tile_order = use_tile_order
        self.fused = fused
        s = scenes.scene_cfg4(n_views=total_views, res=res, n_isolated=n_isolated, n_strips=n_strips)
        self.base = _t(s["base"], dev, True)
        self.tri = _t(s["tri"], dev)
        self.attr = _t(s["attr"], dev, True)
        self.sim = _t(s["sim"][view_lo:view_hi], dev)
        self.res = s["res"]
        n = view_hi - view_lo
        H, W = self.res
        g = torch.Generator(device=dev)
        g.manual_seed(s["target_seed"] * 1000 + view_lo)
        self.tgt0 = torch.randn((n, H, W, 8), generator=g, device=dev)
        self.tgt1 = torch.randn((n, H, W, 8), generator=g, device=dev)
        self.topo = ops.antialias_construct_topology_hash(self.tri)
        self.info = ChainInfo("cfg4", n, self.res, n * H * W)

    def params(self):
        return [self.base, self.attr]

    def shared_params(self):
        return [self.base, self.attr]

    def positions(self):
        return torch.einsum("nij,vj->nvi", self.sim, self.base)

    def step(self):
        if self.fused:
            # Both layers rasterized with interpolate in the same pass (layer
            # 1's MSE included); the VJPs are the separate ones.
            (rast0, _, out0, _, _), (_, _, _, _, loss1) = ops.rasterize_interpolate_layers(
                self.base, self.tri, self.res, self.attr, self.sim, targets=(None, self.tgt1))
        else:
            (rast0, db0), (rast1, db1) = ops.rasterize_layers(self.base, self.tri, self.res, 2, grad_db=True,
                                                              xform=self.sim)
        # Interpolate (its VJPs, and the separate forward) walks the views'
        # tiles grouped by soup region, so the attribute table and its
        # gradient stay in L2 while every view passes over a region.
        order = ops.tile_order(rast0, self.base, self.tri) if self.use_tile_order else None
        with (ops.tile_order_scope(order, rast0.shape[:3]) if order is not None else contextlib.nullcontext()):
            if not self.fused:
                out0, _ = ops.interpolate(self.attr, rast0, self.tri, db0, ops.DiffAttrs.all)
                # Layer 1's interpolation and layer 0's antialias each compute
                # their MSE term in their own kernels (the *_mse ops).
                loss1, _, _ = ops.interpolate_mse(self.attr, rast1, self.tri, self.tgt1, db1, ops.DiffAttrs.all)
            loss0, _ = ops.antialias_mse(out0, rast0, self.base, self.tri, self.tgt0, self.topo, xform=self.sim)
            loss = loss0 + loss1
            loss.backward()
        return loss


# ------------------------------------------------------------------- cfg5

class Cfg5(Chain):
    """Geodesic sphere (f=158: 499,280 triangles), views at 2048^2: interpolate
    per-vertex normals as cube directions, cube texture 6x1024^2x3 sampled
    trilinearly (the normals' screen-space derivatives give the LOD; the
    reference's own cube mode, .linear, with filter_mode=FilterMode.linear),
    antialias, MSE; backward d_verts and d_tex.  The rank's views run as
    micro-batches with gradient accumulation."""

    def __init__(self, dev, view_lo=0, view_hi=256, micro=16, res=2048, freq=158, cube=1024,
                 filter_mode=ops.FilterMode.linearMipmapLinear):
        s = scenes.scene_cfg5(n_views=view_hi, res=res, freq=freq, cube=cube)
        self.verts = _t(np.concatenate([s["verts"], np.ones((s["verts"].shape[0], 1), np.float32)], 1),
                        dev, True)
        self.tri = _t(s["tri"], dev)
        self.nrm = _t(s["unit"], dev)
        self.cube = _t(s["cube"], dev, True)
        self.mvp = _t(s["mvps"][view_lo:view_hi], dev)
        self.res = s["res"]
        n = view_hi - view_lo
        H, W = self.res
        g = torch.Generator(device=dev)
        g.manual_seed(s["target_seed"] * 1000 + view_lo)
        self.target = torch.rand((n, H, W, 3), generator=g, device=dev)
        self.topo = ops.antialias_construct_topology_hash(self.tri)
        self.bg_dir = torch.tensor([0.0, 0.0, 1.0], device=dev)
        self.micro = micro
        self.filter_mode = ops.FilterMode(filter_mode)
        self.info = ChainInfo("cfg5", n, self.res, n * H * W)

    def params(self):
        return [self.verts, self.cube]

    def shared_params(self):
        return [self.verts, self.cube]

    def step(self):
        n = self.mvp.shape[0]
        tot = None
        for a in range(0, n, self.micro):
            b = min(n, a + self.micro)
            xf = self.mvp[a:b]
            mip = self.filter_mode != ops.FilterMode.linear
            ((rast, db),) = ops.rasterize_layers(self.verts, self.tri, self.res, 1, grad_db=mip, xform=xf)
            nrm, nrm_da = ops.interpolate(self.nrm, rast, self.tri, db if mip else None,
                                          ops.DiffAttrs.all if mip else None)
            # Background pixels interpolate a zero normal, which has no cube face
            # (the projection divides by max|dir| = 0): look them up along +z.
            nrm = nrm + (rast[..., 3:] == 0).float() * self.bg_dir
            col = ops.texture(self.cube, nrm, nrm_da if mip else None, self.filter_mode, ops.BoundaryMode.cube)
            mse, _ = ops.antialias_mse(col, rast, self.verts, self.tri, self.target[a:b], self.topo, xform=xf)
            loss = mse * ((b - a) / n)
            self.backward(loss, last=b == n)
            tot = loss.detach() if tot is None else tot + loss.detach()
        return tot


CHAINS = {"cfg1": Cfg1, "cfg2": Cfg2, "cfg3": Cfg3, "cfg4": Cfg4, "cfg5": Cfg5}
TOTAL_VIEWS = {"cfg1": 1, "cfg2": 8, "cfg3": 16, "cfg4": 32, "cfg5": 256}
