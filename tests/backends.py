"""Two implementations behind one numpy-in / numpy-out interface, so every
reference test runs unchanged on the CPU oracle and on the CUDA library.

  OracleBackend -> oracle/ (C++ restatement of the reference kernels; CPU)
  CudaBackend   -> diffrast (libdiffrast.so through its C ABI; GPU)

Backward helpers take explicit cotangents.  The CUDA backend obtains them with
torch autograd through the library's explicit VJP entry points.
"""
from __future__ import annotations

import numpy as np

import oracle as O


class OracleBackend:
    name = "oracle"

    def rasterize(self, pos, tri, res, grad_db=True, ranges=None, peel=None):
        return O.rasterize(pos, tri, res, grad_db=grad_db, ranges=ranges, peel_layer=peel)

    def rasterize_bwd(self, pos, tri, res, d_rast, d_db=None, ranges=None, peel=None):
        rast, _ = O.rasterize(pos, tri, res, grad_db=d_db is not None, ranges=ranges, peel_layer=peel)
        return O.rasterize_bwd(pos, tri, rast, d_rast, d_db, ranges=ranges)

    def interpolate(self, attr, rast, tri, rast_db=None, diff_attrs=None):
        return O.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs=diff_attrs)

    def interpolate_bwd(self, attr, rast, tri, d_out, rast_db=None, diff_attrs=None, d_out_da=None):
        return O.interpolate_bwd(attr, rast, tri, d_out, rast_db=rast_db, diff_attrs=diff_attrs,
                                 d_out_da=d_out_da)

    def texture(self, tex, uv, uv_da=None, filter_mode="linear", boundary_mode="wrap", bias=0.0,
                bias_map=None):
        return O.texture(tex, uv, uv_da, filter_mode, boundary_mode, bias, bias_map)

    def texture_bwd(self, tex, uv, d_out, uv_da=None, filter_mode="linear", boundary_mode="wrap",
                    bias=0.0, bias_map=None, cube_dir_grad=False):
        return O.texture_bwd(tex, uv, d_out, uv_da, filter_mode, boundary_mode, bias, bias_map,
                             cube_dir_grad=cube_dir_grad)

    def construct_mip(self, tex, max_level=None):
        return O.texture_construct_mip(tex, max_level)

    def topology_hash(self, tri):
        return O.topology_hash(tri)

    def antialias(self, color, rast, pos, tri, topo=None):
        return O.antialias(color, rast, pos, tri, topo)

    def antialias_bwd(self, color, rast, pos, tri, d_out, topo=None):
        return O.antialias_bwd(color, rast, pos, tri, d_out, topo)


_FILT = {"nearest": 0, "linear": 1, "linear-mipmap-nearest": 2, "linear-mipmap-linear": 3}
_BND = {"wrap": 0, "clamp": 1, "zero": 2, "cube": 3}


class CudaBackend:
    name = "cuda"

    def __init__(self):
        import torch

        import diffrast
        self.torch = torch
        self.dr = diffrast

    def _t(self, a, grad=False):
        if a is None:
            return None
        t = self.torch.from_numpy(np.ascontiguousarray(a)).cuda()
        if grad:
            t.requires_grad_(True)
        return t

    @staticmethod
    def _n(t):
        return None if t is None else t.detach().cpu().numpy()

    def rasterize(self, pos, tri, res, grad_db=True, ranges=None, peel=None):
        r, db = self.dr.rasterize(self._t(pos), self._t(tri), res, grad_db=grad_db, ranges=self._t(ranges),
                                  peel_layer=self._t(peel))
        return self._n(r), self._n(db)

    def rasterize_bwd(self, pos, tri, res, d_rast, d_db=None, ranges=None, peel=None):
        p = self._t(pos, grad=True)
        r, db = self.dr.rasterize(p, self._t(tri), res, grad_db=d_db is not None, ranges=self._t(ranges),
                                  peel_layer=self._t(peel))
        loss = (r * self._t(d_rast)).sum()
        if d_db is not None:
            loss = loss + (db * self._t(d_db)).sum()
        loss.backward()
        return self._n(p.grad)

    def interpolate(self, attr, rast, tri, rast_db=None, diff_attrs=None):
        o, oda = self.dr.interpolate(self._t(attr), self._t(rast), self._t(tri), self._t(rast_db),
                                     diff_attrs)
        return self._n(o), self._n(oda)

    def interpolate_bwd(self, attr, rast, tri, d_out, rast_db=None, diff_attrs=None, d_out_da=None):
        a = self._t(attr, grad=True)
        r = self._t(rast, grad=True)
        db = self._t(rast_db, grad=diff_attrs is not None) if rast_db is not None else None
        o, oda = self.dr.interpolate(a, r, self._t(tri), db, diff_attrs)
        loss = (o * self._t(d_out)).sum()
        if diff_attrs is not None and d_out_da is not None:
            loss = loss + (oda * self._t(d_out_da)).sum()
        loss.backward()
        return (self._n(a.grad), self._n(r.grad),
                self._n(db.grad) if (db is not None and diff_attrs is not None) else None)

    def texture(self, tex, uv, uv_da=None, filter_mode="linear", boundary_mode="wrap", bias=0.0,
                bias_map=None):
        out = self.dr.texture(self._t(tex), self._t(uv), self._t(uv_da), _FILT[filter_mode],
                              _BND[boundary_mode], bias, self._t(bias_map))
        return self._n(out)

    def texture_bwd(self, tex, uv, d_out, uv_da=None, filter_mode="linear", boundary_mode="wrap",
                    bias=0.0, bias_map=None, cube_dir_grad=False):
        t = self._t(tex, grad=True)
        u = self._t(uv, grad=True)
        mip = filter_mode.startswith("linear-mipmap")
        da = self._t(uv_da, grad=mip) if uv_da is not None else None
        bm = self._t(bias_map, grad=mip) if bias_map is not None else None
        out = self.dr.texture(t, u, da, _FILT[filter_mode], _BND[boundary_mode], bias, bm,
                              cube_dir_grad=cube_dir_grad)
        (out * self._t(d_out)).sum().backward()
        d_da = self._n(da.grad) if (mip and da is not None) else None
        d_bm = (self._n(bm.grad) if bm is not None else
                (np.zeros(uv.shape[:3], np.float32) if mip else None))
        return self._n(t.grad), self._n(u.grad), d_da, d_bm

    def construct_mip(self, tex, max_level=None):
        return [self._n(x) for x in self.dr.texture_construct_mip(self._t(tex), max_level)]

    def topology_hash(self, tri):
        return self._n(self.dr.antialias_construct_topology_hash(self._t(tri)))

    def antialias(self, color, rast, pos, tri, topo=None):
        return self._n(self.dr.antialias(self._t(color), self._t(rast), self._t(pos), self._t(tri),
                                         self._t(topo)))

    def antialias_bwd(self, color, rast, pos, tri, d_out, topo=None):
        c = self._t(color, grad=True)
        p = self._t(pos, grad=True)
        out = self.dr.antialias(c, self._t(rast), p, self._t(tri), self._t(topo))
        (out * self._t(d_out)).sum().backward()
        return self._n(c.grad), self._n(p.grad)


def make(name):
    return OracleBackend() if name == "oracle" else CudaBackend()
