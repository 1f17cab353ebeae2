"""The operators' argument checks, restating the reference's preconditions
(Rasterize.swift:52-99, Interpolate.swift:50-107, Texture.swift:75-113, 147,
Antialias.swift:20-103): each misuse raises before any device work, with the
message naming the argument.  Runs without a GPU (the checks precede the
library call)."""
import pytest
import torch

import diffrast
from diffrast import BoundaryMode as B
from diffrast import FilterMode as F

Z = torch.zeros
TRI = Z((2, 3), dtype=torch.int32)


def _raises(msg, fn, *a, **k):
    with pytest.raises(ValueError, match=msg):
        fn(*a, **k)


def test_rasterize_preconditions():
    pos = Z((1, 4, 4))
    _raises(r"tri must be \[T, 3\]", diffrast.rasterize, pos, Z((2, 4), dtype=torch.int32), (8, 8))
    _raises(r"pos must be \[N, V, 4\]", diffrast.rasterize, Z((1, 4, 3)), TRI, (8, 8))
    _raises(r"with `ranges`, pos must be \[V, 4\]", diffrast.rasterize, pos, TRI, (8, 8),
            ranges=Z((1, 2), dtype=torch.int32))
    _raises(r"ranges must be \[N, 2\]", diffrast.rasterize, Z((4, 4)), TRI, (8, 8),
            ranges=Z((1, 3), dtype=torch.int32))
    _raises(r"peelLayer must match", diffrast.rasterize, pos, TRI, (8, 8), peel_layer=Z((1, 8, 7, 4)))
    _raises(r"num_layers must be >= 1", diffrast.rasterize_layers, pos, TRI, (8, 8), 0)


def test_interpolate_preconditions():
    rast = Z((1, 8, 8, 4))
    attr = Z((4, 3))
    _raises(r"rast must be \[N, H, W, 4\]", diffrast.interpolate, attr, Z((1, 8, 8, 3)), TRI)
    _raises(r"tri must be \[T, 3\]", diffrast.interpolate, attr, rast, Z((2,), dtype=torch.int32))
    _raises(r"attr must be \[V, A\] or \[N, V, A\]", diffrast.interpolate, Z((4,)), rast, TRI)
    _raises(r"attr batch dim 2 incompatible", diffrast.interpolate, Z((2, 4, 3)), rast, TRI)
    _raises(r"rastDB is required", diffrast.interpolate, attr, rast, TRI, None, "all")
    _raises(r"rastDB must match rast shape", diffrast.interpolate, attr, rast, TRI, Z((1, 8, 4, 4)), "all")
    _raises(r"diffAttrs.indices must be non-empty", diffrast.interpolate, attr, rast, TRI, rast,
            diffrast.DiffAttrs.indices([]))
    _raises(r"values must be in \[0, A\)", diffrast.interpolate, attr, rast, TRI, rast,
            diffrast.DiffAttrs.indices([0, 3]))


def test_texture_preconditions():
    tex, uv = Z((1, 8, 8, 3)), Z((2, 4, 4, 2))
    _raises(r"tex must be \[N, H_tex, W_tex, C\]", diffrast.texture, Z((8, 8, 3)), uv)
    _raises(r"uv must be \[N, H_img, W_img, 2\]", diffrast.texture, tex, Z((2, 4, 4, 3)))
    _raises(r"tex batch dim 3 incompatible", diffrast.texture, Z((3, 8, 8, 3)), uv)
    _raises(r"mipmap filterModes require uvDA", diffrast.texture, tex, uv, None, F.linearMipmapLinear)
    _raises(r"uvDA must be \[N, H_img, W_img, 4\]", diffrast.texture, tex, uv, Z((2, 4, 4, 2)),
            F.linearMipmapLinear)
    _raises(r"mipLevelBiasMap must be", diffrast.texture, tex, uv, Z((2, 4, 4, 4)), F.linearMipmapLinear,
            B.wrap, 0.0, Z((2, 4, 3)))
    # cube maps
    cube, d = Z((1, 6, 8, 8, 3)), Z((2, 4, 4, 3))
    _raises(r"cube textures support the linear and mipmap", diffrast.texture, cube, d, None, F.nearest, B.cube)
    _raises(r"cube tex must be \[N, 6, H, W, C\]", diffrast.texture, Z((1, 5, 8, 8, 3)), d, None, F.linear,
            B.cube)
    _raises(r"cube uv must be \[N, H_img, W_img, 3\]", diffrast.texture, cube, uv, None, F.linear, B.cube)
    _raises(r"cube uvDA must be \[N, H_img, W_img, 6\]", diffrast.texture, cube, d, Z((2, 4, 4, 4)),
            F.linearMipmapLinear, B.cube)
    _raises(r"cube_dir_grad applies to cube textures only", diffrast.texture, tex, uv, cube_dir_grad=True)
    _raises(r"textureConstructMip: tex must be \[N, H, W, C\]", diffrast.texture_construct_mip, Z((8, 8, 3)))


def test_antialias_preconditions():
    color, rast, pos = Z((1, 8, 8, 3)), Z((1, 8, 8, 4)), Z((1, 4, 4))
    _raises(r"tri must be \[T, 3\]", diffrast.antialias_construct_topology_hash, Z((2, 2), dtype=torch.int32))
    _raises(r"color must be \[N, H, W, C\]", diffrast.antialias, Z((8, 8, 3)), rast, pos, TRI)
    _raises(r"rast must match color", diffrast.antialias, color, Z((1, 8, 7, 4)), pos, TRI)
    _raises(r"pos must be \[N, V, 4\]", diffrast.antialias, color, rast, Z((1, 4, 3)), TRI)
    _raises(r"pos batch must match color batch", diffrast.antialias, color, rast, Z((2, 4, 4)), TRI)
    _raises(r"tri must be \[T, 3\]", diffrast.antialias, color, rast, pos, Z((2, 4), dtype=torch.int32))


def test_valid_shapes_on_cpu_reach_the_device_check():
    # With every shape valid, the only complaint left is the missing device.
    with pytest.raises(ValueError, match="must be a CUDA tensor"):
        diffrast.texture(Z((1, 8, 8, 3)), Z((1, 4, 4, 2)))
