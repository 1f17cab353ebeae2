"""diffrast — B200-native differentiable rasterization (rasterize -> interpolate ->
texture -> antialias, each with an explicit VJP), the drop-in for
mlx-swift-diffrast's `DiffRast.*` operators.

All compute runs in libdiffrast.so (hand-written sm_100a CUDA behind the C ABI
of include/diffrast.h); this package binds it for torch tensors.
"""
from ._lib import (  # noqa: F401
    DiffRastError,
    launch_count,
    raster_overflow,
    set_raster_list_capacity,
    sync,
    workspace_bytes,
)
from .ops import (  # noqa: F401
    BoundaryMode,
    DiffAttrs,
    FilterMode,
    antialias,
    antialias_construct_topology_hash,
    antialias_mse,
    antialiasConstructTopologyHash,
    interpolate,
    interpolate_mse,
    mse_loss,
    rasterize,
    rasterize_interpolate_layers,
    rasterize_layers,
    set_tile_order,
    texture,
    texture_construct_mip,
    textureConstructMip,
    tile_order,
    tile_order_scope,
)

__all__ = [
    "BoundaryMode", "DiffAttrs", "FilterMode", "DiffRastError",
    "rasterize", "rasterize_layers", "rasterize_interpolate_layers", "interpolate", "texture", "texture_construct_mip", "textureConstructMip",
    "antialias_construct_topology_hash", "antialiasConstructTopologyHash", "antialias",
    "mse_loss", "antialias_mse", "interpolate_mse", "launch_count", "sync", "workspace_bytes", "set_raster_list_capacity", "raster_overflow",
    "tile_order", "set_tile_order", "tile_order_scope",
]
