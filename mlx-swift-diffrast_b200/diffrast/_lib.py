"""ctypes binding of libdiffrast.so (include/diffrast.h).

Loads the in-tree shared library and exposes each C entry point with its
argument types.  There is no fallback: if the library is missing or cannot be
loaded, importing the ops raises, so a GPU run can never silently compute on
something else.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdiffrast.so")

DR_OK, DR_EINVAL, DR_ENOMEM, DR_ECUDA, DR_EOVERFLOW, DR_EDEVICE = range(6)
_STATUS = {0: "DR_OK", 1: "DR_EINVAL", 2: "DR_ENOMEM", 3: "DR_ECUDA", 4: "DR_EOVERFLOW",
           5: "DR_EDEVICE"}

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
F = ctypes.c_float

# name -> (restype, argtypes), mirroring include/diffrast.h
SIGNATURES = {
    "dr_abi_version": (I, []),
    "dr_ctx_create": (I, [I, ctypes.POINTER(P)]),
    "dr_ctx_destroy": (None, [P]),
    "dr_ctx_set_stream": (I, [P, P]),
    "dr_ctx_get_stream": (P, [P]),
    "dr_last_error": (ctypes.c_char_p, [P]),
    "dr_ctx_sync": (I, [P]),
    "dr_ctx_launch_count": (ctypes.c_uint64, [P]),
    "dr_ctx_workspace_bytes": (ctypes.c_size_t, [P]),
    "dr_ctx_set_timing": (I, [P, I]),
    "dr_ctx_timing_report": (I, [P, ctypes.c_char_p, ctypes.c_size_t]),
    "dr_ctx_set_raster_list_capacity": (I, [P, I64]),
    "dr_ctx_raster_overflow": (I, [P, ctypes.POINTER(I64)]),
    "dr_tile_count": (I64, [I, I, I]),
    "dr_tile_order": (I, [P, P, I, I, I, P, I, P, I, P]),
    "dr_ctx_set_tile_order": (I, [P, P, I, I, I]),
    "dr_rasterize_fwd": (I, [P, P, I, P, I, P, I, I, I, P, P, P]),
    "dr_rasterize_bwd": (I, [P, P, I, P, I, P, I, I, I, P, P, P, P]),
    "dr_rasterize_layers_fwd": (I, [P, P, I, P, I, P, I, I, I, I, P, P]),
    "dr_rasterize_layers_bwd": (I, [P, P, I, P, I, P, I, I, I, I, P, P, P, P]),
    "dr_rasterize_xf_fwd": (I, [P, P, I, P, P, I, I, I, I, I, P, P]),
    "dr_rasterize_xf_bwd": (I, [P, P, I, P, P, I, I, I, I, I, P, P, P, P]),
    "dr_rasterize_xf_interp_fwd": (I, [P, P, I, P, P, I, I, I, I, P, I, I, P, P, P, P, P, F, P]),
    "dr_rasterize_xf_interp_bwd": (I, [P, P, I, P, P, I, I, I, I, P, I, I, P, P, P, P, F, P, P, P]),
    "dr_interpolate_fwd": (I, [P, P, I, I, I, P, I, I, I, P, I, P, P, I, P, P]),
    "dr_interpolate_bwd": (I, [P, P, I, I, I, P, I, I, I, P, I, P, P, I, P, P, P, P, P]),
    "dr_texture_mip_layout": (I, [I, I, I, I, I, ctypes.POINTER(I), ctypes.POINTER(I64),
                                  ctypes.POINTER(I), ctypes.POINTER(I), ctypes.POINTER(I64)]),
    "dr_texture_construct_mip": (I, [P, P, I, I, I, I, I, P]),
    "dr_texture_fwd": (I, [P, I, I, P, I, I, I, I, P, I, P, P, F, P, I, I, I, P]),
    "dr_texture_bwd": (I, [P, I, I, P, I, I, I, I, P, I, P, P, F, P, I, I, I, P, P, P, P, P]),
    "dr_antialias_construct_topology_hash": (I, [P, P, I, P]),
    "dr_antialias_construct_topology_hash_static": (I, [P, I, P, P]),
    "dr_antialias_fwd": (I, [P, P, I, I, I, I, P, P, I, P, I, P, P, P]),
    "dr_antialias_bwd": (I, [P, P, I, I, I, I, P, P, I, P, I, P, P, P, P, P]),
    "dr_antialias_work_bytes": (ctypes.c_size_t, [I, I, I]),
    "dr_antialias_xf_fwd": (I, [P, P, I, I, I, I, P, P, I, P, P, I, P, P, P]),
    "dr_antialias_xf_bwd": (I, [P, P, I, I, I, I, P, P, I, P, P, I, P, P, P, P, P]),
    "dr_antialias_fwd_mse": (I, [P, P, I, I, I, I, P, P, I, P, I, P, P, P, P, F, P]),
    "dr_antialias_bwd_mse": (I, [P, P, I, I, I, I, P, P, I, P, I, P, P, P, F, P, P, P, P]),
    "dr_antialias_xf_fwd_mse": (I, [P, P, I, I, I, I, P, P, I, P, P, I, P, P, P, P, F, P]),
    "dr_antialias_xf_bwd_mse": (I, [P, P, I, I, I, I, P, P, I, P, P, I, P, P, P, F, P, P, P, P]),
    "dr_interpolate_fwd_mse": (I, [P, P, I, I, I, P, I, I, I, P, I, P, P, I, P, P, P, F, P]),
    "dr_interpolate_bwd_mse": (I, [P, P, I, I, I, P, I, I, I, P, I, P, P, I, P, P, F, P, P, P, P, P]),
    "dr_mse_fwd_bwd": (I, [P, P, P, I64, F, P, P, I]),
    "dr_mse_bwd": (I, [P, P, P, I64, F, P, P]),
    "dr_adam_step": (I, [P, P, P, P, P, P, I64, F, F, F, F, F, F]),
}

_lib = None
_lock = threading.RLock()
_ctx = {}


class DiffRastError(RuntimeError):
    """A dr_* call returned a non-OK status (message from dr_last_error)."""


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"libdiffrast.so not found at {LIB_PATH}; build it with "
                        "`python mlx-swift-diffrast_b200/build.py`")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def ctx_for(device_index: int):
    """Per-device context (created on first use, kept for the process)."""
    c = _ctx.get(device_index)
    if c is None:
        lib()
        with _lock:
            c = _ctx.get(device_index)
            if c is None:
                h = P()
                st = lib().dr_ctx_create(device_index, ctypes.byref(h))
                if st != DR_OK:
                    raise DiffRastError(f"dr_ctx_create({device_index}) -> {_STATUS.get(st, st)}")
                c = h
                _ctx[device_index] = c
    return c


def check(st: int, ctx, what: str):
    if st != DR_OK:
        msg = lib().dr_last_error(ctx)
        msg = msg.decode() if msg else ""
        err = DiffRastError(f"{what}: {_STATUS.get(st, st)}: {msg}")
        err.status = st
        raise err


def launch_count(device_index: int = 0) -> int:
    return int(lib().dr_ctx_launch_count(ctx_for(device_index)))


def workspace_bytes(device_index: int = 0) -> int:
    return int(lib().dr_ctx_workspace_bytes(ctx_for(device_index)))


def set_timing(enable: bool, device_index: int = 0):
    c = ctx_for(device_index)
    check(lib().dr_ctx_set_timing(c, 1 if enable else 0), c, "dr_ctx_set_timing")


def timing_report(device_index: int = 0) -> dict:
    """{kernel name: (launches, total ms)} since timing was enabled."""
    c = ctx_for(device_index)
    buf = ctypes.create_string_buffer(1 << 16)
    check(lib().dr_ctx_timing_report(c, buf, len(buf)), c, "dr_ctx_timing_report")
    out = {}
    for line in buf.value.decode().splitlines():
        name, cnt, ms = line.split()
        out[name] = (int(cnt), float(ms))
    return out


def sync(device_index: int = 0):
    c = ctx_for(device_index)
    check(lib().dr_ctx_sync(c), c, "dr_ctx_sync")


def set_raster_list_capacity(pairs: int, device_index: int = 0):
    """Fixed (tile, triangle) list capacity for rasterize (0 = exact sizing).

    With a capacity, rasterize reads nothing back to the host, so a whole
    training step can be captured in a CUDA graph; tiles whose list would not
    fit test every triangle of their view instead (same result, slower) and
    are counted by raster_overflow().  Call it before capturing."""
    c = ctx_for(device_index)
    check(lib().dr_ctx_set_raster_list_capacity(c, int(pairs)), c, "dr_ctx_set_raster_list_capacity")


def raster_overflow(device_index: int = 0) -> int:
    """Tiles that scanned every triangle since the last call (synchronizes)."""
    c = ctx_for(device_index)
    n = I64(0)
    check(lib().dr_ctx_raster_overflow(c, ctypes.byref(n)), c, "dr_ctx_raster_overflow")
    return int(n.value)
