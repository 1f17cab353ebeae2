"""The allocation-free topology-hash entry point, called through the C ABI.

dr_antialias_construct_topology_hash_static is for callers that cannot
allocate device memory (their host owns the GPU's memory through its own pool,
or they must avoid cudaMalloc's device-wide synchronisation).  It uses a fixed
table compiled into the library instead of a context workspace.  This test
checks that two calls in a row give exactly what the allocating entry point
gives (the topology table is integer data: bit-exact is the tolerance), and
that a mesh above the table's stated limit is rejected before any launch.

The file sorts last so that a `-x` run has already run every other test if it
fails; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_TRIS = 65536  # DR_STATIC_TOPO_MAX_TRIS


def _mesh(seed, n_iso, n_strips):
    from diffrast import scenes
    _, tri = scenes.triangle_soup(n_iso, n_strips, 10, seed=seed)
    g = np.random.default_rng(seed)
    extra = g.integers(0, 64, size=(200, 3)).astype(np.int32)  # repeated and non-manifold edges
    return np.concatenate([tri, extra], 0)


def test_static_topology_hash_matches_allocating_entry_point():
    import torch

    import diffrast
    from diffrast import _lib

    fn = _lib.lib().dr_antialias_construct_topology_hash_static
    stream = torch.cuda.current_stream().cuda_stream
    meshes = [_mesh(31, 20000, 1000), _mesh(32, 5000, 3000)]
    assert all(m.shape[0] <= MAX_TRIS for m in meshes)
    for tri_np in meshes:  # two calls in a row reuse (and must clear) the shared table
        tri = torch.from_numpy(tri_np).cuda()
        ref = diffrast.antialias_construct_topology_hash(tri)
        out = torch.full_like(tri, 7)
        st = fn(ctypes.c_void_p(tri.data_ptr()), tri.shape[0], ctypes.c_void_p(out.data_ptr()),
                ctypes.c_void_p(stream))
        assert st == _lib.DR_OK
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert (out >= 0).any() and (out == -1).any() and (out == -2).any()


def test_static_topology_hash_large_then_small_mesh():
    # A mesh near the table's limit fills slots far above a small mesh's range;
    # the small mesh that follows must not see them (each call clears and
    # probes only its own range).
    import torch

    import diffrast
    from diffrast import _lib

    fn = _lib.lib().dr_antialias_construct_topology_hash_static
    stream = torch.cuda.current_stream().cuda_stream
    big = _mesh(33, 50000, 1500)[: MAX_TRIS - 16]
    small = np.array([[0, 1, 2], [2, 1, 3], [3, 1, 4], [0, 2, 5], [6, 7, 8]], np.int32)
    for tri_np in (big, small):
        tri = torch.from_numpy(np.ascontiguousarray(tri_np)).cuda()
        ref = diffrast.antialias_construct_topology_hash(tri)
        out = torch.full_like(tri, 7)
        st = fn(ctypes.c_void_p(tri.data_ptr()), tri.shape[0], ctypes.c_void_p(out.data_ptr()),
                ctypes.c_void_p(stream))
        assert st == _lib.DR_OK
        torch.cuda.synchronize()
        assert torch.equal(out, ref), tri_np.shape


def test_static_topology_hash_rejects_meshes_above_its_limit():
    import torch

    from diffrast import _lib

    fn = _lib.lib().dr_antialias_construct_topology_hash_static
    tri = torch.zeros((MAX_TRIS + 1, 3), dtype=torch.int32, device="cuda")
    out = torch.full_like(tri, 7)
    st = fn(ctypes.c_void_p(tri.data_ptr()), tri.shape[0], ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.DR_EINVAL
    torch.cuda.synchronize()
    assert bool((out == 7).all())  # nothing was launched
