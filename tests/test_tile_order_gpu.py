"""Tile order (dr_tile_order / dr_ctx_set_tile_order): interpolate's forward
and VJP walking a batch tile by tile in a world-grouped order return what
they return in image order.
  out, out_da, d_rast, d_rast_db (per-pixel, no atomics): bit-identical
  d_attr (atomics in another order): <= 1e-5 relative L2
  fused loss: <= 1e-6 relative
Sizes include partial edge tiles (100 x 72 pixels) and a batch whose shape differs
from the one the order was set for (image order again)."""
import numpy as np
import pytest

from diffrast import scenes
from helpers import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def scene():
    import torch
    import diffrast
    base, tri = scenes.triangle_soup(6000, 300, 10, seed=51)
    M = scenes.similarity_matrices(3, seed=52).astype(np.float32)
    base, tri, M = torch.from_numpy(base).cuda(), torch.from_numpy(tri).cuda(), torch.from_numpy(M).cuda()
    layers = diffrast.rasterize_layers(base, tri, (100, 72), 2, grad_db=True, xform=M)
    return base, tri, M, layers


def _tile_shape():
    """(width, height) of the library's order tiles, from dr_tile_count."""
    from diffrast import _lib
    count = _lib.lib().dr_tile_count
    tw = next(w for w in range(1, 1025) if count(1, 1, w + 1) == 2)
    th = next(h for h in range(1, 1025) if count(1, h + 1, 1) == 2)
    assert tw * th == 256
    return tw, th


def test_order_is_a_permutation_with_empty_tiles_last(scene):
    import torch
    import diffrast
    base, tri, M, ((rast, _), _) = scene
    order = diffrast.tile_order(rast, base, tri)
    tw, th = _tile_shape()
    ntx, nty = -(-72 // tw), -(-100 // th)
    n = 3 * ntx * nty
    assert order.dtype == torch.int32 and order.numel() == n
    o = order.cpu().numpy()
    assert np.array_equal(np.sort(o), np.arange(n))
    # Tiles whose sample pixels show nothing come last.
    r = rast.cpu().numpy()
    def shows(t):
        v, k = divmod(int(t), ntx * nty)
        ty, tx = divmod(k, ntx)
        pts = [(th // 2, tw // 2), (th // 4, tw // 4), (th // 4, 3 * tw // 4), (3 * th // 4, tw // 4),
               (3 * th // 4, 3 * tw // 4)]
        return any(r[v, min(ty * th + y, 99), min(tx * tw + x, 71), 3] > 0 for y, x in pts)
    flags = [shows(t) for t in o]
    first_empty = flags.index(False) if False in flags else len(flags)
    assert all(not f for f in flags[first_empty:])
    assert all(flags[:first_empty])
    # The order is deterministic.
    assert torch.equal(diffrast.tile_order(rast, base, tri), order)


@pytest.mark.parametrize("shared,diff,fused", [(True, "all", False), (False, None, False), (True, [1, 3], True),
                                               (False, "all", True)])
def test_interpolate_same_in_tile_order(scene, shared, diff, fused):
    import torch
    import diffrast
    base, tri, M, ((rast0, db0), (rast1, db1)) = scene
    N, H, W = rast1.shape[:3]
    V, A = base.shape[0], 4
    g = torch.Generator(device="cuda")
    g.manual_seed(61)
    attr = torch.randn(((V, A) if shared else (N, V, A)), generator=g, device="cuda")
    w = torch.randn((N, H, W, A), generator=g, device="cuda")
    target = torch.randn((N, H, W, A), generator=g, device="cuda")
    K = 0 if diff is None else (A if diff == "all" else len(diff))
    w_da = torch.randn((N, H, W, 2 * K), generator=g, device="cuda") if K else None
    order = diffrast.tile_order(rast0, base, tri)
    res = []
    for use in (False, True):
        a = attr.clone().requires_grad_(True)
        r = rast1.clone().requires_grad_(True)
        d = db1.clone().requires_grad_(True) if diff is not None else None
        if use:
            diffrast.set_tile_order(order, (N, H, W))
        try:
            if fused:
                loss, out, out_da = diffrast.interpolate_mse(a, r, tri, target, d, diff)
                total = loss * 0.5
            else:
                out, out_da = diffrast.interpolate(a, r, tri, d, diff)
                loss = (out * w).sum()
                total = loss
            if K:
                total = total + (out_da * w_da).sum()
            total.backward()
        finally:
            diffrast.set_tile_order(None)
        res.append((float(loss), out.detach().cpu().numpy(), out_da.detach().cpu().numpy(), a.grad.cpu().numpy(),
                    r.grad.cpu().numpy(), d.grad.cpu().numpy() if d is not None else None))
    (l0, o0, da0, ga0, gr0, gd0), (l1, o1, da1, ga1, gr1, gd1) = res
    assert np.array_equal(o0, o1) and np.array_equal(da0, da1)
    if fused:
        assert abs(l1 - l0) <= 1e-6 * abs(l0)
    assert rel_l2(ga1, ga0) < 1e-5 and np.abs(ga0).sum() > 0
    assert np.array_equal(gr0, gr1)
    if gd0 is not None:
        assert np.array_equal(gd0, gd1)


def test_order_applies_only_to_its_shape(scene):
    import torch
    import diffrast
    base, tri, M, ((rast0, _), (rast1, _)) = scene
    attr = torch.randn((base.shape[0], 3), device="cuda")
    ref, _ = diffrast.interpolate(attr, rast1[:2], tri)
    order = diffrast.tile_order(rast0, base, tri)
    with diffrast.tile_order_scope(order, rast0.shape[:3]):
        other, _ = diffrast.interpolate(attr, rast1[:2], tri)   # [2, 100, 72]: image order
        full, _ = diffrast.interpolate(attr, rast1, tri)        # [3, 100, 72]: tile order
    assert torch.equal(ref, other)
    assert torch.equal(full[:2], ref)


def test_set_tile_order_rejects_a_wrong_length(scene):
    import torch
    import diffrast
    base, tri, M, ((rast0, _), _) = scene
    order = diffrast.tile_order(rast0, base, tri)
    with pytest.raises(ValueError, match="tiles"):
        diffrast.set_tile_order(order[:-1], rast0.shape[:3])
    with pytest.raises(ValueError, match="int32"):
        diffrast.set_tile_order(order.long(), rast0.shape[:3])
