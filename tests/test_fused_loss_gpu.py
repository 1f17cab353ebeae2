"""The ops fused with their mean-squared-error loss (interpolate_mse,
antialias_mse) against the same op followed by the stand-alone MSE, on the
same inputs:
  out: bit-identical (the same forward kernels write it)
  loss: <= 1e-5 relative (the summation order differs)
  d_color of antialias (gather form, no atomics) and d_rast / d_rast_db of
  interpolate: bit-identical (the fused cotangent repeats the stand-alone
  MSE VJP's arithmetic)
  atomically accumulated gradients (d_pos, d_attr): <= 1e-4 relative L2
The loss's cotangent is scaled (0.7) so the device-side d_loss is exercised.
A target that starts 4 bytes past a 16-byte boundary takes the kernels'
scalar paths (their float4 loads need 16-byte alignment).
"""
import numpy as np
import pytest

from diffrast import scenes
from helpers import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def soup():
    import torch
    base, tri = scenes.triangle_soup(20000, 1000, 10, seed=41)
    M = scenes.similarity_matrices(3, seed=42).astype(np.float32)
    return torch.from_numpy(base).cuda(), torch.from_numpy(tri).cuda(), torch.from_numpy(M).cuda()


def _leaf(t):
    return t.detach().clone().requires_grad_(True)


def _offset(t):
    """A contiguous copy of t whose data starts one float past t's alignment."""
    import torch
    buf = torch.empty(t.numel() + 1, device=t.device, dtype=t.dtype)
    v = buf[1:].view(t.shape)
    v.copy_(t)
    return v


@pytest.mark.parametrize("xf,C,odd_target", [(False, 8, False), (True, 8, False), (False, 3, False),
                                              (True, 3, False), (False, 8, True), (True, 4, True)])
def test_antialias_mse_matches_op_then_mse(soup, xf, C, odd_target):
    import torch

    import diffrast
    base, tri, M = soup
    res = (192, 160)
    pos_all = torch.einsum("nij,vj->nvi", M, base).contiguous()
    ((rast, _),) = diffrast.rasterize_layers(base, tri, res, 1, grad_db=False, xform=M)
    g = torch.Generator(device="cuda")
    g.manual_seed(7 + C)
    color = torch.rand((3,) + res + (C,), generator=g, device="cuda")
    target = torch.rand((3,) + res + (C,), generator=g, device="cuda")
    if odd_target:
        target = _offset(target)
        assert target.data_ptr() % 16 == 4
    topo = diffrast.antialias_construct_topology_hash(tri)
    grads = []
    for fused in (False, True):
        c = _leaf(color)
        p = _leaf(base if xf else pos_all)
        kw = dict(xform=M) if xf else {}
        if fused:
            loss, out = diffrast.antialias_mse(c, rast, p, tri, target, topo, **kw)
        else:
            out = diffrast.antialias(c, rast, p, tri, topo, **kw)
            loss = diffrast.mse_loss(out, target)
        (loss * 0.7).backward()
        grads.append((float(loss), out.detach().cpu().numpy(), c.grad.cpu().numpy(), p.grad.cpu().numpy()))
    (l0, o0, dc0, dp0), (l1, o1, dc1, dp1) = grads
    assert np.array_equal(o0, o1)
    assert abs(l1 - l0) <= 1e-5 * abs(l0)
    assert np.array_equal(dc0, dc1)
    assert rel_l2(dp1, dp0) < 1e-4 and np.abs(dp0).sum() > 0


@pytest.mark.parametrize("diff,da_loss,odd_target", [(None, False, False), ("all", False, False), ("all", True, False),
                                                     ([2, 0], True, False), ("all", True, True)])
@pytest.mark.parametrize("shared", [True, False])
def test_interpolate_mse_matches_op_then_mse(soup, diff, da_loss, odd_target, shared):
    import torch

    import diffrast
    base, tri, M = soup
    res = (160, 192)
    ((rast, db),) = diffrast.rasterize_layers(base, tri, res, 1, grad_db=True, xform=M)
    V, A = base.shape[0], 4
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    attr = torch.randn(((V, A) if shared else (3, V, A)), generator=g, device="cuda")
    target = torch.randn((3,) + res + (A,), generator=g, device="cuda")
    if odd_target:
        target = _offset(target)
    K = 0 if diff is None else (A if diff == "all" else len(diff))
    w_da = torch.randn((3,) + res + (2 * K,), generator=g, device="cuda") if K else None
    grads = []
    for fused in (False, True):
        a = _leaf(attr)
        r = _leaf(rast)
        d = _leaf(db) if diff is not None else None
        if fused:
            loss, out, out_da = diffrast.interpolate_mse(a, r, tri, target, d, diff)
        else:
            out, out_da = diffrast.interpolate(a, r, tri, d, diff)
            loss = diffrast.mse_loss(out, target)
        total = loss * 0.7
        if da_loss:
            total = total + (out_da * w_da).sum()
        total.backward()
        grads.append((float(loss), out.detach().cpu().numpy(), out_da.detach().cpu().numpy(), a.grad.cpu().numpy(),
                      r.grad.cpu().numpy(), d.grad.cpu().numpy() if (d is not None and d.grad is not None) else None))
    (l0, o0, da0, ga0, gr0, gd0), (l1, o1, da1, ga1, gr1, gd1) = grads
    assert np.array_equal(o0, o1) and np.array_equal(da0, da1)
    assert abs(l1 - l0) <= 1e-5 * abs(l0)
    assert rel_l2(ga1, ga0) < 1e-4
    assert np.array_equal(gr0, gr1)
    if gd0 is not None:
        assert np.array_equal(gd0, gd1)


def test_fused_ops_reject_a_target_of_another_shape(soup):
    import torch

    import diffrast
    base, tri, M = soup
    ((rast, _),) = diffrast.rasterize_layers(base, tri, (32, 32), 1, grad_db=False, xform=M)
    attr = torch.randn((base.shape[0], 3), device="cuda")
    with pytest.raises(ValueError, match="target"):
        diffrast.interpolate_mse(attr, rast, tri, torch.zeros((3, 32, 32, 4), device="cuda"))
    color = torch.rand((3, 32, 32, 3), device="cuda")
    with pytest.raises(ValueError, match="target"):
        diffrast.antialias_mse(color, rast, base, tri, torch.zeros((3, 32, 32, 2), device="cuda"), xform=M)
