"""rasterize_interpolate_layers (interpolate fused into the two-layer
rasterizer pass) against rasterize_layers followed by interpolate /
interpolate_mse on each layer, on the same inputs:
  rast, rast_db, out, out_da: bit-identical (the same arithmetic, shared code)
  fused loss: <= 1e-5 relative (its blocks sum other pixels)
  d_attr, d_verts: <= 1e-5 / 1e-4 relative L2 (atomics in another order)
Sizes include partial edge tiles (100 x 72), shared and per-view attributes,
and both layers with a target."""
import numpy as np
import pytest

from diffrast import scenes
from helpers import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def soup():
    import torch
    base, tri = scenes.triangle_soup(8000, 400, 10, seed=71)
    M = scenes.similarity_matrices(3, seed=72).astype(np.float32)
    return torch.from_numpy(base).cuda(), torch.from_numpy(tri).cuda(), torch.from_numpy(M).cuda()


@pytest.mark.parametrize("shared,targets", [(True, (False, True)), (False, (False, True)), (True, (True, True)),
                                            (True, (False, False))])
def test_fused_matches_separate_ops(soup, shared, targets):
    import torch

    import diffrast
    base, tri, M = soup
    res = (100, 72)
    N, V, A = M.shape[0], base.shape[0], 8
    g = torch.Generator(device="cuda")
    g.manual_seed(81)
    attr = torch.randn(((V, A) if shared else (N, V, A)), generator=g, device="cuda")
    tg = [torch.randn((N,) + res + (A,), generator=g, device="cuda") if t else None for t in targets]
    w = [torch.randn((N,) + res + (A,), generator=g, device="cuda") for _ in range(2)]
    res_all = []
    for fused in (False, True):
        b = base.clone().requires_grad_(True)
        a = attr.clone().requires_grad_(True)
        if fused:
            layers = diffrast.rasterize_interpolate_layers(b, tri, res, a, M, targets=tuple(tg))
            outs = [(r, d, o, od, (lo if tg[l] is not None else None)) for l, (r, d, o, od, lo) in enumerate(layers)]
        else:
            outs = []
            for l, (r, d) in enumerate(diffrast.rasterize_layers(b, tri, res, 2, grad_db=True, xform=M)):
                if tg[l] is not None:
                    lo, o, od = diffrast.interpolate_mse(a, r, tri, tg[l], d, "all")
                else:
                    (o, od), lo = diffrast.interpolate(a, r, tri, d, "all"), None
                outs.append((r, d, o, od, lo))
        total = 0.0
        for l, (r, d, o, od, lo) in enumerate(outs):
            total = total + (lo if lo is not None else (o * w[l]).sum())
        total.backward()
        res_all.append(([[t.detach().cpu().numpy() for t in x[:4]] for x in outs],
                        [float(x[4]) if x[4] is not None else None for x in outs],
                        a.grad.cpu().numpy(), b.grad.cpu().numpy()))
    (t0, l0, ga0, gb0), (t1, l1, ga1, gb1) = res_all
    for l in range(2):
        for k in range(4):
            assert np.array_equal(t0[l][k], t1[l][k]), (l, k)
        if l0[l] is not None:
            assert abs(l1[l] - l0[l]) <= 1e-5 * abs(l0[l])
    assert rel_l2(ga1, ga0) < 1e-5 and np.abs(ga0).sum() > 0
    assert rel_l2(gb1, gb0) < 1e-4 and np.abs(gb0).sum() > 0


def test_fused_rejects_a_channel_count_off_four(soup):
    import torch

    import diffrast
    base, tri, M = soup
    with pytest.raises(ValueError, match="multiple of 4"):
        diffrast.rasterize_interpolate_layers(base, tri, (32, 32), torch.zeros((base.shape[0], 3), device="cuda"), M)


@pytest.mark.parametrize("shared", [True, False])
@pytest.mark.parametrize("use_da", [False, True])
def test_fused_vjp_matches_separate_vjps(soup, shared, use_da):
    # The one-pass VJP (only out reaches the loss: a plain cotangent on layer 0,
    # the fused loss on layer 1) against the separate VJP kernels on the same
    # forward.  With out_da in the loss both runs take the separate VJPs.
    import torch

    import diffrast
    from diffrast import ops
    base, tri, M = soup
    res = (100, 72)
    N, V, A = M.shape[0], base.shape[0], 8
    g = torch.Generator(device="cuda")
    g.manual_seed(91)
    attr = torch.randn(((V, A) if shared else (N, V, A)), generator=g, device="cuda")
    tg1 = torch.randn((N,) + res + (A,), generator=g, device="cuda")
    w0 = torch.randn((N,) + res + (A,), generator=g, device="cuda")
    wd = torch.randn((N,) + res + (2 * A,), generator=g, device="cuda")
    grads = []
    for fused_vjp in (True, False):
        ops.FUSED_LAYERS_VJP = fused_vjp
        try:
            b = base.clone().requires_grad_(True)
            a = attr.clone().requires_grad_(True)
            l0, l1 = diffrast.rasterize_interpolate_layers(b, tri, res, a, M, targets=(None, tg1))
            total = (l0[2] * w0).sum() + 0.5 * l1[4]
            if use_da:
                total = total + (l0[3] * wd).sum()
            total.backward()
        finally:
            ops.FUSED_LAYERS_VJP = True
        grads.append((a.grad.cpu().numpy(), b.grad.cpu().numpy()))
    (ga0, gb0), (ga1, gb1) = grads
    assert rel_l2(ga0, ga1) < 1e-5 and np.abs(ga1).sum() > 0
    assert rel_l2(gb0, gb1) < 1e-4 and np.abs(gb1).sum() > 0


def test_fused_vjp_abi_checks(soup):
    # dr_rasterize_xf_interp_bwd's own argument checks (through the C ABI):
    # inconsistent cotangents and misaligned or misshaped tables are
    # DR_EINVAL with a message; no cotangent at all zeroes both outputs.
    import ctypes

    import torch

    from diffrast import _lib
    base, tri, M = soup
    L = _lib.lib()
    c = _lib.ctx_for(base.device.index or 0)
    N, V, T, H, W, A = M.shape[0], base.shape[0], tri.shape[0], 16, 24, 8
    attr = torch.randn((V, A), device="cuda")
    rast = [torch.zeros((N, H, W, 4), device="cuda") for _ in range(2)]
    out = [torch.zeros((N, H, W, A), device="cuda") for _ in range(2)]
    tgt = torch.zeros((N, H, W, A), device="cuda")
    dl = torch.ones((), device="cuda")
    d_attr = torch.full((V, A), 7.0, device="cuda")
    d_verts = torch.full((V, 4), 7.0, device="cuda")

    def pair(a, b):
        return ctypes.cast((ctypes.c_void_p * 2)(a.data_ptr() if a is not None else None,
                                                  b.data_ptr() if b is not None else None), ctypes.c_void_p)

    def call(A_=A, attr_=attr, d_out=None, o=None, t=None, d=None):
        return L.dr_rasterize_xf_interp_bwd(c, base.data_ptr(), V, M.data_ptr(), tri.data_ptr(), T, N, H, W,
                                            attr_.data_ptr(), 1, A_, pair(*rast), d_out, o, t, 1.0 / out[0].numel(),
                                            d, d_attr.data_ptr(), d_verts.data_ptr())

    st = call(o=pair(out[0], None), t=pair(None, None), d=pair(dl, None))
    assert st == _lib.DR_EINVAL and b"go together" in L.dr_last_error(c)
    st = call(d_out=pair(out[1], None), o=pair(out[0], None), t=pair(tgt, None), d=pair(dl, None))
    assert st == _lib.DR_EINVAL and b"not both" in L.dr_last_error(c)
    st = call(A_=6)
    assert st == _lib.DR_EINVAL and b"multiple of 4" in L.dr_last_error(c)
    flat = torch.zeros(V * A + 4, device="cuda")
    st = call(attr_=flat[1:1 + V * A])
    assert st == _lib.DR_EINVAL and b"16-byte aligned" in L.dr_last_error(c)
    st = call()
    torch.cuda.synchronize()
    assert st == _lib.DR_OK
    assert float(d_attr.abs().sum()) == 0.0 and float(d_verts.abs().sum()) == 0.0
