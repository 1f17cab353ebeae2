"""Whole benchmark chains (forward + every VJP) on the CUDA library vs the same
chains composed from the CPU oracle, per configuration at reduced sizes:
loss within 1e-5 relative, every parameter gradient within 1e-4 relative L2."""
import numpy as np
import pytest

from helpers import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch
    return torch.device("cuda", 0)


def _check(loss, grads, ref_loss, ref_grads):
    assert abs(float(loss) - ref_loss) <= 1e-5 * max(1.0, abs(ref_loss)), (float(loss), ref_loss)
    for k, g in grads.items():
        r = rel_l2(g, ref_grads[k])
        assert r < 1e-4, (k, r)


def test_cfg1_chain(dev):
    import oracle.chains as OC
    from diffrast import chains, scenes
    c = chains.Cfg1(dev)
    loss = c.step()
    s = scenes.scene_cfg1()
    ref_loss, ref = OC.cfg1(s["pos"], s["tri"], s["attr"], s["target"], s["res"])
    _check(loss.detach(), {"pos": c.pos.grad.cpu().numpy(), "rgb": c.rgb.grad.cpu().numpy()}, ref_loss, ref)


def test_cfg2_chain(dev):
    import oracle.chains as OC
    from diffrast import chains, scenes
    c = chains.Cfg2(dev, 0, 2, res=128, tex=64)
    loss = c.step()
    s = scenes.scene_cfg2(n_views=2, res=128, tex=64)
    ref_loss, ref = OC.cfg2(s["pos"], s["tri"], s["rgb"], s["uv"], s["tex"], s["target"], s["res"])
    got = {k: getattr(c, k).grad.cpu().numpy() for k in ("pos", "rgb", "uv", "tex")}
    _check(loss.detach(), got, ref_loss, ref)


def test_cfg3_chain(dev):
    import oracle.chains as OC
    from diffrast import chains, scenes
    c = chains.Cfg3(dev, 0, 1, res=128, tex=256)
    loss = c.step()
    s = scenes.scene_cfg3(n_views=1, res=128, tex=256)
    ref_loss, ref = OC.cfg3(s["pos"], s["tri"], s["uv"], s["tex"], s["bias_map"], s["target"], s["res"])
    got = {k: getattr(c, k).grad.cpu().numpy() for k in ("pos", "uv", "tex")}
    _check(loss.detach(), got, ref_loss, ref)


def test_cfg4_chain_per_view_transform(dev):
    import oracle
    import oracle.chains as OC
    from diffrast import chains
    c = chains.Cfg4(dev, 0, 2, total_views=2, res=256, n_isolated=20000, n_strips=1000)
    loss = c.step()
    base, sim = c.base.detach().cpu().numpy(), c.sim.cpu().numpy()
    pos = oracle.xf_positions(base, sim)
    ref_loss, ref = OC.cfg4(pos, c.tri.cpu().numpy(), c.attr.detach().cpu().numpy(), c.tgt0.cpu().numpy(),
                            c.tgt1.cpu().numpy(), c.res)
    ref = {"base": oracle.xf_vertex_grad(ref["pos"], sim), "attr": ref["attr"]}
    got = {"base": c.base.grad.cpu().numpy(), "attr": c.attr.grad.cpu().numpy()}
    _check(loss.detach(), got, ref_loss, ref)


@pytest.mark.parametrize("filt", ["linear", "linear-mipmap-linear"])
def test_cfg5_chain_microbatched_cube(dev, filt):
    import oracle
    import oracle.chains as OC
    from diffrast import chains, ops
    fm = ops.FilterMode.linear if filt == "linear" else ops.FilterMode.linearMipmapLinear
    c = chains.Cfg5(dev, 0, 3, micro=2, res=128, freq=8, cube=32, filter_mode=fm)
    loss = c.step()
    verts, mvp = c.verts.detach().cpu().numpy(), c.mvp.cpu().numpy()
    pos = oracle.xf_positions(verts, mvp)
    ref_loss, ref = OC.cfg5(pos, c.tri.cpu().numpy(), c.nrm.cpu().numpy(), c.cube.detach().cpu().numpy(),
                            c.target.cpu().numpy(), c.res, filter_mode=filt)
    ref = {"verts": oracle.xf_vertex_grad(ref["pos"], mvp), "cube": ref["cube"]}
    got = {"verts": c.verts.grad.cpu().numpy(), "cube": c.cube.grad.cpu().numpy()}
    _check(loss, got, ref_loss, ref)
