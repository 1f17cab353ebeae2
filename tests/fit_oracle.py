"""The example fits driven by the CPU oracle (test infrastructure): the same
scenes and loops as mlx-swift-diffrast_b200/examples/fits.py, every op and
VJP from oracle/, Adam from oracle.adam_step."""
import numpy as np

import oracle
import oracle.chains as OC


def run_color(s, steps=None):
    res = (s["res"], s["res"])
    rast, _ = oracle.rasterize(s["pos"], s["tri"], res, grad_db=False)
    target_img, _ = oracle.interpolate(s["target"], rast, s["tri"])
    attr = s["init"].copy()
    m = np.zeros_like(attr); v = np.zeros_like(attr)
    losses = []
    for t in range(1, (steps or s["steps"]) + 1):
        out, _ = oracle.interpolate(attr, rast, s["tri"])
        loss, d_out = oracle.mse_fwd_bwd(out, target_img, 1.0 / out.size)
        d_attr, _, _ = oracle.interpolate_bwd(attr, rast, s["tri"], d_out)
        losses.append(float(loss))
        attr, m, v = oracle.adam_step(attr, d_attr.reshape(attr.shape), m, v, t, s["lr"])
    return losses, attr


def run_pos(s, steps=None):
    res = (s["res"], s["res"])
    topo = oracle.topology_hash(s["tri"])

    def render(p):
        rast, _ = oracle.rasterize(p, s["tri"], res, grad_db=False)
        col, _ = oracle.interpolate(s["attr"], rast, s["tri"])
        return oracle.antialias(col, rast, p, s["tri"], topo)

    target_img = render(s["target"])
    pos = s["init"].copy()
    m = np.zeros_like(pos); v = np.zeros_like(pos)
    losses = []
    for t in range(1, (steps or s["steps"]) + 1):
        loss, g = OC.cfg1(pos, s["tri"], s["attr"], target_img, res, topo=topo)
        losses.append(float(loss))
        pos, m, v = oracle.adam_step(pos, g["pos"], m, v, t, s["lr"], mask=s["mask"])
    return losses, pos
