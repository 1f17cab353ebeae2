"""The reference's three example fits (Sources/ColorFitExample,
PoseFitExample, MeshFitExample), driven through diffrast on the GPU:
rasterize -> interpolate [-> antialias] -> MSE, Adam on the parameter.

Each `*_scene()` returns the fixed scene data as numpy arrays (shared with
the tests); `run_*` optimises on CUDA and returns (losses, final parameter,
target parameter, rendered target, final render).
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def color_scene():
    """ColorFitExample/main.swift: one triangle, 64^2, per-vertex RGB from
    mid-gray toward pure R, G, B; Adam lr 0.05, 120 steps; no antialias."""
    pos = np.array([[[-0.8, 0.8, 0, 1], [-0.8, -0.8, 0, 1], [0.8, 0.0, 0, 1]]], np.float32)
    tri = np.array([[0, 1, 2]], np.int32)
    target = np.array([[[1, 0, 0], [0, 1, 0], [0, 0, 1]]], np.float32)
    init = np.full((1, 3, 3), 0.5, np.float32)
    return dict(res=64, pos=pos, tri=tri, target=target, init=init, lr=0.05, steps=120)


def pose_scene():
    """PoseFitExample/main.swift: a two-triangle quad (x/y of its 4 vertices
    optimised), 64^2, reddish constant colour, antialias on; lr 0.01, 300 steps."""
    tri = np.array([[0, 1, 2], [0, 2, 3]], np.int32)
    attr = np.tile(np.array([0.95, 0.2, 0.2], np.float32), (1, 4, 1))
    target = np.array([[[-0.4, 0.4, 0, 1], [0.4, 0.4, 0, 1], [0.4, -0.4, 0, 1], [-0.4, -0.4, 0, 1]]], np.float32)
    init = np.array([[[-0.25, 0.55, 0, 1], [0.55, 0.55, 0, 1], [0.55, -0.25, 0, 1], [-0.25, -0.25, 0, 1]]],
                    np.float32)
    mask = np.tile(np.array([1, 1, 0, 0], np.float32), (1, 4, 1))
    return dict(res=64, tri=tri, attr=attr, target=target, init=init, mask=mask, lr=0.01, steps=300)


def _hexagon(cx, cy, r):
    v = [[cx, cy, 0, 1]]
    for k in range(6):
        a = np.float32(k) * np.float32(math.pi / 3)
        v.append([cx + r * math.cos(a), cy + r * math.sin(a), 0, 1])
    return np.array([v], np.float32)


def mesh_scene():
    """MeshFitExample/main.swift: a 7-vertex / 6-triangle hexagonal pie with
    per-vertex colours, 96^2, antialias on; lr 0.015, 400 steps."""
    tri = np.array([[0, 1, 2], [0, 2, 3], [0, 3, 4], [0, 4, 5], [0, 5, 6], [0, 6, 1]], np.int32)
    attr = np.array([[[1.0, 1.0, 1.0], [1.0, 0.2, 0.2], [1.0, 0.9, 0.2], [0.2, 0.9, 0.3], [0.2, 0.9, 0.9],
                      [0.3, 0.4, 1.0], [1.0, 0.3, 0.9]]], np.float32)
    target = _hexagon(0.0, 0.0, 0.55)
    init = _hexagon(0.13, -0.09, 0.42)
    mask = np.tile(np.array([1, 1, 0, 0], np.float32), (1, 7, 1))
    return dict(res=96, tri=tri, attr=attr, target=target, init=init, mask=mask, lr=0.015, steps=400)


def run_color(steps=None, device="cuda"):
    import torch

    import diffrast
    from diffrast.optim import Adam
    s = color_scene()
    dev = torch.device(device)
    pos, tri = torch.from_numpy(s["pos"]).to(dev), torch.from_numpy(s["tri"]).to(dev)
    rast, _ = diffrast.rasterize(pos, tri, (s["res"], s["res"]), grad_db=False)  # pos is fixed
    render = lambda a: diffrast.interpolate(a, rast, tri)[0]
    target_img = render(torch.from_numpy(s["target"]).to(dev))
    attr = torch.from_numpy(s["init"]).to(dev)
    opt = Adam(attr.shape, learning_rate=s["lr"], device=dev)
    losses = []
    for _ in range(steps or s["steps"]):
        a = attr.clone().requires_grad_(True)
        loss = diffrast.mse_loss(render(a), target_img)
        loss.backward()
        losses.append(float(loss.detach()))
        opt.step(attr, a.grad)
    return losses, attr.cpu().numpy(), s["target"], target_img.cpu().numpy(), render(attr).cpu().numpy()


def _run_pos(s, steps, device):
    import torch

    import diffrast
    from diffrast.optim import Adam
    dev = torch.device(device)
    tri = torch.from_numpy(s["tri"]).to(dev)
    attr = torch.from_numpy(s["attr"]).to(dev)
    topo = diffrast.antialias_construct_topology_hash(tri)
    hw = (s["res"], s["res"])

    def render(p):
        rast, _ = diffrast.rasterize(p, tri, hw, grad_db=False)
        col, _ = diffrast.interpolate(attr, rast, tri)
        return diffrast.antialias(col, rast, p, tri, topo)

    target_img = render(torch.from_numpy(s["target"]).to(dev))
    pos = torch.from_numpy(s["init"]).to(dev)
    mask = torch.from_numpy(s["mask"]).to(dev)
    opt = Adam(pos.shape, learning_rate=s["lr"], device=dev)
    losses = []
    for _ in range(steps or s["steps"]):
        p = pos.clone().requires_grad_(True)
        loss = diffrast.mse_loss(render(p), target_img)
        loss.backward()
        losses.append(float(loss.detach()))
        opt.step(pos, p.grad, mask)
    return losses, pos.cpu().numpy(), s["target"], target_img.cpu().numpy(), render(pos).cpu().numpy()


def run_pose(steps=None, device="cuda"):
    return _run_pos(pose_scene(), steps, device)


def run_mesh(steps=None, device="cuda"):
    return _run_pos(mesh_scene(), steps, device)


def write_side_by_side(path, target_img, current_img):
    """Headless image output: target | current as a binary PPM (the
    reference writes GIF frames through CoreGraphics)."""
    t = np.clip(target_img.reshape(target_img.shape[-3:]), 0, 1)
    c = np.clip(current_img.reshape(current_img.shape[-3:]), 0, 1)
    img = (np.concatenate([t, c], axis=1) * 255 + 0.5).astype(np.uint8)
    with open(path, "wb") as f:
        f.write(b"P6 %d %d 255\n" % (img.shape[1], img.shape[0]))
        f.write(img.tobytes())
