"""Seeded synthetic scenes for the benchmark configurations (numpy, host side).

The reference publishes no dataset or benchmark inputs; these generators build
the scenes the configurations describe (icosphere mesh fits, a large triangle
soup with edge-sharing strips, a geodesic sphere with a cube map) from fixed
numpy PCG64 seeds, so every run and every rank sees identical data.
"""
from __future__ import annotations

import math

import numpy as np


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


# ------------------------------------------------------------------ meshes

def _icosahedron():
    t = (1.0 + 5.0 ** 0.5) / 2.0
    v = np.array([[-1, t, 0], [1, t, 0], [-1, -t, 0], [1, -t, 0], [0, -1, t], [0, 1, t], [0, -1, -t],
                  [0, 1, -t], [t, 0, -1], [t, 0, 1], [-t, 0, -1], [-t, 0, 1]], np.float64)
    f = np.array([[0, 11, 5], [0, 5, 1], [0, 1, 7], [0, 7, 10], [0, 10, 11], [1, 5, 9], [5, 11, 4],
                  [11, 10, 2], [10, 7, 6], [7, 1, 8], [3, 9, 4], [3, 4, 2], [3, 2, 6], [3, 6, 8],
                  [3, 8, 9], [4, 9, 5], [2, 4, 11], [6, 2, 10], [8, 6, 7], [9, 8, 1]], np.int64)
    return v / np.linalg.norm(v, axis=1, keepdims=True), f


def geodesic_sphere(freq: int):
    """Frequency-`freq` geodesic sphere: each icosahedron face split into freq^2
    triangles, vertices projected to the unit sphere.  V = 10 f^2 + 2, T = 20 f^2."""
    v0, f0 = _icosahedron()
    verts = {}
    out_v = []

    def vid(key, p):
        if key not in verts:
            verts[key] = len(out_v)
            out_v.append(p / np.linalg.norm(p))
        return verts[key]

    def key_of(face_corners, i, j):
        # Canonical key: barycentric point expressed on the global corner ids so
        # shared edges and corners dedupe across faces.
        a, b, c = face_corners
        k = freq - i - j
        items = sorted([(a, k), (b, i), (c, j)])
        return tuple((cid, w) for cid, w in items if w > 0)

    tris = []
    for fa in f0:
        A, B, C = v0[fa[0]], v0[fa[1]], v0[fa[2]]
        idx = {}
        for i in range(freq + 1):
            for j in range(freq + 1 - i):
                k = freq - i - j
                p = (A * k + B * i + C * j) / freq
                idx[(i, j)] = vid(key_of(fa, i, j), p)
        for i in range(freq):
            for j in range(freq - i):
                tris.append([idx[(i, j)], idx[(i + 1, j)], idx[(i, j + 1)]])
                if i + j < freq - 1:
                    tris.append([idx[(i + 1, j)], idx[(i + 1, j + 1)], idx[(i, j + 1)]])
    return np.array(out_v, np.float64), np.array(tris, np.int32)


def icosphere(level: int):
    """Icosphere of subdivision level L (frequency-2^L geodesic split, the same
    topology as L midpoint subdivisions): 10*4^L + 2 vertices, 20*4^L faces."""
    return geodesic_sphere(2 ** level)


def jitter_radial(v: np.ndarray, sigma: float, seed: int) -> np.ndarray:
    r = 1.0 + rng(seed).normal(0.0, sigma, size=(v.shape[0], 1))
    return v * r


def random_rotations(n: int, seed: int) -> np.ndarray:
    """n uniformly random rotation matrices (uniform unit quaternions)."""
    g = rng(seed)
    q = g.normal(size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    R = np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)], -1),
        np.stack([2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)], -1),
        np.stack([2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)], -1)], 1)
    return R


def perspective(fov_deg=45.0, aspect=1.0, near=1.0, far=10.0) -> np.ndarray:
    f = 1.0 / math.tan(math.radians(fov_deg) / 2)
    return np.array([[f / aspect, 0, 0, 0], [0, f, 0, 0],
                     [0, 0, -(far + near) / (far - near), -2 * far * near / (far - near)],
                     [0, 0, -1, 0]], np.float64)


def view_mvps(n_views: int, seed: int, distance: float = 3.0) -> np.ndarray:
    """[n, 4, 4] clip-from-object matrices: random rotation, camera at z=+distance
    looking at the origin, perspective fov 45 deg, near 1, far 10."""
    R = random_rotations(n_views, seed)
    M = np.zeros((n_views, 4, 4))
    M[:, :3, :3] = R
    M[:, 3, 3] = 1.0
    Vw = np.eye(4)
    Vw[2, 3] = -distance
    return perspective() @ Vw @ M


def clip_positions(verts: np.ndarray, mvps: np.ndarray) -> np.ndarray:
    vh = np.concatenate([verts, np.ones((verts.shape[0], 1))], 1)
    return np.einsum("nij,vj->nvi", mvps, vh).astype(np.float32)


def spherical_uv(unit: np.ndarray) -> np.ndarray:
    u = 0.5 + np.arctan2(unit[:, 2], unit[:, 0]) / (2 * np.pi)
    v = 0.5 - np.arcsin(np.clip(unit[:, 1], -1, 1)) / np.pi
    return np.stack([u, v], 1).astype(np.float32)


def value_noise(H: int, W: int, C: int, seed: int, octaves: int = 4) -> np.ndarray:
    """Smooth periodic value noise in [0, 1]: sum of octaves of bilinearly
    upsampled random lattices (base lattice 8x8, doubling per octave)."""
    g = rng(seed)
    out = np.zeros((H, W, C), np.float64)
    amp, tot = 1.0, 0.0
    for o in range(octaves):
        n = 8 * (2 ** o)
        lat = g.random((n, n, C))
        ys = (np.arange(H) + 0.5) * n / H - 0.5
        xs = (np.arange(W) + 0.5) * n / W - 0.5
        y0 = np.floor(ys).astype(int); fy = (ys - y0)[:, None, None]
        x0 = np.floor(xs).astype(int); fx = (xs - x0)[None, :, None]
        y0m, y1m = y0 % n, (y0 + 1) % n
        x0m, x1m = x0 % n, (x0 + 1) % n
        a = lat[y0m][:, x0m]; b = lat[y0m][:, x1m]; c = lat[y1m][:, x0m]; d = lat[y1m][:, x1m]
        out += amp * ((1 - fy) * ((1 - fx) * a + fx * b) + fy * ((1 - fx) * c + fx * d))
        tot += amp
        amp *= 0.5
    return (out / tot).astype(np.float32)


# ------------------------------------------------------- triangle soup (cfg4)

def triangle_soup(n_isolated: int, n_strips: int, strip_len: int, seed: int):
    """Clip-space triangle soup: isolated triangles plus edge-sharing strips.

    Centres ~U[-1,1]^2 (NDC), edge length ~U[0.002, 0.02], random orientation,
    per-vertex w ~U[1, 10] with (x, y, z) = ndc * w and z_ndc ~U[-0.9, 0.9].
    Returns pos [V, 4] float32 and tri [T, 3] int32 (isolated first, strips after).
    """
    g = rng(seed)
    # isolated triangles: 3 fresh vertices each
    c = g.uniform(-1, 1, size=(n_isolated, 2))
    L = g.uniform(0.002, 0.02, size=(n_isolated, 1))
    th = g.uniform(0, 2 * np.pi, size=(n_isolated, 1))
    ang = th + np.array([0.0, 2 * np.pi / 3, 4 * np.pi / 3])[None, :]
    r = L / np.sqrt(3.0)
    xy_iso = np.stack([c[:, :1] + r * np.cos(ang), c[:, 1:] + r * np.sin(ang)], -1).reshape(-1, 2)
    # strips: strip_len triangles over strip_len + 2 vertices zig-zagging along a direction
    nv_s = strip_len + 2
    cs = g.uniform(-1, 1, size=(n_strips, 1, 2))
    Ls = g.uniform(0.002, 0.02, size=(n_strips, 1, 1))
    ths = g.uniform(0, 2 * np.pi, size=(n_strips, 1))
    d = np.stack([np.cos(ths), np.sin(ths)], -1)            # [S,1,2] strip direction
    nrm = np.stack([-np.sin(ths), np.cos(ths)], -1)         # [S,1,2] side normal
    k = np.arange(nv_s)[None, :, None]
    side = np.where(k % 2 == 0, -0.5, 0.5)
    xy_str = cs + Ls * (0.5 * (k - (nv_s - 1) / 2.0) * d + side * np.sqrt(3.0) * nrm)
    xy_str = xy_str.reshape(-1, 2)
    xy = np.concatenate([xy_iso, xy_str], 0)
    V = xy.shape[0]
    w = g.uniform(1.0, 10.0, size=(V, 1))
    z = g.uniform(-0.9, 0.9, size=(V, 1))
    pos = np.concatenate([xy * w, z * w, w], 1).astype(np.float32)
    tri_iso = np.arange(3 * n_isolated, dtype=np.int64).reshape(-1, 3)
    base = 3 * n_isolated + nv_s * np.arange(n_strips)[:, None]
    j = np.arange(strip_len)[None, :]
    tri_str = np.stack([base + j, base + j + 1, base + j + 2], -1).reshape(-1, 3)
    tri = np.concatenate([tri_iso, tri_str], 0).astype(np.int32)
    return pos, tri


def similarity_matrices(n_views: int, seed: int) -> np.ndarray:
    """[n, 4, 4] clip-space matrices applying a 2-D similarity to NDC xy:
    ndc' = s R ndc + shift, i.e. x' = s(R00 x + R01 y) + shift_x w."""
    g = rng(seed)
    th = g.uniform(0, 2 * np.pi, n_views)
    s = g.uniform(0.9, 1.1, n_views)
    sh = g.uniform(-0.05, 0.05, size=(n_views, 2))
    M = np.zeros((n_views, 4, 4))
    M[:, 0, 0] = s * np.cos(th); M[:, 0, 1] = -s * np.sin(th); M[:, 0, 3] = sh[:, 0]
    M[:, 1, 0] = s * np.sin(th); M[:, 1, 1] = s * np.cos(th); M[:, 1, 3] = sh[:, 1]
    M[:, 2, 2] = 1.0
    M[:, 3, 3] = 1.0
    return M


# ------------------------------------------------------------ config scenes

def scene_cfg1():
    pos = np.array([[[-0.8, -0.8, 0, 1], [0.8, -0.8, 0, 1], [0, 0.8, 0, 1]]], np.float32)
    tri = np.array([[0, 1, 2]], np.int32)
    rgb = rng(1).random((3, 3)).astype(np.float32)
    target = rng(2).random((1, 256, 256, 3)).astype(np.float32)
    return dict(pos=pos, tri=tri, attr=rgb, target=target, res=(256, 256))


def scene_icosphere_views(n_views: int, res: int, jitter: float = 0.02, level: int = 4,
                          seed_mesh: int = 3, seed_rot: int = 4):
    unit, tri = icosphere(level)
    verts = jitter_radial(unit, jitter, seed_mesh)
    mvps = view_mvps(n_views, seed_rot)
    pos = clip_positions(verts, mvps)
    return dict(unit=unit.astype(np.float32), verts=verts.astype(np.float32), tri=tri,
                mvps=mvps.astype(np.float32), pos=pos, res=(res, res))


def scene_cfg2(n_views: int = 8, res: int = 512, tex: int = 512, level: int = 4):
    s = scene_icosphere_views(n_views, res, level=level)
    V = s["pos"].shape[1]
    s["rgb"] = rng(5).random((V, 3)).astype(np.float32)
    s["uv"] = spherical_uv(s["unit"])
    s["tex"] = rng(6).random((1, tex, tex, 3)).astype(np.float32)
    s["target"] = rng(7).random((n_views, res, res, 3)).astype(np.float32)
    return s


def scene_cfg3(n_views: int = 16, res: int = 1024, tex: int = 2048, level: int = 4):
    s = scene_icosphere_views(n_views, res, level=level)
    s["uv"] = spherical_uv(s["unit"])
    s["tex"] = value_noise(tex, tex, 4, seed=8)[None]
    s["bias_map"] = rng(9).uniform(-1, 1, (n_views, res, res)).astype(np.float32)
    s["target"] = rng(10).random((n_views, res, res, 4)).astype(np.float32)
    return s


def scene_cfg4(n_views: int = 32, res: int = 1024, n_isolated: int = 800_000, n_strips: int = 20_000,
               strip_len: int = 10):
    base, tri = triangle_soup(n_isolated, n_strips, strip_len, seed=10)
    M = similarity_matrices(n_views, seed=11)
    V = base.shape[0]
    attr = rng(12).normal(size=(V, 8)).astype(np.float32)
    return dict(base=base, tri=tri, sim=M.astype(np.float32), attr=attr, res=(res, res),
                n_views=n_views, target_seed=13)


def scene_cfg5(n_views: int = 256, res: int = 2048, freq: int = 158, cube: int = 1024):
    unit, tri = geodesic_sphere(freq)
    verts = jitter_radial(unit, 0.01, 13)
    mvps = view_mvps(n_views, 14)
    cube_tex = rng(15).random((1, 6, cube, cube, 3)).astype(np.float32)
    return dict(unit=unit.astype(np.float32), verts=verts.astype(np.float32), tri=tri,
                mvps=mvps.astype(np.float32), cube=cube_tex, res=(res, res), n_views=n_views, target_seed=16)
