"""Small numeric helpers shared by the tests."""
import numpy as np


def fd_grad(f, x, eps=1e-3, skip=None):
    """Central finite differences of scalar f at x (float32 array), as the
    reference's gradchecks compute them (eps 1e-3)."""
    x = np.array(x, np.float32)
    g = np.zeros(x.size, np.float64)
    flat = x.reshape(-1)
    for i in range(flat.size):
        if skip is not None and skip(i):
            continue
        p = flat.copy(); p[i] += eps
        m = flat.copy(); m[i] -= eps
        g[i] = (f(p.reshape(x.shape)) - f(m.reshape(x.shape))) / (2 * eps)
    return g.reshape(x.shape)


def wsum(a, w):
    return float(np.sum(np.asarray(a, np.float64) * np.asarray(w, np.float64)))


def rel_l2(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    d = np.linalg.norm(a - b)
    n = np.linalg.norm(b)
    return d / n if n > 0 else d
