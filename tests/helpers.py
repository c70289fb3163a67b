"""Shared test helpers: error metrics and seeded inputs.

Parity bar (north star): max |d| / ||ref||_inf <= 1e-3 and
max_i |d_i| / max(|ref_i|, 1e-3 * ||ref||_inf) <= 1e-3, fp32 accumulation.
"""
import numpy as np

TOL = 1e-3


def errs(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    inf = np.abs(ref).max()
    d = np.abs(y - ref)
    if inf == 0:
        return float(d.max()), float(d.max())
    return float(d.max() / inf), float((d / np.maximum(np.abs(ref), 1e-3 * inf)).max())


def assert_close(y, ref, tol=TOL, what=""):
    a, b = errs(y, ref)
    assert a <= tol and b <= tol, f"{what}: max|d|/||ref||={a:.3e} max elementwise rel={b:.3e} (tol {tol})"
    return a, b


def rng(seed):
    return np.random.default_rng(seed)
