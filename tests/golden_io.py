"""Loader for the committed golden vectors (tests/golden/*.npz)."""
from __future__ import annotations

import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cases(group: str) -> dict[str, dict[str, np.ndarray]]:
    z = np.load(os.path.join(GOLDEN, f"{group}.npz"))
    out: dict[str, dict[str, np.ndarray]] = {}
    for key in z.files:
        case, name = key.split("/", 1)
        out.setdefault(case, {})[name] = z[key]
    return out


def relerr(x, ref) -> float:
    """max |x - ref| / max |ref| (complex magnitudes for complex arrays)."""
    x = np.asarray(x)
    ref = np.asarray(ref)
    den = float(np.max(np.abs(ref))) if ref.size else 0.0
    num = float(np.max(np.abs(x - ref))) if ref.size else 0.0
    return num / max(den, 1e-30)


def cell_args(d):
    eps, eta, var_eps, dt_init, dt_min, dt_max = [float(v) for v in d["scalars"][:6]]
    rb = d["robust"]
    robust = None if rb[0] < 0 else (int(rb[0]), float(rb[1]), float(rb[2]))
    return dict(eps=eps, eta=eta, var_eps=var_eps, dt_init=dt_init, dt_min=dt_min,
                dt_max=dt_max, robust=robust)


def decisive(resid, eps, robust, margin=1e-5):
    """Mask of steps whose gate is decided by more than `margin` (r vs eps_l)."""
    gap = np.abs(resid - eps)
    if robust is not None:
        gap = np.minimum(gap, np.abs(resid - np.float32(eps) * np.float32(robust[2])))
    return gap > margin


def assert_cell_match(got, ref, eps, robust, tol=1e-4):
    """Gate masks bit-exact and outputs within tol, row by row up to the first
    step whose residual is within 1e-5 of its threshold (after it the
    trajectories may legitimately part).  Returns the steps compared."""
    y, g, r = got
    y_ref, g_ref, r_ref = ref
    dec = decisive(r_ref, eps, robust)
    compared = 0
    for bi in range(g_ref.shape[0]):
        bad = np.where(~dec[bi])[0]
        stop = int(bad[0]) if bad.size else g_ref.shape[1]
        assert np.array_equal(g[bi, :stop], g_ref[bi, :stop]), f"row {bi}: gates differ"
        assert relerr(r[bi, :stop], r_ref[bi, :stop]) < tol, f"row {bi}: resid"
        assert relerr(y[bi, :stop], y_ref[bi, :stop]) < tol, f"row {bi}: y"
        compared += stop
    assert compared >= 0.9 * g_ref.size
    return compared
