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
