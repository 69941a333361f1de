"""Seeded synthetic inputs for the parity tests (numpy, CPU)."""
from __future__ import annotations

import numpy as np


def lam_init(rng, H, N, tau_min, tau_max, imag_scale=1.0):
    """spectral_init.py:28-47: Re = -1/tau (tau log-uniform), Im = pi*n*imag_scale."""
    log_tau = rng.uniform(np.log(tau_min), np.log(tau_max), (H, N))
    re = -np.exp(-log_tau)
    im = np.broadcast_to(np.pi * np.arange(N) * imag_scale, (H, N))
    return (re + 1j * im).astype(np.complex64)


def timestamps(rng, B, L, kind="exp", mean=0.25):
    if kind == "exp":
        dt = np.clip(rng.exponential(mean, (B, L)), 1 / 30, 2.0)
    else:  # adaptive-sampler style: U[0.25, 2] with 10% bursts at 0.25 s
        dt = rng.uniform(0.25, 2.0, (B, L))
        dt[rng.random((B, L)) < 0.1] = 0.25
    return np.cumsum(dt, 1).astype(np.float32)


def cplx(rng, shape, scale):
    return ((rng.standard_normal(shape) + 1j * rng.standard_normal(shape)) * scale).astype(np.complex64)


def cell_inputs(B, L, H, N, seed, tau=(0.5, 4.0), t_kind="exp"):
    rng = np.random.default_rng(seed)
    d = dict(
        lam=lam_init(rng, H, N, *tau),
        log_dt=(rng.standard_normal(H) * 0.2).astype(np.float32),
        u=rng.standard_normal((B, L, H)).astype(np.float32),
        Bc=cplx(rng, (B, L, N), 1 / np.sqrt(2 * N)),
        Cc=cplx(rng, (B, L, N), 1 / np.sqrt(2 * N)),
        t=timestamps(rng, B, L, t_kind),
        D=rng.standard_normal(H).astype(np.float32),
        mean=(rng.standard_normal(H) * 0.1).astype(np.float32),
        var=rng.uniform(0.5, 1.5, H).astype(np.float32),
    )
    return d


def scan_inputs(B, L, H, N, seed):
    rng = np.random.default_rng(seed)
    mag = rng.uniform(0.69, 0.999, (B, L, H, N))
    ph = rng.uniform(0, 2 * np.pi, (B, L, H, N))
    a = (mag * np.exp(1j * ph)).astype(np.complex64)
    b = cplx(rng, (B, L, H, N), 1.0)
    g = cplx(rng, (B, L, H, N), 1.0)
    return a, b, g
