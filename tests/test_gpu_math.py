"""Accuracy of the fused discretisation (own sincos / expm1) against
complex128 ground truth, evaluated through eacs_zoh_kernels.

The ground truth is computed from the same float32 products a = Re(lam) dt,
b = Im(lam) dt the kernel forms, so the check isolates the function error.
Bounds on the complex values: dB_bar relative 2e-6 everywhere; dA relative
1e-6 where |dA| >= 1e-3 and absolute 1e-8 below (there e^a < 1e-3 and the
reference's own float expm1(a) + 1 is already 0 for a < -17).
"""
import numpy as np
import pytest
import torch

from golden_io import cases, relerr

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from eacs_b200.ops.discretization import zoh_kernels


def _truth(lam, dt):
    lr = lam.real.astype(np.float32)[None]
    li = lam.imag.astype(np.float32)[None]
    d = dt.astype(np.float32)[:, :, None]
    a = (lr * d).astype(np.float64)
    b = (li * d).astype(np.float64)
    z = a + 1j * b
    dA = np.exp(z)
    E = np.expm1(a) * np.cos(b) - 2 * np.sin(0.5 * b) ** 2 + 1j * np.exp(a) * np.sin(b)
    return dA, E / lam.astype(np.complex128)[None]


def _check(lam, dt, tol_a=1e-6, tol_b=2e-6):
    dA, dB = zoh_kernels(torch.from_numpy(lam).cuda(), torch.from_numpy(dt).cuda())
    dA = dA.cpu().numpy().astype(np.complex128)
    dB = dB.cpu().numpy().astype(np.complex128)
    tA, tB = _truth(lam, dt)
    ea = np.abs(dA - tA) / np.maximum(np.abs(tA), 1e-30)
    eb = np.abs(dB - tB) / np.maximum(np.abs(tB), 1e-30)
    big = np.abs(tA) >= 1e-3
    assert float(ea[big].max()) < tol_a, float(ea[big].max())
    assert float(np.abs(dA - tA)[~big].max(initial=0.0)) < 1e-8
    assert float(eb.max()) < tol_b, float(eb.max())


def test_zoh_config_ranges():
    rng = np.random.default_rng(0)
    H, N, M = 64, 64, 256
    tau = np.exp(rng.uniform(np.log(0.1), np.log(3600.0), (H, N)))
    im = np.pi * np.arange(N)[None, :] * rng.choice([1.0, 0.3, 0.1], (H, 1))
    lam = (-1.0 / tau + 1j * im).astype(np.complex64)
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(2.0 * 4), (M, H))).astype(np.float32)
    _check(lam, dt)


def test_zoh_wide_arguments():
    rng = np.random.default_rng(1)
    H, N, M = 32, 32, 128
    lam = (-np.exp(rng.uniform(-8, 3, (H, N))) + 1j * rng.uniform(-400, 400, (H, N))).astype(np.complex64)
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e3), (M, H))).astype(np.float32)
    # includes |b/2| well past the 8192 switch to the library sincosf and a < -87
    _check(lam, dt)


def test_zoh_small_angles():
    """Short steps on the first imaginary modes: |z| down to ~1e-3, where
    expm1(z) must stay relatively exact (it sets dB_bar ~ dt)."""
    rng = np.random.default_rng(2)
    H, N, M = 32, 32, 128
    lam = (-np.exp(rng.uniform(-6, 0, (H, N))) + 1j * np.pi * rng.integers(1, 4, (H, N))).astype(np.complex64)
    dt = np.exp(rng.uniform(np.log(1e-3), np.log(3e-2), (M, H))).astype(np.float32)
    _check(lam, dt)


def test_zoh_near_full_turns():
    """b close to multiples of 2 pi with small a: |expm1(z)| small again."""
    rng = np.random.default_rng(3)
    H, N, M = 16, 16, 64
    n = rng.integers(1, 40, (H, N))
    lam = (-np.exp(rng.uniform(-7, -3, (H, N))) + 1j * np.pi * n).astype(np.complex64)
    # dt = 2 m / n (+ tiny offsets) puts b = pi n dt near 2 pi m
    m = rng.integers(1, 5, (M, H, N))
    base = (2.0 * m / n[None]) * (1 + rng.uniform(-1e-3, 1e-3, (M, H, N)))
    dt = base[:, :, 0].astype(np.float32)  # one dt per (step, channel): exact for n[:, 0]
    _check(lam, dt)


def test_zoh_against_reference_golden():
    """Values the reference's own zoh_kernels fed into its scan (ssm golden)."""
    d = cases("ssm")["ssm_odd"]
    t = d["t"]
    dt = np.zeros_like(t)
    dt[:, 1:] = np.maximum(t[:, 1:] - t[:, :-1], 0)
    dt[:, 0] = dt[:, 1]
    dte = np.clip(dt[..., None] * np.exp(d["log_dt"])[None, None], 1e-3, 1e3).astype(np.float32)
    dA, dB = zoh_kernels(torch.from_numpy(d["lam"]).cuda(), torch.from_numpy(dte).cuda())
    tA, tB = _truth(d["lam"], dte.reshape(-1, dte.shape[-1]))
    assert relerr(dA.cpu().numpy().reshape(tA.shape), tA) < 1e-6
    assert relerr(dB.cpu().numpy().reshape(tB.shape), tB) < 2e-6
