"""What the reference's own gated-cell CUDA kernel computes on B200.

The kernel is eacs_cell_fwd_kernel (cst_ssm/ops/csrc/eacs_cell_cuda.cu:36-168,
"K3"), compiled unchanged for sm_100a by oracle/build_ref.py into
oracle/_ref/ (skipped when that build is absent).  Read step by step, its
source is the reference's scan_range (modules/eacs.py:145-173): a numpy
transliteration of it agrees with the oracle to ~2e-7 on bench.py's inputs.
On B200 its outputs differ from that for every channel h with h mod 256 != 0
(K3 runs 256 threads per row, thread h mod 256 owning channel h), and they are
reproduced to ~1e-7 by `stale_t_model` below: the same recurrence in which
every thread except thread 0 keeps the row's initial committed time
t_pi = t_0 - dt_init for all steps.  In the source, t_pi[b] sits behind a
`float* __restrict__` pointer that thread 0 alone stores to (:164) and all
threads load (:79); the observed outputs are what results if the threads
that never store keep their first load of it in a register.

This project's kernels are held to the reference's scan_range semantics (the
oracle, pinned by tests/golden/ to the reference's PyTorch code); K3 is used
as a timing baseline only.
"""
import os

import numpy as np
import pytest
import torch

from golden_io import assert_cell_match, relerr
from oracle import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
K3_SO = os.path.join(ROOT, "oracle", "_ref", "ref_eacs_cell_cuda", "ref_eacs_cell_cuda.so")
pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not os.path.exists(K3_SO), reason="K3 not built")]

THREADS = 256  # K3's block size (eacs_cell_cuda.cu:204)
f32 = np.float32


def stale_t_model(lam, log_dt, u, Bc, Cc, t, D, mean, var, eps, eta=1e-6, var_eps=1e-5,
                  dt_init=1.0, dt_min=1e-3, dt_max=1e3):
    """scan_range's hard-gate cell in float32, except that channels owned by
    threads other than 0 use t_pi = t_0 - dt_init at every step."""
    B, L, H = u.shape
    y = np.zeros((B, L, H), f32)
    gate = np.zeros((B, L), f32)
    resid = np.zeros((B, L), f32)
    scale = np.exp(log_dt).astype(f32)
    sd = np.sqrt(var + f32(var_eps)).astype(f32)
    owner0 = (np.arange(H) % THREADS) == 0
    for b in range(B):
        h = np.zeros(lam.shape, np.complex64)
        u_pi, B_pi, C_pi = u[b, 0].copy(), Bc[b, 0].copy(), Cc[b, 0].copy()
        t0 = f32(t[b, 0] - f32(dt_init))
        t_pi = t0
        for l in range(L):
            t_seen = np.where(owner0, t_pi, t0).astype(f32)
            delta = np.maximum(f32(t[b, l]) - t_seen, f32(0))
            dte = np.clip(delta * scale, f32(dt_min), f32(dt_max)).astype(f32)
            z = (lam * dte[:, None]).astype(np.complex64)
            dA = np.exp(z).astype(np.complex64)
            a, bb = z.real, z.imag
            sh = np.sin(f32(0.5) * bb)
            E = (np.expm1(a) * np.cos(bb) - f32(2) * sh * sh + 1j * (np.expm1(a) + f32(1)) * np.sin(bb))
            dBbar = (E.astype(np.complex64) / lam).astype(np.complex64)
            x_hat = dA * h + dBbar * B_pi[None, :] * u_pi[:, None]
            y_hat = (C_pi[None, :] * x_hat).real.sum(1).astype(f32)
            diff = (u[b, l] - y_hat) / sd
            obs = (u[b, l] - mean) / sd
            r = np.sqrt((diff * diff).sum()) / (np.sqrt((obs * obs).sum()) + f32(eta))
            g = f32(r > eps)
            gate[b, l], resid[b, l] = g, r
            if g > 0.5:
                h = (dA * h + dBbar * Bc[b, l][None, :] * u[b, l][:, None]).astype(np.complex64)
                y[b, l] = (Cc[b, l][None, :] * h).real.sum(1) + D * u[b, l]
                u_pi, B_pi, C_pi, t_pi = u[b, l].copy(), Bc[b, l].copy(), Cc[b, l].copy(), f32(t[b, l])
            else:
                y[b, l] = (Cc[b, l][None, :] * x_hat).real.sum(1) + D * u[b, l]
    return y, gate, resid


def _case(B, L, H, N, seed):
    rng = np.random.default_rng(seed)
    tau = np.exp(rng.uniform(np.log(0.1), np.log(1.0), (H, N)))
    return dict(
        lam=(-1.0 / tau + 1j * np.pi * np.arange(N)[None, :]).astype(np.complex64),
        log_dt=(0.1 * rng.standard_normal(H)).astype(f32),
        u=rng.standard_normal((B, L, H)).astype(f32),
        Bc=((rng.standard_normal((B, L, N)) + 1j * rng.standard_normal((B, L, N))) / 4).astype(np.complex64),
        Cc=((rng.standard_normal((B, L, N)) + 1j * rng.standard_normal((B, L, N))) / 4).astype(np.complex64),
        t=np.cumsum(rng.uniform(0.25, 2.0, (B, L)), 1).astype(f32),
        D=rng.standard_normal(H).astype(f32),
        mean=(0.1 * rng.standard_normal(H)).astype(f32),
        var=rng.uniform(0.5, 2, H).astype(f32))


def _k3():
    import importlib.machinery
    import importlib.util
    loader = importlib.machinery.ExtensionFileLoader("ref_eacs_cell_cuda", K3_SO)
    mod = importlib.util.module_from_spec(importlib.util.spec_from_loader("ref_eacs_cell_cuda", loader))
    loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("B,L,H,N,eps", [(1, 8, 4, 2, 0.12), (1, 48, 300, 16, 0.12), (2, 16, 1, 3, 0.9),
                                         (2, 40, 20, 4, 0.9)])
def test_k3_on_b200_is_the_stale_t_pi_recurrence(B, L, H, N, eps):
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward
    d = _case(B, L, H, N, seed=B + L + H + N)
    T = {k: torch.from_numpy(v).to("cuda:0") for k, v in d.items()}
    args = (T["lam"], T["log_dt"], T["u"], T["Bc"], T["Cc"], T["t"], T["D"], T["mean"], T["var"])
    yk, gk, rk = (x.cpu().numpy() for x in _k3().eacs_cell_fwd(*args, eps, 1e-6, 1e-5, 1.0, 1e-3, 1e3))
    ym, gm, rm = stale_t_model(**d, eps=eps)
    yo, go, ro = oracle.cell_fwd(**d, eps=eps, eta=1e-6)
    y, g, r = (x.cpu().numpy() for x in eacs_cell_forward(*args, eps=eps, eta=1e-6))
    # K3 on B200 = the stale-t_pi recurrence
    assert_cell_match((yk, gk, rk), (ym, gm, rm), eps, None, tol=1e-5)
    # this library = scan_range (the oracle)
    assert_cell_match((y, g, r), (yo, go, ro), eps, None)
    if H == 1:  # thread 0 owns every channel: K3 is scan_range
        assert relerr(yk, yo) < 1e-5
    else:
        assert relerr(yk, yo) > 1e-4
