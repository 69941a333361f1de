"""Training path (GatedEACSCellFunction) against the reference's autograd
(golden vectors) and the double-precision oracle backward.

Tolerances: forward values 1e-4 relative, gradients 1e-3
relative (max |x - ref| / max |ref| per gradient tensor).
"""
import numpy as np
import pytest
import torch

from golden_io import cases, relerr
from inputs import cell_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from eacs_b200.ops.eacs_cell_train import GatedEACSCellFunction, fused_gated_scan

GRAD_TOL = 1e-3
FWD_TOL = 1e-4
NAMES = ["du", "dBc", "dCc", "dt", "dlam", "dlog_dt", "dD", "deps"]


def _run(d, eps, T, mode, gy, ggs=None, grs=None, gns=None, dt_max=1e3, u_dtype=torch.float32):
    dev = "cuda:0"
    def t(x, grad=True):
        v = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
        return v.requires_grad_(grad)
    u = t(d["u"]).detach().to(u_dtype).requires_grad_(True)
    Bc, Cc, tt = t(d["Bc"]), t(d["Cc"]), t(d["t"])
    lam, log_dt, D = t(d["lam"]), t(d["log_dt"]), t(d["D"])
    e = torch.tensor(float(eps), device=dev, requires_grad=True)
    mean, var = t(d["mean"], False), t(d["var"], False)
    ys, gs, rs, ns = GatedEACSCellFunction.apply(u, Bc, Cc, tt, lam, log_dt, D, e, mean, var, T,
                                                 1e-6, 1e-5, 1.0, mode, True, dt_max)
    outs, grads_in = [ys, gs, rs, ns], [gy, ggs, grs, gns]
    pairs = [(o, torch.from_numpy(g).to(dev)) for o, g in zip(outs, grads_in) if g is not None]
    grads = torch.autograd.grad([p[0] for p in pairs], [u, Bc, Cc, tt, lam, log_dt, D, e],
                                [p[1] for p in pairs])
    fwd = [x.detach().float().cpu().numpy() for x in (ys, gs, rs, ns)]
    return fwd, [g.detach().cpu().numpy() for g in grads]


@pytest.mark.parametrize("name", sorted(cases("train")))
def test_train_golden(name):
    d = cases("train")[name]
    eps, eta, var_eps, dt_init, dt_min, dt_max, T = [float(v) for v in d["scalars"]]
    mode = "ste" if int(d["gate_mode"][0]) == 0 else "soft"
    fwd, grads = _run(d, eps, T, mode, d["gy"], d["ggs"], d["grs"], d["gns"], dt_max=dt_max)
    y, g, r, n = fwd
    assert relerr(y, d["y"]) < FWD_TOL
    assert np.max(np.abs(g - d["gate"])) <= (0 if mode == "ste" else 1e-4)
    assert relerr(r, d["resid"]) < FWD_TOL
    assert np.array_equal(n, r)
    for k, v in zip(NAMES, grads):
        assert relerr(v.reshape(d[k].shape), d[k]) < GRAD_TOL, (k, relerr(v.reshape(d[k].shape), d[k]))


def _calibrated(d, rate):
    lo, hi = 0.0, 4.0
    for _ in range(30):
        mid = 0.5 * (lo + hi)
        _, g, _ = oracle.cell_fwd(**d, eps=mid, eta=1e-6, train_exp=True)
        lo, hi = (mid, hi) if g.mean() > rate else (lo, mid)
    eps = 0.5 * (lo + hi)
    for _ in range(200):
        _, _, r = oracle.cell_fwd(**d, eps=eps, eta=1e-6, train_exp=True)
        if np.abs(r - eps).min() > 2e-4:
            return eps
        eps *= 1.0006
    raise AssertionError("no eps away from the residuals")


@pytest.mark.parametrize("B,L,H,N,rate,T,mode", [
    (2, 40, 48, 16, 0.5, 0.3, "ste"),     # mixed gates, one CTA per row
    (2, 24, 768, 16, None, 0.1, "ste"),   # config-3 channels: 16-CTA cluster per row
    (2, 37, 100, 32, 0.6, 0.5, "ste"),    # 2-CTA clusters, ragged chunk
    (1, 20, 33, 5, 0.5, 0.4, "soft"),
    (3, 18, 20, 64, 0.4, 0.2, "ste"),
])
def test_train_vs_oracle(B, L, H, N, rate, T, mode):
    d = cell_inputs(B, L, H, N, seed=B * 100 + L + H + N)
    eps = 0.12 if rate is None else _calibrated(d, rate)
    rng = np.random.default_rng(L)
    gy = rng.standard_normal((B, L, H)).astype(np.float32)
    ggs = rng.standard_normal((B, L)).astype(np.float32)
    grs = rng.standard_normal((B, L)).astype(np.float32)
    gns = rng.standard_normal((B, L)).astype(np.float32)
    gate_mode = 0 if mode == "ste" else 1
    y_ref, g_ref, r_ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6, gate_mode=gate_mode, T=T,
                                          train_exp=True)
    fwd, grads = _run(d, eps, T, mode, gy, ggs, grs, gns)
    assert relerr(fwd[0], y_ref) < FWD_TOL
    assert np.max(np.abs(fwd[1] - g_ref)) <= (0 if mode == "ste" else 1e-4)
    ref = oracle.cell_bwd(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                          d["mean"], d["var"], eps, 1e-6, 1e-5, 1.0, 1e3, T, gate_mode,
                          fwd[1], gy, ggs, grs, gns)
    for k, v, rv in zip(NAMES, grads, ref):
        assert relerr(v.reshape(rv.shape), rv) < GRAD_TOL, (k, relerr(v.reshape(rv.shape), rv))


def test_fused_gated_scan_api_and_bf16_u():
    d = cell_inputs(2, 30, 64, 16, seed=5)
    dev = "cuda:0"
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    u = T(d["u"]).to(torch.bfloat16).requires_grad_(True)
    lam = T(d["lam"]).requires_grad_(True)
    eps = torch.tensor(0.12, device=dev, requires_grad=True)
    y, g, r = fused_gated_scan(u, T(d["Bc"]), T(d["Cc"]), T(d["t"]), lam, T(d["log_dt"]), T(d["D"]),
                               eps, T(d["mean"]), T(d["var"]), 0.1, 1e-6)
    (y.sum() + r.sum()).backward()
    assert u.grad.dtype == torch.bfloat16 and lam.grad.dtype == torch.complex64
    assert eps.grad.shape == eps.shape
    d["u"] = u.detach().float().cpu().numpy()
    gy = np.ones(y.shape, np.float32)
    ref = oracle.cell_bwd(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                          d["mean"], d["var"], 0.12, 1e-6, 1e-5, 1.0, 1e3, 0.1, 0,
                          g.detach().cpu().numpy(), gy, None, np.ones(r.shape, np.float32), None)
    assert relerr(lam.grad.cpu().numpy(), ref[4]) < GRAD_TOL


@pytest.mark.parametrize("B,L,H,N,rate,T,mode", [
    (2, 70, 768, 16, None, 0.1, "ste"),   # every frame commits: checkpoints from the speculative pass
    (2, 45, 64, 16, 0.5, 0.3, "ste"),     # skips: checkpoints from l* on from the repair pass
    (2, 33, 40, 32, 0.5, 0.4, "soft"),    # soft gate: every checkpoint from the repair pass
])
def test_forward_checkpoints_match_backward_pass(B, L, H, N, rate, T, mode):
    """The backward from the checkpoints the forward wrote
    (eacs_cell_train_fwd_ckpt / _bwd_ckpt) against the backward that runs its
    own checkpoint pass: the same gradients up to rounding (the two compute the
    checkpointed states with differently ordered arithmetic)."""
    from eacs_b200 import _lib
    from eacs_b200.ops.eacs_cell_train import _train_bwd, _train_fwd
    d = cell_inputs(B, L, H, N, seed=B + L + H + N)
    eps = 0.12 if rate is None else _calibrated(d, rate)
    dev = "cuda:0"
    tt = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in d.items()}
    rng = np.random.default_rng(7)
    gy = torch.from_numpy(rng.standard_normal((B, L, H)).astype(np.float32)).to(dev)
    grs = torch.from_numpy(rng.standard_normal((B, L)).astype(np.float32)).to(dev)
    args = (tt["u"], tt["Bc"], tt["Cc"], tt["t"], tt["lam"], tt["log_dt"], tt["D"], eps, tt["mean"], tt["var"],
            T, 1e-6, 1e-5, 1.0, mode, 1e3)
    ws = torch.empty(int(_lib.lib().eacs_cell_train_bwd_workspace_size(B, L, H, N)), dtype=torch.uint8,
                     device=dev)
    outs = []
    for bwd_ws in (None, ws):
        _, gs, rs, stats, prep = _train_fwd(*args, bwd_ws)
        outs.append((gs, _train_bwd(prep, gs, rs, stats, eps, T, 1e-6, 1e-5, 1.0, 1e3, gy, None, grs, None,
                                    bwd_ws)))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0], outs[1][0])
    if rate is not None:
        assert 0.0 < float(outs[0][0].mean()) < 1.0
    for k, a, b in zip(NAMES, outs[0][1], outs[1][1]):
        assert relerr(b.cpu().numpy(), a.cpu().numpy()) < 1e-5, (k, relerr(b.cpu().numpy(), a.cpu().numpy()))
