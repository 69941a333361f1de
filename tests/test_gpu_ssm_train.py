"""Training path of the fused ungated SSM core (eacs_ssm_train_fwd / eacs_ssm_bwd,
through SSMCoreFunction) against the reference's autograd (golden vectors,
tests/golden/ssm.npz) and the double-precision oracle.

Tolerances: forward 1e-4 relative, gradients 1e-3 relative, both as
max |x - ref| / max |ref| per output tensor.
"""
import numpy as np
import pytest
import torch

from golden_io import cases, relerr
from inputs import cell_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from eacs_b200 import _lib
    from eacs_b200.ops.continuous_ssm import ssm_forward

FWD_TOL = 1e-4
GRAD_TOL = 1e-3
DEV = "cuda:0"
NAMES = ["du", "dBc", "dCc", "dt", "dlam", "dlog_dt", "dD"]
U_DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _run(d, gy, u_dtype=torch.float32, dt_min=1e-3, dt_max=1e3):
    """y and the seven gradients through the autograd function."""
    lam, log_dt, t, Bc, Cc = (_t(d[k]).requires_grad_(True) for k in ("lam", "log_dt", "t", "Bc", "Cc"))
    u = _t(d["u"]).to(u_dtype).requires_grad_(True)
    D = _t(d["D"]).requires_grad_(True)
    y = ssm_forward(lam, log_dt, t, Bc, Cc, u, D, dt_min=dt_min, dt_max=dt_max)
    g = torch.autograd.grad(y, [lam, log_dt, t, Bc, Cc, u, D], _t(gy))
    got = dict(du=g[5], dBc=g[3], dCc=g[4], dt=g[2], dlam=g[0], dlog_dt=g[1], dD=g[6])
    return y.detach().cpu().numpy(), {k: v.float().cpu().numpy() if not v.is_complex()
                                      else v.cpu().numpy() for k, v in got.items()}


def _oracle(d, gy, dt_min=1e-3, dt_max=1e3):
    out = oracle.ssm_bwd(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"], d["u"], d["D"], gy,
                         dt_min=dt_min, dt_max=dt_max)
    return dict(zip(NAMES, out))


def _assert_grads(got, ref, tol=GRAD_TOL, du_tol=GRAD_TOL):
    for k in NAMES:
        e = relerr(got[k], ref[k])
        assert e < (du_tol if k == "du" else tol), (k, e)


@pytest.mark.parametrize("name", sorted(cases("ssm")))
def test_ssm_train_golden(name):
    d = cases("ssm")[name]
    y, got = _run(d, d["gy"])
    assert relerr(y, d["y"]) < FWD_TOL
    _assert_grads(got, d)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("B,L,H,N", [(2, 256, 64, 16), (1, 300, 40, 32), (2, 77, 19, 64),
                                     (3, 64, 33, 3), (1, 40, 128, 8), (2, 13, 7, 5),
                                     (1, 1, 4, 4), (1, 9, 130, 16), (2, 8, 16, 16)])
@pytest.mark.parametrize("u_dtype", ["f32", "bf16"])
def test_ssm_train_vs_oracle(B, L, H, N, u_dtype):
    d = cell_inputs(B, L, H, N, seed=B * L + N + H, tau=(0.5, 64.0))
    tdt = U_DTYPES[u_dtype]
    d["u"] = _t(d["u"]).to(tdt).float().cpu().numpy()  # the values the kernel reads
    gy = np.random.default_rng(B + L).standard_normal((B, L, H)).astype(np.float32)
    y, got = _run(d, gy, tdt)
    assert relerr(y, oracle.ssm_fwd(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"], d["u"],
                                    d["D"])) < FWD_TOL
    # du comes back in u's dtype: bf16 holds it to 2^-9 relative
    _assert_grads(got, _oracle(d, gy), du_tol=GRAD_TOL if u_dtype == "f32" else 4e-3)


def test_ssm_train_clamps_and_timestamp_edges():
    """dt clamped at both ends, repeated and decreasing timestamps (the
    clamp_min(0) of the differences), nonzero log_dt."""
    B, L, H, N = 2, 203, 24, 16
    d = cell_inputs(B, L, H, N, seed=5, tau=(0.5, 64.0))
    d["log_dt"] = (np.random.default_rng(1).standard_normal(H) * 0.8).astype(np.float32)
    t = d["t"].copy()
    t[0, 10] = t[0, 9]            # zero step
    t[0, 50] = t[0, 49] - 0.3     # backwards step
    t[1, 1] = t[1, 0]             # dt_1 = 0 also sets dt_0
    d["t"] = t
    gy = np.random.default_rng(2).standard_normal((B, L, H)).astype(np.float32)
    for dt_min, dt_max in [(1e-3, 1e3), (0.05, 0.4)]:
        y, got = _run(d, gy, dt_min=dt_min, dt_max=dt_max)
        y_ref = oracle.ssm_fwd(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"], d["u"], d["D"],
                               dt_min=dt_min, dt_max=dt_max)
        assert relerr(y, y_ref) < FWD_TOL
        _assert_grads(got, _oracle(d, gy, dt_min=dt_min, dt_max=dt_max))


def test_ssm_train_forward_matches_inference_and_is_deterministic():
    d = cell_inputs(2, 517, 96, 16, seed=11, tau=(0.5, 64.0))
    gy = np.random.default_rng(3).standard_normal((2, 517, 96)).astype(np.float32)
    y1, g1 = _run(d, gy, torch.bfloat16)
    y2, g2 = _run(d, gy, torch.bfloat16)
    with torch.no_grad():
        y0 = ssm_forward(*(_t(d[k]) for k in ("lam", "log_dt", "t", "Bc", "Cc")),
                         _t(d["u"]).to(torch.bfloat16), _t(d["D"])).cpu().numpy()
    assert np.array_equal(y0, y1) and np.array_equal(y1, y2)
    for k in NAMES:
        assert np.array_equal(g1[k], g2[k]), k


def test_ssm_train_linear_in_upstream_gradient():
    """At a size past what the oracle is run on: the VJP is linear in gy."""
    B, L, H, N = 2, 4096, 256, 16
    d = cell_inputs(B, L, H, N, seed=21, tau=(0.5, 64.0))
    rng = np.random.default_rng(4)
    g1 = rng.standard_normal((B, L, H)).astype(np.float32)
    g2 = rng.standard_normal((B, L, H)).astype(np.float32)
    _, a = _run(d, g1, torch.bfloat16)
    _, b = _run(d, g2, torch.bfloat16)
    _, c = _run(d, g1 + g2, torch.bfloat16)
    for k in NAMES:  # du is bf16 (u's dtype)
        assert relerr(a[k] + b[k], c[k]) < (8e-3 if k == "du" else 1e-4), k


def test_ssm_bwd_rejects_small_buffers():
    B, L, H, N = 1, 16, 8, 4
    L_ = _lib.lib()
    need = int(L_.eacs_ssm_ckpt_size(B, L, H, N))
    assert need == B * 2 * H * N * 8
    z = torch.zeros(1 << 16, device=DEV)
    p = z.data_ptr()
    rc = L_.eacs_ssm_train_fwd(p, p, p, p, p, p, 0, p, p, p, need - 1, B, L, H, N, 1e-3, 1e3, None)
    assert rc == _lib.EACS_ERR_WORKSPACE
    ws = int(L_.eacs_ssm_bwd_workspace_size(B, L, H, N))
    rc = L_.eacs_ssm_bwd(p, p, p, p, p, p, 0, p, p, p, need, p, p, p, p, p, p, p, p, ws - 1,
                         B, L, H, N, 1e-3, 1e3, None)
    assert rc == _lib.EACS_ERR_WORKSPACE
