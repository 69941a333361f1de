"""Per-frame commits (eacs_cell_commits) and continuous-time query readouts
(eacs_query_index / eacs_query_readout) against the reference's own outputs
(tests/golden/query.npz: run_with_commits + readout_from_commits) and the
oracle.

Tolerances: gates bit-exact on steps whose residual is more than 1e-5 from
the threshold (the golden and calibrated cases have none closer); commits,
outputs and readouts 1e-4 relative (max |x - ref| / max |ref|).
"""
import numpy as np
import pytest
import torch

from golden_io import cases, relerr
from inputs import cell_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-4
DEV = "cuda:0"

if torch.cuda.is_available():
    from eacs_b200 import _lib
    from eacs_b200.ops.continuous_query import cell_commits, query_readout, segment_index

KEYS = ("h", "t", "u", "B", "C")
OKEYS = ("ch", "ct", "cu", "cB", "cC")


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _commits(d, eps, u_dtype=torch.float32, robust=None, dt_max=1e3):
    ys, gs, rs, cm = cell_commits(_t(d["lam"]), _t(d["log_dt"]), _t(d["u"]).to(u_dtype), _t(d["Bc"]),
                                  _t(d["Cc"]), _t(d["t"]), _t(d["D"]), _t(d["mean"]), _t(d["var"]),
                                  eps, 1e-6, dt_max=dt_max, robust=robust)
    return ys, gs, rs, cm


@pytest.mark.parametrize("name", sorted(cases("query")))
def test_commits_and_queries_golden(name):
    d = cases("query")[name]
    eps, eta, var_eps, dt_init, dt_min, dt_max = [float(v) for v in d["scalars"]]
    ys, gs, rs, cm = _commits(d, eps, dt_max=dt_max)
    assert np.array_equal(gs.cpu().numpy(), d["gate"])
    assert relerr(rs.cpu().numpy(), d["resid"]) < TOL
    assert relerr(ys.cpu().numpy(), d["y"]) < TOL
    for k, ok in zip(KEYS, OKEYS):
        assert relerr(cm[k].cpu().numpy(), d[ok]) < TOL, k
    cm["frame_t"] = _t(d["t"])
    yq = query_readout(_t(d["lam"]), _t(d["log_dt"]), _t(d["D"]), cm, _t(d["t_query"]),
                       dt_max=dt_max)
    assert relerr(yq.cpu().numpy(), d["yq"]) < TOL
    B, L = d["t"].shape
    idx = torch.arange(L, device=DEV).expand(B, L)
    yf = query_readout(_t(d["lam"]), _t(d["log_dt"]), _t(d["D"]), cm, _t(d["t"]), idx, dt_max=dt_max)
    assert relerr(yf.cpu().numpy(), d["yf"]) < TOL
    assert _lib.device_status() == 0


@pytest.mark.parametrize("B,L,H,N,rate,robust", [
    (2, 300, 96, 16, 0.5, None),
    (3, 77, 40, 32, 0.3, None),
    (2, 64, 24, 5, 0.7, (3, 2.0, 0.3)),
    (1, 1, 8, 4, None, None),
    (2, 50, 130, 64, 0.6, None),
])
def test_commits_vs_oracle(B, L, H, N, rate, robust):
    from test_gpu_kernels import _calibrated_eps
    d = cell_inputs(B, L, H, N, seed=B * L + H + N)
    eps = 0.12 if rate is None else _calibrated_eps(d, rate, robust)
    ys, gs, rs, cm = _commits(d, eps, robust=robust)
    ref = oracle.cell_commits(**d, eps=eps, eta=1e-6, robust=robust)
    assert np.array_equal(gs.cpu().numpy(), ref[1])
    assert relerr(rs.cpu().numpy(), ref[2]) < TOL
    assert relerr(ys.cpu().numpy(), ref[0]) < TOL
    for k, r in zip(KEYS, ref[3:]):
        assert relerr(cm[k].cpu().numpy(), r) < TOL, k
    # queries: inside segments, on frames, before the first and past the last frame
    rng = np.random.default_rng(L)
    t = d["t"]
    Q = 3 * L + 5
    tq = t[:, :1] - 0.5 + (t[:, -1:] - t[:, :1] + 1.0) * rng.random((B, Q))
    tq[:, :L] = t
    tq = np.sort(tq, 1).astype(np.float32)
    cm["frame_t"] = _t(t)
    idx = segment_index(_t(t), _t(tq)).cpu().numpy()
    ref_idx = np.stack([np.clip(np.searchsorted(t[b], tq[b], side="right") - 1, 0, L - 1)
                        for b in range(B)])
    assert np.array_equal(idx, ref_idx)
    yq = query_readout(_t(d["lam"]), _t(d["log_dt"]), _t(d["D"]), cm, _t(tq))
    yq_ref = oracle.query_readout(d["lam"], d["log_dt"], d["D"], *ref[3:], t, tq)
    assert relerr(yq.cpu().numpy(), yq_ref) < TOL
    assert _lib.device_status() == 0


def test_query_index_clamped_and_half_inputs():
    d = cell_inputs(2, 40, 32, 16, seed=3)
    d["u"] = _t(d["u"]).to(torch.bfloat16).float().cpu().numpy()
    ys, gs, rs, cm = _commits(d, 0.12, torch.bfloat16)
    ref = oracle.cell_commits(**d, eps=0.12, eta=1e-6)
    assert relerr(ys.cpu().numpy(), ref[0]) < TOL
    cm["frame_t"] = _t(d["t"])
    tq = _t(d["t"][:, :7] + 0.05)
    bad = torch.tensor([[-5, 0, 3, 39, 40, 1000, 7]] * 2, device=DEV)
    y_bad = query_readout(_t(d["lam"]), _t(d["log_dt"]), _t(d["D"]), cm, tq, bad)
    y_ok = query_readout(_t(d["lam"]), _t(d["log_dt"]), _t(d["D"]), cm, tq, bad.clamp(0, 39))
    assert torch.equal(y_bad, y_ok)
