"""Training through per-frame commits and continuous-time queries on the GPU.

The reference runs EACSLayer._commit_range (modules/eacs.py:386-401) and
readout_from_commits (modules/continuous_query.py:20-54) under autograd; here
CellCommitsFunction (eacs_cell_train_commits_fwd/_bwd) and
QueryReadoutFunction (eacs_query_readout, eacs_query_readout_bwd) take their
place.  Checked against the reference's own autograd outputs (golden
fixtures, tests/golden/qtrain.npz) and against the CPU oracle's composition
of the same two adjoints (oracle/eacs_oracle.c: eacs_oracle_cell_bwd_commits,
eacs_oracle_query_readout_bwd) on larger seeded inputs, with the gates the
GPU decided pinned in the oracle (a residual on the threshold may decide
either way in another summation order).  Tolerances: forward 1e-4 relative
(commits 1e-4), gradients 1e-3 relative (max |x - ref| / max |ref|).
"""
import numpy as np
import pytest
import torch

from golden_io import cases, relerr

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
FWD_TOL = 1e-4
GRAD_TOL = 1e-3
QTRAIN = cases("qtrain")
NAMES = ["du", "dBc", "dCc", "dt", "dlam", "dlog_dt", "dD", "deps", "dtq"]


def _run_gpu(d, mode, gq, gf, gy, ggs, grs):
    """Forward and gradients through the library's two functions; the loss is
    the sum of the outputs weighted by the given upstream gradients."""
    from eacs_b200 import _lib
    from eacs_b200.ops.continuous_query import QueryReadoutFunction, cell_commits_train, segment_index
    eps, eta, var_eps, dt_init, dt_min, dt_max, T = [float(v) for v in d["scalars"]]
    T_ = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV)  # noqa: E731
    leaves = [T_(d[k]).requires_grad_(True) for k in ("u", "Bc", "Cc", "t", "lam", "log_dt", "D")]
    eps_t = torch.tensor(eps, device=DEV, requires_grad=True)
    tq = T_(d["t_query"]).requires_grad_(True)
    u, Bc, Cc, t, lam, log_dt, D = leaves
    n0 = _lib.kernel_launches()
    ys, gs, rs, c = cell_commits_train(lam, log_dt, u, Bc, Cc, t, D, T_(d["mean"]), T_(d["var"]), eps_t,
                                       eta, T, mode, var_eps, dt_init, dt_max)
    B, L = t.shape
    com = (lam, log_dt, D, c["h"], c["t"], c["u"], c["B"], c["C"])
    yq = QueryReadoutFunction.apply(*com, tq, segment_index(t.detach(), tq.detach()), dt_min, dt_max)
    yf = QueryReadoutFunction.apply(*com, t, torch.arange(L, device=DEV).expand(B, L), dt_min, dt_max)
    outs, ups = [ys, yq, yf], [gy, gq, gf]
    if mode != "hard":
        outs += [gs, rs]
        ups += [ggs, grs]
    grads = torch.autograd.grad(outs, leaves + [eps_t, tq], [T_(g) for g in ups], allow_unused=True)
    torch.cuda.synchronize()
    assert _lib.kernel_launches() > n0
    assert _lib.device_status() == 0
    fwd = [x.detach().cpu().numpy() for x in (ys, gs, rs, c["h"], c["t"], c["u"], c["B"], c["C"], yq, yf)]
    grads = [np.zeros(1, np.float32) if g is None else g.detach().cpu().numpy() for g in grads]
    return fwd, dict(zip(NAMES, grads))


@pytest.mark.parametrize("name", sorted(QTRAIN))
def test_commit_training_golden(name):
    """Against the reference's autograd on its own fixtures."""
    d = QTRAIN[name]
    mode = "ste" if int(d["gate_mode"][0]) == 0 else "soft"
    fwd, grads = _run_gpu(d, mode, d["gq"], d["gf"], d["gy"], d["ggs"], d["grs"])
    y, g, r, ch, ct, cu, cB, cC, yq, yf = fwd
    assert np.max(np.abs(g - d["gate"])) <= (0 if mode == "ste" else 1e-5)
    for got, key in zip((y, r, ch, ct, cu, cB, cC, yq, yf),
                        ("y", "resid", "ch", "ct", "cu", "cB", "cC", "yq", "yf")):
        assert relerr(got, d[key]) < FWD_TOL, key
    for k in NAMES:
        assert relerr(grads[k], d[k]) < GRAD_TOL, (k, relerr(grads[k], d[k]))


def _inputs(B, L, H, N, Q, seed, tau=(0.5, 4.0), dup=True):
    rng = np.random.default_rng(seed)
    lam = (-1.0 / np.exp(rng.uniform(np.log(tau[0]), np.log(tau[1]), (H, N)))
           + 1j * np.pi * rng.uniform(0, 2, (H, N))).astype(np.complex64)
    u = rng.standard_normal((B, L, H)).astype(np.float32)
    if dup:  # runs of repeated frames, so the gate skips
        for l in range(1, L):
            if (l // 3) % 2 == 1:
                u[:, l] = u[:, l - 1] + 0.01 * rng.standard_normal((B, H)).astype(np.float32)
    cs = 1 / np.sqrt(2 * N)
    Bc = ((rng.standard_normal((B, L, N)) + 1j * rng.standard_normal((B, L, N))) * cs).astype(np.complex64)
    Cc = ((rng.standard_normal((B, L, N)) + 1j * rng.standard_normal((B, L, N))) * cs).astype(np.complex64)
    t = np.cumsum(np.clip(rng.exponential(0.25, (B, L)), 1 / 30, 2.0), 1).astype(np.float32)
    tq = (t[:, :1] - 0.3 + (t[:, -1:] - t[:, :1] + 0.8) * rng.random((B, Q))).astype(np.float32)
    d = dict(lam=lam, log_dt=(0.2 * rng.standard_normal(H)).astype(np.float32), u=u, Bc=Bc, Cc=Cc, t=t,
             D=rng.standard_normal(H).astype(np.float32),
             mean=(0.1 * rng.standard_normal(H)).astype(np.float32),
             var=rng.uniform(0.5, 1.5, H).astype(np.float32), t_query=tq)
    up = dict(gy=rng.standard_normal((B, L, H)), ggs=rng.standard_normal((B, L)),
              grs=rng.standard_normal((B, L)), gq=rng.standard_normal((B, Q, H)),
              gf=rng.standard_normal((B, L, H)))
    return d, {k: v.astype(np.float32) for k, v in up.items()}


def _oracle(d, gates, mode, up):
    from oracle import oracle
    eps, eta, var_eps, dt_init, dt_min, dt_max, T = [float(v) for v in d["scalars"]]
    gm = {"ste": 0, "soft": 1, "hard": 2}[mode]
    B, L = d["t"].shape
    fwd, _ = oracle.cell_train_commits(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                                       d["mean"], d["var"], eps, eta, var_eps, dt_init, dt_max, T, gm,
                                       gs=gates if gm != 1 else None)
    y, g, r, ch, ct, cu, cB, cC = fwd
    com = (d["lam"], d["log_dt"], d["D"], ch, ct, cu, cB, cC, d["t"])
    gq, gtq, dlq, dlogq, dDq = oracle.query_readout_bwd(*com, d["t_query"], up["gq"], dt_min=dt_min,
                                                        dt_max=dt_max)
    idx = np.broadcast_to(np.arange(L, dtype=np.int32), (B, L))
    gf, gtf, dlf, dlogf, dDf = oracle.query_readout_bwd(*com, d["t"], up["gf"], idx=idx, dt_min=dt_min,
                                                        dt_max=dt_max)
    gc = {k: gq[k] + gf[k] for k in gq}
    live = mode != "hard"
    _, (du, dBc, dCc, dt, dlam, dlog, dD, deps) = oracle.cell_train_commits(
        d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"], d["mean"], d["var"], eps, eta,
        var_eps, dt_init, dt_max, T, gm, gs=g, gy=up["gy"], ggs=up["ggs"] if live else None,
        grs=up["grs"] if live else None, gc=gc)
    yq = oracle.query_readout(*com, d["t_query"], dt_min=dt_min, dt_max=dt_max)
    return (y, g, r, ch, ct, cu, cB, cC, yq), dict(
        du=du, dBc=dBc, dCc=dCc, dt=dt + gtf, dlam=dlam + dlq + dlf, dlog_dt=dlog + dlogq + dlogf,
        dD=dD + dDq + dDf, deps=deps, dtq=gtq)


@pytest.mark.parametrize("B,L,H,N,Q,mode,seed", [
    (2, 200, 64, 16, 150, "ste", 1),
    (2, 160, 48, 8, 90, "soft", 2),
    (1, 96, 768, 16, 64, "ste", 3),      # config 1's width, one row (16-CTA cluster)
    (6, 64, 768, 16, 40, "ste", 4),      # config 1's width, 8-CTA clusters
    (2, 120, 40, 32, 70, "hard", 5),     # eval-mode gate: no gradient through it
    (2, 80, 24, 5, 200, "ste", 6),       # more queries than frames, ragged N
])
def test_commit_training_vs_oracle(B, L, H, N, Q, mode, seed):
    """Threshold at the median residual of an all-commit run, so that both
    branches of the gate run."""
    from oracle import oracle
    oracle.set_threads(0)
    d, up = _inputs(B, L, H, N, Q, seed)
    _, _, r_all = oracle.cell_fwd(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                                  d["mean"], d["var"], 0.0, 1e-6)
    eps = float(np.median(r_all))
    d["scalars"] = np.array([eps, 1e-6, 1e-5, 1.0, 1e-3, 1e3, 0.3])
    fwd, grads = _run_gpu(d, mode, up["gq"], up["gf"], up["gy"], up["ggs"], up["grs"])
    y, g, r, ch, ct, cu, cB, cC, yq, yf = fwd
    if mode != "soft":
        assert 0.05 < g.mean() < 0.98, g.mean()
    ofwd, ograds = _oracle(d, g, mode, up)
    oy, og, orr, och, oct_, ocu, ocB, ocC, oyq = ofwd
    if mode == "soft":
        assert np.max(np.abs(g - og)) < 1e-5
    for got, ref, key in zip((y, r, ch, ct, cu, cB, cC, yq), (oy, orr, och, oct_, ocu, ocB, ocC, oyq),
                             ("y", "resid", "h", "t", "u", "B", "C", "yq")):
        assert relerr(got, ref) < FWD_TOL, (key, relerr(got, ref))
    for k in NAMES:
        assert relerr(grads[k], ograds[k]) < GRAD_TOL, (k, relerr(grads[k], ograds[k]))


def test_unsorted_queries_and_workspace_reuse():
    """Queries in random order (the function sorts them per row and scatters
    the query times' gradients back) give the gradients of the sorted order."""
    from eacs_b200.ops.continuous_query import QueryReadoutFunction, cell_commits_train, segment_index
    d, up = _inputs(2, 64, 32, 16, 50, 9)
    T_ = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV)  # noqa: E731
    perm = np.stack([np.random.default_rng(10 + b).permutation(50) for b in range(2)])
    res = []
    for tq_np, gq_np in ((d["t_query"], up["gq"]),
                         (np.take_along_axis(d["t_query"], perm, 1),
                          np.take_along_axis(up["gq"], perm[..., None], 1))):
        lam = T_(d["lam"]).requires_grad_(True)
        u = T_(d["u"]).requires_grad_(True)
        tq = T_(tq_np).requires_grad_(True)
        ys, gs, rs, c = cell_commits_train(lam, T_(d["log_dt"]), u, T_(d["Bc"]), T_(d["Cc"]), T_(d["t"]),
                                           T_(d["D"]), T_(d["mean"]), T_(d["var"]), 0.5, 1e-6, 0.3, "ste")
        com = (lam, T_(d["log_dt"]), T_(d["D"]), c["h"], c["t"], c["u"], c["B"], c["C"])
        yq = QueryReadoutFunction.apply(*com, tq, segment_index(T_(d["t"]), tq.detach()), 1e-3, 1e3)
        gl, gu, gt = torch.autograd.grad(yq, [lam, u, tq], T_(gq_np))
        res.append((gl.cpu().numpy(), gu.cpu().numpy(), gt.cpu().numpy()))
    (gl0, gu0, gt0), (gl1, gu1, gt1) = res
    assert relerr(gl1, gl0) < 1e-5 and relerr(gu1, gu0) < 1e-5
    assert relerr(gt1, np.take_along_axis(gt0, perm, 1)) < 1e-5


def test_edge_shapes():
    """One frame (L = 1), a row's queries all before its first frame, and no
    queries at all (Q = 0: the commits' adjoints are zero)."""
    from eacs_b200.ops.continuous_query import QueryReadoutFunction, cell_commits_train
    for L, Q in ((1, 3), (5, 0), (7, 4)):
        d, up = _inputs(2, L, 16, 8, max(Q, 1), 40 + L)
        d["scalars"] = np.array([0.5, 1e-6, 1e-5, 1.0, 1e-3, 1e3, 0.3])
        if Q:
            d["t_query"] = d["t_query"][:, :Q] if L > 1 else np.stack([d["t"][:, 0] - 0.5, d["t"][:, 0],
                                                                       d["t"][:, 0] + 0.3], 1).astype(np.float32)
            if L == 7:
                d["t_query"] = (d["t"][:, :1] - 1.0 - np.arange(Q)[None, :] * 0.1).astype(np.float32)
            up["gq"] = up["gq"][:, :Q]
        else:
            d["t_query"] = np.zeros((2, 0), np.float32)
            up["gq"] = np.zeros((2, 0, 16), np.float32)
        fwd, grads = _run_gpu(d, "ste", up["gq"], up["gf"], up["gy"], up["ggs"], up["grs"])
        _, ograds = _oracle(d, fwd[1], "ste", up)
        for k in NAMES:
            if k == "dtq" and Q == 0:
                continue
            assert relerr(grads[k], ograds[k]) < GRAD_TOL, (L, Q, k, relerr(grads[k], ograds[k]))
