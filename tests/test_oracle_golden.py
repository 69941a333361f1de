"""The CPU oracle against golden vectors produced by the reference itself."""
import numpy as np
import pytest

from golden_io import cases, cell_args, decisive, relerr
from oracle import oracle

SCAN = cases("scan")
SSM = cases("ssm")
CELL = cases("cell")
TRAIN = cases("train")


@pytest.mark.parametrize("name", sorted(SCAN))
def test_scan_fwd_bwd(name):
    d = SCAN[name]
    h = oracle.scan_fwd(d["a"], d["b"])
    assert relerr(h, d["h"]) < 1e-6
    assert relerr(d["h_assoc"], d["h"]) < 1e-5  # reference's own two scans agree
    ga, gb = oracle.scan_bwd(d["a"], d["h"], d["gh"])
    assert relerr(ga, d["ga"]) < 1e-6
    assert relerr(gb, d["gb"]) < 1e-6


@pytest.mark.parametrize("name", sorted(SSM))
def test_ssm_fwd(name):
    d = SSM[name]
    y = oracle.ssm_fwd(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"], d["u"], d["D"])
    assert relerr(y, d["y"]) < 1e-5


@pytest.mark.parametrize("name", sorted(SSM))
def test_ssm_bwd(name):
    d = SSM[name]
    got = oracle.ssm_bwd(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"], d["u"], d["D"], d["gy"])
    # gradient tolerance 1e-3 (the L=1 case has |dlam| ~ 1e-7, where the
    # reference's own float32 autograd differs from the double oracle by 2.5e-4)
    for k, v in zip(["du", "dBc", "dCc", "dt", "dlam", "dlog_dt", "dD"], got):
        assert relerr(v, d[k]) < 1e-3, (k, relerr(v, d[k]))


@pytest.mark.parametrize("name", sorted(CELL))
def test_cell_fwd(name):
    d = CELL[name]
    a = cell_args(d)
    y, g, r = oracle.cell_fwd(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                              d["mean"], d["var"], **a)
    assert np.array_equal(g, d["gate"]), "gate masks differ"
    assert decisive(d["resid"], a["eps"], a["robust"]).all()
    assert relerr(r, d["resid"]) < 1e-5
    assert relerr(y, d["y"]) < 1e-5


@pytest.mark.parametrize("name", sorted(TRAIN))
def test_train_fwd(name):
    d = TRAIN[name]
    eps, eta, var_eps, dt_init, dt_min, dt_max, T = [float(v) for v in d["scalars"]]
    mode = int(d["gate_mode"][0])
    y, g, r = oracle.cell_fwd(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                              d["mean"], d["var"], eps, eta, var_eps, dt_init, dt_min, dt_max,
                              gate_mode=mode, T=T, train_exp=True)
    tol_g = 0 if mode == 0 else 1e-5
    assert np.max(np.abs(g - d["gate"])) <= tol_g
    assert relerr(r, d["resid"]) < 1e-5
    assert relerr(y, d["y"]) < 1e-5
    assert np.array_equal(d["innov"], d["resid"])


@pytest.mark.parametrize("name", sorted(TRAIN))
def test_train_bwd(name):
    d = TRAIN[name]
    eps, eta, var_eps, dt_init, dt_min, dt_max, T = [float(v) for v in d["scalars"]]
    mode = int(d["gate_mode"][0])
    got = oracle.cell_bwd(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                          d["mean"], d["var"], eps, eta, var_eps, dt_init, dt_max, T, mode,
                          d["gate"], d["gy"], d["ggs"], d["grs"], d["gns"])
    names = ["du", "dBc", "dCc", "dt", "dlam", "dlog_dt", "dD", "deps"]
    for k, v in zip(names, got):
        assert relerr(v, d[k]) < 1e-4, (k, relerr(v, d[k]))


QUERY = cases("query")


@pytest.mark.parametrize("name", sorted(QUERY))
def test_commits_and_query_readout(name):
    """run_with_commits + readout_from_commits (eacs.py:386-439,
    continuous_query.py:12-61): gates bit-exact (eps calibrated away from the
    residuals), commits and readouts to 1e-5."""
    d = QUERY[name]
    eps, eta, var_eps, dt_init, dt_min, dt_max = [float(v) for v in d["scalars"]]
    y, g, r, ch, ct, cu, cB, cC = oracle.cell_commits(
        d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"], d["mean"], d["var"],
        eps, eta, var_eps, dt_init, dt_min, dt_max)
    assert np.array_equal(g, d["gate"])
    assert relerr(r, d["resid"]) < 1e-5
    assert relerr(y, d["y"]) < 1e-5
    for got, key in zip((ch, ct, cu, cB, cC), ("ch", "ct", "cu", "cB", "cC")):
        assert relerr(got, d[key]) < 1e-5, key
    yq = oracle.query_readout(d["lam"], d["log_dt"], d["D"], d["ch"], d["ct"], d["cu"], d["cB"],
                              d["cC"], d["t"], d["t_query"], dt_min=dt_min, dt_max=dt_max)
    assert relerr(yq, d["yq"]) < 1e-5
    B, L = d["t"].shape
    idx = np.broadcast_to(np.arange(L, dtype=np.int32), (B, L))
    yf = oracle.query_readout(d["lam"], d["log_dt"], d["D"], d["ch"], d["ct"], d["cu"], d["cB"],
                              d["cC"], d["t"], d["t"], idx=idx, dt_min=dt_min, dt_max=dt_max)
    assert relerr(yf, d["yf"]) < 1e-5


STREAM = cases("stream")


def stream_args(d):
    eps, eta, var_eps, dt_init, dt_min, dt_max, m, T, soft, mid = [float(v) for v in d["scalars"]]
    return dict(eps=eps, eta=eta, var_eps=var_eps, dt_init=dt_init, dt_min=dt_min, dt_max=dt_max,
                cpi_mod=m, gate_mode=int(soft), T=T), int(mid)


def zero_state(d):
    B, K, H = d["u"].shape
    N = d["lam"].shape[1]
    return (np.zeros((B, H, N), np.complex64), np.zeros(B, np.float32), np.zeros((B, H), np.float32),
            np.zeros((B, N), np.complex64), np.zeros((B, N), np.complex64), np.zeros(B, np.uint8))


@pytest.mark.parametrize("name", sorted(STREAM))
def test_stream_chunk(name):
    """temporal_step (streaming.py:45-85): the whole sequence as one chunk and
    as two chunks through the intermediate state."""
    d = STREAM[name]
    kw, mid = stream_args(d)
    cpi = d.get("cpi")
    ins = (d["lam"], d["log_dt"], d["D"], d["mean"], d["var"])
    y, g, r, n, st = oracle.stream_chunk(*ins, d["u"], d["Bc"], d["Cc"], d["t"], d["valid"], cpi,
                                         zero_state(d), **kw)
    assert relerr(y, d["y"]) < 1e-5
    assert relerr(g, d["gate"]) < 1e-5
    assert relerr(r, d["resid"]) < 1e-5
    assert relerr(n, d["innov"]) < 1e-5
    for got, key in zip(st, ("h", "st_t", "st_u", "st_B", "st_C", "st_init")):
        assert relerr(got, d[key]) < 1e-5, key
    # two chunks: [0, mid) then [mid, K) from the state after step mid-1
    sl = lambda a, lo, hi: None if a is None else a[:, lo:hi]
    _, _, _, _, st1 = oracle.stream_chunk(*ins, *(sl(d[k], 0, mid) for k in ("u", "Bc", "Cc", "t", "valid")),
                                          sl(cpi, 0, mid), zero_state(d), **kw)
    for got, key in zip(st1, ("mid_h", "mid_t", "mid_u", "mid_B", "mid_C", "mid_init")):
        assert relerr(got, d[key]) < 1e-5, key
    K = d["u"].shape[1]
    y2, _, _, _, st2 = oracle.stream_chunk(*ins, *(sl(d[k], mid, K) for k in ("u", "Bc", "Cc", "t", "valid")),
                                           sl(cpi, mid, K), st1, **kw)
    assert relerr(y2, d["y"][:, mid:]) < 1e-5
    assert relerr(st2[0], d["h"]) < 1e-5


QTRAIN = cases("qtrain")


def qtrain_grads(d, fwd_from_oracle=True):
    """The oracle's composition for a commit-training fixture: the readout
    adjoints of the query and frame-time readouts feed the cell backward as
    commit adjoints; the parameter and time gradients of the pieces add.
    Returns (forward, grads) in the fixture's key order."""
    eps, eta, var_eps, dt_init, dt_min, dt_max, T = [float(v) for v in d["scalars"]]
    mode = int(d["gate_mode"][0])
    B, L = d["t"].shape
    fwd, _ = oracle.cell_train_commits(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"],
                                       d["D"], d["mean"], d["var"], eps, eta, var_eps, dt_init,
                                       dt_max, T, mode)
    y, g, r, ch, ct, cu, cB, cC = fwd if fwd_from_oracle else (
        d["y"], d["gate"], d["resid"], d["ch"], d["ct"], d["cu"], d["cB"], d["cC"])
    com = (d["lam"], d["log_dt"], d["D"], ch, ct, cu, cB, cC, d["t"])
    gq, gtq, dlq, dlogq, dDq = oracle.query_readout_bwd(*com, d["t_query"], d["gq"],
                                                        dt_min=dt_min, dt_max=dt_max)
    idx = np.broadcast_to(np.arange(L, dtype=np.int32), (B, L))
    gf, gtf, dlf, dlogf, dDf = oracle.query_readout_bwd(*com, d["t"], d["gf"], idx=idx,
                                                        dt_min=dt_min, dt_max=dt_max)
    gc = {k: gq[k] + gf[k] for k in gq}
    _, (du, dBc, dCc, dt, dlam, dlog, dD, deps) = oracle.cell_train_commits(
        d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"], d["mean"], d["var"],
        eps, eta, var_eps, dt_init, dt_max, T, mode, gs=g, gy=d["gy"], ggs=d["ggs"], grs=d["grs"],
        gc=gc)
    grads = dict(du=du, dBc=dBc, dCc=dCc, dt=dt + gtf, dlam=dlam + dlq + dlf,
                 dlog_dt=dlog + dlogq + dlogf, dD=dD + dDq + dDf, deps=deps, dtq=gtq)
    return fwd, grads


@pytest.mark.parametrize("name", sorted(QTRAIN))
def test_commit_training(name):
    """_commit_range + readout_from_commits under autograd (eacs.py:386-401,
    continuous_query.py:20-54): the training forward (gates, commits) and every
    gradient, including those of the query times, to 1e-4."""
    d = QTRAIN[name]
    mode = int(d["gate_mode"][0])
    (y, g, r, ch, ct, cu, cB, cC), grads = qtrain_grads(d)
    assert np.max(np.abs(g - d["gate"])) <= (0 if mode == 0 else 1e-5)
    assert relerr(r, d["resid"]) < 1e-5
    assert relerr(y, d["y"]) < 1e-5
    for got, key in zip((ch, ct, cu, cB, cC), ("ch", "ct", "cu", "cB", "cC")):
        assert relerr(got, d[key]) < 1e-5, key
    for k, v in grads.items():
        assert relerr(v, d[k]) < 1e-4, (k, relerr(v, d[k]))


SGRAD = cases("sgrad")


def sgrad_oracle(d, pin=None):
    """The oracle's K-step streaming scan for a temporal_step-gradient fixture:
    the steps forward one at a time (eacs_oracle_stream_chunk, K = 1), then
    their backwards in reverse (eacs_oracle_stream_step_bwd), the state's
    adjoint passed from step to step.  pin: gate outputs (B,K) to pin in the
    hard modes.  Returns (outputs (y, gate, resid, innov), final state, grads)."""
    eps, eta, var_eps, dt_init, dt_min, dt_max, m, T = [float(v) for v in d["scalars"]]
    mode = int(d["gate_mode"][0])
    ins = (d["lam"], d["log_dt"], d["D"], d["mean"], d["var"])
    cpi = d.get("cpi")
    B, K, H = d["u"].shape
    kw = dict(var_eps=var_eps, dt_init=dt_init, dt_min=dt_min, dt_max=dt_max)
    states = [(d["h0"], d["t0"], d["u0"], d["B0"], d["C0"], d["init0"])]
    outs = []
    for k in range(K):
        sl = slice(k, k + 1)
        y, g, r, n, st = oracle.stream_chunk(*ins, d["u"][:, sl], d["Bc"][:, sl], d["Cc"][:, sl], d["t"][:, sl],
                                             d["valid"][:, sl], None if cpi is None else cpi[:, sl], states[-1],
                                             eps, eta, cpi_mod=m, gate_mode=1 if mode == 1 else 0, T=T, **kw)
        outs.append((y[:, 0], g[:, 0], r[:, 0], n[:, 0]))
        states.append(st)
    adj = dict(h=d["gh"], t=d["gt"], u=d["gu"], B=d["gB"], C=d["gC"])
    per = {k: [None] * K for k in ("du", "dBc", "dCc", "dt", "dcpi")}
    tot = dict(dlam=0, dlog_dt=0, dD=0, deps=0)
    for k in reversed(range(K)):
        up = dict(y=d["gy"][:, k], gate=d["gg"][:, k], resid=d["gr"][:, k], innov=d["gn"][:, k], **adj)
        o = oracle.stream_step_bwd(*ins, d["u"][:, k], d["Bc"][:, k], d["Cc"][:, k], d["t"][:, k],
                                   d["valid"][:, k], None if cpi is None else cpi[:, k], states[k], up, eps, eta,
                                   cpi_mod=m, gate_mode=mode, T=T, gs=None if pin is None else pin[:, k], **kw)
        for key in per:
            per[key][k] = o[key]
        for key in tot:
            tot[key] = tot[key] + o[key]
        adj = dict(h=o["dh"], t=o["dt_in"], u=o["du_in"], B=o["dB_in"], C=o["dC_in"])
    grads = {key: np.stack(v, 1) for key, v in per.items()}
    grads.update(dh0=adj["h"], dt0=adj["t"], du0=adj["u"], dB0=adj["B"], dC0=adj["C"], **tot)
    outputs = tuple(np.stack([o[i] for o in outs], 1) for i in range(4))
    return outputs, states[-1], grads


@pytest.mark.parametrize("name", sorted(SGRAD))
def test_stream_step_gradients(name):
    """temporal_step under autograd over K steps (streaming.py:45-85): the
    outputs, the final state and every gradient (per-step inputs, initial
    state, parameters, threshold, CPI) to 1e-4."""
    d = SGRAD[name]
    (y, g, r, n), st, grads = sgrad_oracle(d)
    for got, key in zip((y, g, r, n), ("y", "gate", "resid", "innov")):
        assert relerr(got, d[key]) < 1e-5, key
    for got, key in zip(st[:5], ("fh", "ft", "fu", "fB", "fC")):
        assert relerr(got, d[key]) < 1e-5, key
    names = ["du", "dBc", "dCc", "dt"] + (["dcpi"] if "cpi" in d else []) + \
        ["dh0", "dt0", "du0", "dB0", "dC0", "dlam", "dlog_dt", "dD", "deps"]
    for k in names:
        assert relerr(grads[k], d[k]) < 1e-4, (k, relerr(grads[k], d[k]))
