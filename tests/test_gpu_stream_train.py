"""Streaming steps under autograd on the GPU (temporal_step in training).

The reference differentiates temporal_step (modules/streaming.py:45-85) step
by step through its tensor graph; here each branch's step is one
StreamStepFunction (forward: eacs_stream_chunk with K = 1; backward:
eacs_stream_step_bwd) and autograd chains the steps through the state.
Checked against the reference's own autograd outputs over multi-step scans
(golden fixtures, tests/golden/sgrad.npz: STE, soft, CPI-modulated and eval
gates, masked frames, rows starting uninitialised), against the CPU oracle's
composition of eacs_oracle_stream_step_bwd on larger seeded inputs, and
through the unmodified reference's temporal_step with and without
install(streaming=True).  Tolerances: forward 1e-4 relative, gradients 1e-3
relative (max |x - ref| / max |ref|).
"""
import copy

import numpy as np
import pytest
import torch

from golden_io import cases, relerr
from ref_pkg import import_reference, reference_only, reference_root, restore, snapshot
from test_oracle_golden import sgrad_oracle

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
FWD_TOL = 1e-4
GRAD_TOL = 1e-3
SGRAD = cases("sgrad")
MODES = {0: "ste", 1: "soft", 2: "hard"}


def _scan_gpu(d):
    """The fixture's K steps through StreamStepFunction; returns (outputs,
    final state, grads) as numpy, keyed like the fixture."""
    from eacs_b200 import _lib
    from eacs_b200.ops.streaming import StreamStepFunction
    eps, eta, var_eps, dt_init, dt_min, dt_max, m, T = [float(v) for v in d["scalars"]]
    mode = MODES[int(d["gate_mode"][0])]
    T_ = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(DEV)  # noqa: E731
    has_cpi = "cpi" in d
    names = ["u", "Bc", "Cc", "t"] + (["cpi"] if has_cpi else []) + ["h0", "t0", "u0", "B0", "C0", "lam",
                                                                     "log_dt", "D"]
    lv = {k: T_(d[k]).requires_grad_(True) for k in names}
    eps_t = torch.tensor(eps, device=DEV, requires_grad=True)
    valid = T_(d["valid"]).bool()
    init = T_(d["init0"]).bool()
    mean, var = T_(d["mean"]), T_(d["var"])
    hp = (eta, var_eps, dt_init, dt_min, dt_max, m if has_cpi else 0.0, mode, T)
    st = [lv["h0"], lv["t0"], lv["u0"], lv["B0"], lv["C0"]]
    K = d["u"].shape[1]
    outs = {"y": [], "gate": [], "resid": [], "innov": []}
    n0 = _lib.kernel_launches()
    for k in range(K):
        y, g, r, n, h1, t1, u1, B1, C1, i1 = StreamStepFunction.apply(
            lv["u"][:, k], lv["Bc"][:, k], lv["Cc"][:, k], lv["t"][:, k], lv["cpi"][:, k] if has_cpi else None,
            *st, lv["lam"], lv["log_dt"], lv["D"], eps_t, init, valid[:, k], mean, var, hp)
        for key, v in zip(("y", "gate", "resid", "innov"), (y, g, r, n)):
            outs[key].append(v)
        st, init = [h1, t1, u1, B1, C1], i1
    outs = {k: torch.stack(v, 1) for k, v in outs.items()}
    terms = [(outs["y"], d["gy"]), (outs["gate"], d["gg"]), (outs["resid"], d["gr"]), (outs["innov"], d["gn"])]
    terms += list(zip(st, (d["gh"], d["gt"], d["gu"], d["gB"], d["gC"])))
    wrt = [lv[k] for k in names] + [eps_t]
    grads = torch.autograd.grad([o for o, _ in terms], wrt, [T_(g) for _, g in terms], allow_unused=True)
    torch.cuda.synchronize()
    assert _lib.kernel_launches() > n0
    assert _lib.device_status() == 0
    gnames = ["du", "dBc", "dCc", "dt"] + (["dcpi"] if has_cpi else []) + \
        ["dh0", "dt0", "du0", "dB0", "dC0", "dlam", "dlog_dt", "dD", "deps"]
    npy = lambda x: x.detach().cpu().numpy()  # noqa: E731
    return ({k: npy(v) for k, v in outs.items()}, [npy(x) for x in st],
            {k: (np.zeros(1, np.float32) if g is None else npy(g)) for k, g in zip(gnames, grads)})


@pytest.mark.parametrize("name", sorted(SGRAD))
def test_stream_step_gradients_golden(name):
    """Against the reference's autograd over its own multi-step fixtures."""
    d = SGRAD[name]
    outs, st, grads = _scan_gpu(d)
    for key in ("y", "gate", "resid", "innov"):
        assert relerr(outs[key], d[key]) < FWD_TOL, key
    for got, key in zip(st, ("fh", "ft", "fu", "fB", "fC")):
        assert relerr(got, d[key]) < FWD_TOL, key
    for k, v in grads.items():
        assert relerr(v, d[k]) < GRAD_TOL, (k, relerr(v, d[k]))


def _random_case(B, K, H, N, mode, seed, cpi_mod=0.0):
    rng = np.random.default_rng(seed)
    s = 1 / np.sqrt(2 * N)
    cplx = lambda *sh: ((rng.standard_normal(sh) + 1j * rng.standard_normal(sh)) * s).astype(np.complex64)  # noqa: E731
    u = rng.standard_normal((B, K, H)).astype(np.float32)
    for k in range(2, K, 3):  # repeated frames: skipped steps
        u[:, k] = u[:, k - 1] + 0.02 * rng.standard_normal((B, H)).astype(np.float32)
    lam = (-1.0 / np.exp(rng.uniform(np.log(0.5), np.log(4.0), (H, N)))
           + 1j * np.pi * rng.uniform(0, 2, (H, N))).astype(np.complex64)
    valid = np.ones((B, K), np.uint8)
    valid[1, :2] = 0
    valid[0, K // 2] = 0
    d = dict(lam=lam, log_dt=(0.2 * rng.standard_normal(H)).astype(np.float32),
             D=rng.standard_normal(H).astype(np.float32), mean=(0.1 * rng.standard_normal(H)).astype(np.float32),
             var=rng.uniform(0.5, 1.5, H).astype(np.float32), u=u, Bc=cplx(B, K, N), Cc=cplx(B, K, N),
             t=(1.0 + np.cumsum(np.clip(rng.exponential(0.25, (B, K)), 1 / 30, 2.0), 1)).astype(np.float32),
             valid=valid, h0=(cplx(B, H, N) * 0.5).astype(np.complex64),
             t0=(0.5 * rng.random(B)).astype(np.float32), u0=rng.standard_normal((B, H)).astype(np.float32),
             B0=cplx(B, N), C0=cplx(B, N), init0=(np.arange(B) % 2 == 0).astype(np.uint8),
             gate_mode=np.array([{"ste": 0, "soft": 1, "hard": 2}[mode]]))
    if cpi_mod > 0:
        d["cpi"] = (rng.random((B, K)) * 1.4 - 0.2).astype(np.float32)
    for key, shape, cx in (("gy", (B, K, H), False), ("gg", (B, K), False), ("gr", (B, K), False),
                           ("gn", (B, K), False), ("gh", (B, H, N), True), ("gt", (B,), False),
                           ("gu", (B, H), False), ("gB", (B, N), True), ("gC", (B, N), True)):
        d[key] = cplx(*shape) if cx else rng.standard_normal(shape).astype(np.float32)
    return d


@pytest.mark.parametrize("B,K,H,N,mode,cpi_mod,seed", [
    (4, 8, 768, 16, "ste", 0.0, 1),    # config 1's width
    (3, 6, 96, 32, "soft", 0.0, 2),
    (3, 6, 64, 5, "ste", 0.5, 3),      # CPI-modulated threshold, ragged N
    (2, 5, 40, 64, "hard", 0.0, 4),    # eval gate, the widest state
])
def test_stream_step_gradients_vs_oracle(B, K, H, N, mode, cpi_mod, seed):
    """The oracle takes the GPU's gate decisions (a residual on the threshold
    may decide either way in another summation order); the threshold sits
    between the residuals of an all-commit scan (its median, or its 97th percentile
    where the CPI lowers it)."""
    from oracle import oracle
    d = _random_case(B, K, H, N, mode, seed, cpi_mod)
    _, _, r0, _, _ = oracle.stream_chunk(d["lam"], d["log_dt"], d["D"], d["mean"], d["var"], d["u"], d["Bc"],
                                         d["Cc"], d["t"], d["valid"], d.get("cpi"),
                                         (d["h0"], d["t0"], d["u0"], d["B0"], d["C0"], d["init0"]), 0.0, 1e-6)
    eps = float(np.quantile(r0[d["valid"] > 0], 0.97 if cpi_mod > 0 else 0.5)) + 1e-4  # off every residual
    d["scalars"] = np.array([eps, 1e-6, 1e-5, 1.0, 1e-3, 1e3, cpi_mod, 0.3])
    outs, st, grads = _scan_gpu(d)
    if mode != "soft":
        assert 0.1 < outs["gate"][d["valid"] > 0].mean() < 0.95
    (oy, og, orr, on), ost, ograds = sgrad_oracle(d, pin=outs["gate"] if mode != "soft" else None)
    for got, ref, key in ((outs["y"], oy, "y"), (outs["resid"], orr, "resid"), (outs["innov"], on, "innov")):
        assert relerr(got, ref) < FWD_TOL, key
    for got, ref in zip(st, ost[:5]):
        assert relerr(got, ref) < FWD_TOL
    for k, v in grads.items():
        assert relerr(v, ograds[k]) < GRAD_TOL, (k, relerr(v, ograds[k]))


@pytest.fixture()
def ref():
    if reference_root() is None:
        pytest.skip("reference package not present")
    mods = import_reference()
    if mods is None:
        pytest.skip("reference not importable")
    import importlib
    mods["modules.streaming"] = importlib.import_module("cst_ssm.modules.streaming")
    saved = snapshot(mods) + [(mods["modules.streaming"], "temporal_step", mods["modules.streaming"].temporal_step)]
    reference_only(mods)
    yield mods
    restore(saved)


@pytest.mark.parametrize("train", [True, False])
def test_reference_temporal_step_gradients(ref, train):
    """The unmodified reference's temporal_step over 6 frames of a two-branch
    MultiScaleEACS (H=64) under autograd, with and without
    install(streaming=True): outputs, final states and the gradients of every
    parameter and of the input frames."""
    from cst_ssm.ops.spectral_init import BranchSpec
    ms_mod, st_mod = ref["modules.multiscale"], ref["modules.streaming"]
    torch.manual_seed(0)
    temporal = ms_mod.MultiScaleEACS(64, branches=[BranchSpec("a", 16, 0.5, 4.0), BranchSpec("b", 8, 4.0, 32.0)],
                                     gate_kwargs=dict(init_eps=0.6, eps_max=3.0, temperature=0.2)).to(DEV)
    temporal.train(train)
    twin = copy.deepcopy(temporal)
    g = torch.Generator().manual_seed(1)
    B, K = 3, 6
    x = torch.randn(B, K, 64, generator=g)
    x[:, 2] = x[:, 1] + 0.02 * torch.randn(B, 64, generator=g)
    x[:, 5] = x[:, 4]
    x = x.to(DEV)
    t = (1.0 + torch.cumsum(torch.rand(B, K, generator=g) * 0.5 + 0.05, 1)).to(DEV)
    valid = torch.ones(B, K, dtype=torch.bool, device=DEV)
    valid[1, 0] = False
    gy = torch.randn(B, K, 64, generator=g).to(DEV)

    def run(m):
        xx = x.clone().requires_grad_(True)
        states = st_mod.initial_states(m, B, DEV)
        ys, gs, rs = [], [], []
        for k in range(K):
            y, gk, r, n, w, states = st_mod.temporal_step(m, xx[:, k], t[:, k], states, valid[:, k])
            ys.append(y)
            gs.append(gk)
            rs.append(r)
        ys = torch.stack(ys, 1)
        loss = (ys * gy).sum() + sum((s.h.abs() ** 2).sum() * 0.01 + s.u.sum() * 0.1 for s in states)
        loss.backward()
        return ys.detach(), torch.stack(gs, 1).detach(), xx.grad, states, torch.stack(rs, 1).detach()

    from eacs_b200 import _lib
    n0 = _lib.kernel_launches()
    y_ref, g_ref, gx_ref, st_ref, r_ref = run(temporal)
    assert _lib.kernel_launches() == n0
    # every gate decided by more than 1e-4 (no residual on a threshold)
    eps = torch.tensor([float(b.gate.eps.detach()) for b in temporal.branches], device=DEV)
    assert float((r_ref - eps).abs()[valid].min()) > 1e-4
    import eacs_b200
    eacs_b200.install("cst_ssm", streaming=True)
    y, gates, gx, st, _ = run(twin)
    assert _lib.kernel_launches() > n0
    assert 0.1 < float(g_ref.float().mean()) < 0.95
    assert torch.equal(gates.float(), g_ref.float())
    assert relerr(y.cpu().numpy(), y_ref.cpu().numpy()) < FWD_TOL
    for s, s_ref in zip(st, st_ref):
        assert relerr(s.h.detach().cpu().numpy(), s_ref.h.detach().cpu().numpy()) < FWD_TOL
    assert relerr(gx.cpu().numpy(), gx_ref.cpu().numpy()) < GRAD_TOL
    for (name, p), p_ref in zip(twin.named_parameters(), temporal.parameters()):
        if p_ref.grad is None:
            assert p.grad is None or not p.grad.any(), name
            continue
        assert relerr(p.grad.cpu().numpy(), p_ref.grad.cpu().numpy()) < GRAD_TOL, name


def test_all_rows_masked_and_first_steps():
    """A step where no row is valid passes the state's adjoints through and
    gives the frame none; a step where every row starts (first observation)."""
    d = _random_case(3, 3, 32, 8, "ste", 11)
    d["valid"][:] = 1
    d["valid"][:, 1] = 0
    d["init0"][:] = 0
    d["scalars"] = np.array([0.5, 1e-6, 1e-5, 1.0, 1e-3, 1e3, 0.0, 0.3])
    outs, st, grads = _scan_gpu(d)
    (oy, og, orr, on), ost, ograds = sgrad_oracle(d, pin=outs["gate"])
    assert np.all(outs["gate"][:, 0] == 1.0) and np.all(outs["gate"][:, 1] == 0.0)
    assert not grads["du"][:, 1].any() and not grads["dt"][:, 1].any()
    for k, v in grads.items():
        assert relerr(v, ograds[k]) < GRAD_TOL, (k, relerr(v, ograds[k]))
