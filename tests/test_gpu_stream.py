"""Streaming steps with explicit branch state (eacs_stream_chunk, through
eacs_b200.ops.streaming) against the reference's temporal_step outputs
(tests/golden/stream.npz) and the oracle.

Tolerance: 1e-4 relative (max |x - ref| / max |ref|) on outputs and states;
gates exact (the golden cases keep every residual > 0.04 from its threshold).
"""
import numpy as np
import pytest
import torch
from torch import nn

from golden_io import cases, relerr
from inputs import cell_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-4
DEV = "cuda:0"

if torch.cuda.is_available():
    from eacs_b200 import _lib
    from eacs_b200.ops.streaming import stream_chunk, temporal_step

ST_KEYS = ("h", "st_t", "st_u", "st_B", "st_C", "st_init")


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _args(d):
    eps, eta, var_eps, dt_init, dt_min, dt_max, m, T, soft, mid = [float(v) for v in d["scalars"]]
    return dict(eps=eps, eta=eta, var_eps=var_eps, dt_init=dt_init, dt_min=dt_min, dt_max=dt_max,
                cpi_modulation=m, gate_mode="soft" if soft else "hard", temperature=T), int(mid)


def _zero_state(B, H, N):
    return (torch.zeros(B, H, N, dtype=torch.complex64, device=DEV), torch.zeros(B, device=DEV),
            torch.zeros(B, H, device=DEV), torch.zeros(B, N, dtype=torch.complex64, device=DEV),
            torch.zeros(B, N, dtype=torch.complex64, device=DEV),
            torch.zeros(B, dtype=torch.bool, device=DEV))


def _run(d, lo, hi, state, kw, u_dtype=torch.float32):
    sl = lambda k: _t(d[k][:, lo:hi])
    cpi = None if d.get("cpi") is None else sl("cpi")
    return stream_chunk(_t(d["lam"]), _t(d["log_dt"]), _t(d["D"]), _t(d["mean"]), _t(d["var"]),
                        sl("u").to(u_dtype), sl("Bc"), sl("Cc"), sl("t"), sl("valid").bool(), cpi,
                        state, **kw)


@pytest.mark.parametrize("name", sorted(cases("stream")))
def test_stream_golden(name):
    d = cases("stream")[name]
    kw, mid = _args(d)
    B, K, H = d["u"].shape
    N = d["lam"].shape[1]
    y, g, r, n, st = _run(d, 0, K, _zero_state(B, H, N), kw)
    assert np.array_equal(g.cpu().numpy() > 0.5, d["gate"] > 0.5)
    for got, key in zip((y, g, r, n), ("y", "gate", "resid", "innov")):
        assert relerr(got.cpu().numpy(), d[key]) < TOL, key
    for got, key in zip(st, ST_KEYS):
        assert relerr(got.cpu().numpy(), d[key]) < TOL, key
    # the same sequence one step per launch (temporal_step's granularity) and in two chunks
    state = _zero_state(B, H, N)
    ys = []
    for k in range(K):
        yk, _, _, _, state = _run(d, k, k + 1, state, kw)
        ys.append(yk)
        if k == mid - 1:
            for got, key in zip(state, ("mid_h", "mid_t", "mid_u", "mid_B", "mid_C", "mid_init")):
                assert relerr(got.cpu().numpy(), d[key]) < TOL, key
    assert torch.equal(torch.cat(ys, 1), y)
    assert torch.equal(state[0], st[0])
    assert _lib.device_status() == 0


@pytest.mark.parametrize("B,K,H,N,soft,cpi_mod,eps", [
    (3, 40, 96, 16, False, 0.0, 1.0), (2, 25, 40, 32, True, 0.0, 1.0),
    (2, 30, 24, 5, False, 0.6, 1.1), (1, 7, 130, 64, False, 0.0, 1.0),
    (4, 1, 16, 4, True, 0.3, 1.0),
])
def test_stream_vs_oracle(B, K, H, N, soft, cpi_mod, eps):
    """Mixed gates (update rates 0.33-0.88 on the hard cases, every residual at
    least 1.3e-4 from its threshold), random valid masks, bf16 u."""
    d = cell_inputs(B, K, H, N, seed=B * K + H + N)
    rng = np.random.default_rng(K)
    valid = (rng.random((B, K)) > 0.2).astype(np.uint8)
    cpi = (rng.random((B, K)) * 1.4 - 0.2).astype(np.float32) if cpi_mod > 0 else None
    kw = dict(eps=eps, eta=1e-6, cpi_modulation=cpi_mod, gate_mode="soft" if soft else "hard",
              temperature=0.2)
    state = _zero_state(B, H, N)
    y, g, r, n, st = stream_chunk(_t(d["lam"]), _t(d["log_dt"]), _t(d["D"]), _t(d["mean"]),
                                  _t(d["var"]), _t(d["u"]).to(torch.bfloat16), _t(d["Bc"]),
                                  _t(d["Cc"]), _t(d["t"]), _t(valid).bool(),
                                  None if cpi is None else _t(cpi), state, **kw)
    u_seen = _t(d["u"]).to(torch.bfloat16).float().cpu().numpy()
    z = tuple(x.cpu().numpy() for x in state)
    ref = oracle.stream_chunk(d["lam"], d["log_dt"], d["D"], d["mean"], d["var"], u_seen, d["Bc"],
                              d["Cc"], d["t"], valid, cpi, z, eps, 1e-6, cpi_mod=cpi_mod,
                              gate_mode=int(soft), T=0.2)
    eps_l = np.full(ref[2].shape, eps, np.float32)
    if cpi is not None:
        eps_l = np.maximum(eps * (1 - cpi_mod * np.clip(cpi, 0, 1)), 1e-3)
    seen = valid.astype(bool) & (ref[3] != 0)  # valid steps after a row's first
    assert soft or not seen.any() or np.abs(ref[2] - eps_l)[seen].min() > 1e-4
    for got, want in zip((y, g, r, n), ref[:4]):
        assert relerr(got.cpu().numpy(), want) < TOL
    for got, want in zip(st, ref[4]):
        assert relerr(got.cpu().numpy(), want) < TOL
    # the input state is left untouched
    assert not bool(state[5].any()) and not bool(state[0].abs().sum())


class _Gate(nn.Module):
    def __init__(self, eps):
        super().__init__()
        self.eps = torch.tensor(eps)
        self.norm_eta = 1e-6
        self.gate_kind = "event"
        self.cpi_modulation = 0.0
        self.use_ste = True
        self.temperature = torch.tensor(0.1)


class _Std(nn.Module):
    def __init__(self, mean, var):
        super().__init__()
        self.register_buffer("running_mean", mean)
        self.register_buffer("running_var", var)
        self.eps = 1e-5


class StreamBranch(nn.Module):
    """A branch whose projections return the test's own per-step B and C."""

    def __init__(self, d, eps):
        super().__init__()
        self.lam_c = _t(d["lam"])
        self.log_dt_scale = _t(d["log_dt"])
        self.D = _t(d["D"])
        self.obs_norm = _Std(_t(d["mean"]), _t(d["var"]))
        self.gate = _Gate(eps)
        self.disc_mode = "continuous"
        self.robust_guard = False
        self.dt_init, self.dt_max = 1.0, 1e3
        self.Bc, self.Cc = _t(d["Bc"]), _t(d["Cc"])
        self.k = 0
        self.norm = nn.Identity()
        self.proj_out = nn.Identity()

    def lam(self):
        return self.lam_c

    def _project(self, x):
        return x.float(), self.Bc[:, self.k], self.Cc[:, self.k]


class StreamState:  # field order of streaming.py's BranchState
    def __init__(self, h, t, u, B, C, initialized):
        self.h, self.t, self.u, self.B, self.C, self.initialized = h, t, u, B, C, initialized


def test_temporal_step_one_branch():
    B, K, H, N = 2, 20, 32, 16
    d = cell_inputs(B, K, H, N, seed=77)
    br = StreamBranch(d, 0.9).eval()
    temporal = nn.Module()
    temporal.branches = nn.ModuleList([br])
    temporal.fusion = nn.Linear(H, 1).to(DEV)
    temporal.out_norm = nn.Identity()
    valid = np.ones((B, K), np.uint8)
    valid[1, :4] = 0
    states = [StreamState(*_zero_state(B, H, N))]
    ys = []
    with torch.no_grad():
        for k in range(K):
            br.k = k
            x = _t(d["u"][:, k])
            y, g, r, n, w, states = temporal_step(temporal, x, _t(d["t"][:, k]), states,
                                                  _t(valid[:, k]).bool())
            ys.append(y - x * _t(valid[:, k])[:, None].float())
    z = tuple(x.cpu().numpy() for x in _zero_state(B, H, N))
    ref = oracle.stream_chunk(d["lam"], d["log_dt"], d["D"], d["mean"], d["var"], d["u"], d["Bc"],
                              d["Cc"], d["t"], valid, None, z, 0.9, 1e-6)
    assert relerr(torch.stack(ys, 1).cpu().numpy(), ref[0]) < TOL
    assert relerr(states[0].h.cpu().numpy(), ref[4][0]) < TOL
