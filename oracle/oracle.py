"""ctypes binding of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm import this module; the product path never does.  All arrays are numpy,
complex arrays are complex64 (interleaved float pairs), real arrays float32.
Each function names the reference code it restates (paths inside the
CST-SSM project, BitGao-ai/LongVideo-main).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libeacs_oracle.so")
_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_I = ctypes.c_int


def build() -> str:
    """Compile eacs_oracle.c with the committed Makefile; returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.eacs_oracle_scan_fwd.argtypes = [_P, _P, _P, _I64, _I64, _I64, _I64]
        L.eacs_oracle_scan_bwd.argtypes = [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64]
        L.eacs_oracle_ssm_fwd.argtypes = [_P] * 8 + [_I64] * 4 + [_F, _F]
        L.eacs_oracle_ssm_bwd.argtypes = [_P] * 15 + [_I64] * 4 + [_F, _F]
        L.eacs_oracle_cell_fwd.argtypes = ([_P] * 9 + [_F] * 6 + [_I, _I, _F, _F, _I, _F, _I]
                                           + [_P] * 3 + [_I64] * 4)
        L.eacs_oracle_cell_bwd.argtypes = ([_P] * 9 + [_F] * 5 + [_F, _I] + [_P] * 5
                                           + [_P] * 8 + [_I64] * 4)
        L.eacs_oracle_cell_commits.argtypes = ([_P] * 9 + [_F] * 6 + [_I, _I, _F, _F]
                                               + [_P] * 8 + [_I64] * 4)
        L.eacs_oracle_query_readout.argtypes = [_P] * 12 + [_I64] * 5 + [_F, _F]
        L.eacs_oracle_cell_bwd_commits.argtypes = ([_P] * 9 + [_F] * 5 + [_F, _I] + [_P] * 4
                                                   + [_P] * 5 + [_P] * 8 + [_P] * 8 + [_I64] * 4)
        L.eacs_oracle_query_readout_bwd.argtypes = [_P] * 21 + [_I64] * 5 + [_F, _F]
        L.eacs_oracle_stream_step_bwd.argtypes = [_P] * 41 + [_F] * 7 + [_I, _F] + [_I64] * 3
        L.eacs_oracle_stream_chunk.argtypes = [_P] * 27 + [_F] * 7 + [_I, _F] + [_I64] * 4
        L.eacs_oracle_set_threads.argtypes = [_I]
        L.eacs_oracle_version.restype = ctypes.c_char_p
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    """Number of OpenMP threads the oracle uses (0 = all available)."""
    lib().eacs_oracle_set_threads(int(n))


def _c(x, dtype):
    return np.ascontiguousarray(np.asarray(x), dtype=dtype)


def _ptr(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def scan_fwd(a, b):
    """sequential_scan_diag (cst_ssm/ops/scan.py:36-44): h_l = a_l h_{l-1} + b_l."""
    a = _c(a, np.complex64)
    b = _c(b, np.complex64)
    B, L, H, N = a.shape
    h = np.empty_like(a)
    lib().eacs_oracle_scan_fwd(_ptr(a), _ptr(b), _ptr(h), B, L, H, N)
    return h


def scan_bwd(a, h, gh):
    """Adjoint of the scan (cst_ssm/ops/csrc/eacs_scan_cuda.cu:40-60)."""
    a = _c(a, np.complex64)
    h = _c(h, np.complex64)
    gh = _c(gh, np.complex64)
    B, L, H, N = a.shape
    ga = np.empty_like(a)
    gb = np.empty_like(a)
    lib().eacs_oracle_scan_bwd(_ptr(a), _ptr(h), _ptr(gh), _ptr(ga), _ptr(gb), B, L, H, N)
    return ga, gb


def ssm_fwd(lam, log_dt, t, Bc, Cc, u, D, dt_min=1e-3, dt_max=1e3):
    """ContinuousSSMLayer core (cst_ssm/modules/continuous_ssm.py:44-55)."""
    lam = _c(lam, np.complex64)
    log_dt = _c(log_dt, np.float32)
    t = _c(t, np.float32)
    Bc = _c(Bc, np.complex64)
    Cc = _c(Cc, np.complex64)
    u = _c(u, np.float32)
    D = _c(D, np.float32)
    B, L, H = u.shape
    N = lam.shape[1]
    y = np.empty((B, L, H), np.float32)
    lib().eacs_oracle_ssm_fwd(_ptr(lam), _ptr(log_dt), _ptr(t), _ptr(Bc), _ptr(Cc), _ptr(u),
                              _ptr(D), _ptr(y), B, L, H, N, dt_min, dt_max)
    return y


def ssm_bwd(lam, log_dt, t, Bc, Cc, u, D, gy, dt_min=1e-3, dt_max=1e3):
    """Backward of the ungated core (autograd of continuous_ssm.py:44-55).

    Returns (du, dBc, dCc, dt, dlam, dlog_dt, dD)."""
    lam = _c(lam, np.complex64)
    log_dt = _c(log_dt, np.float32)
    t = _c(t, np.float32)
    Bc = _c(Bc, np.complex64)
    Cc = _c(Cc, np.complex64)
    u = _c(u, np.float32)
    D = _c(D, np.float32)
    gy = _c(gy, np.float32)
    B, L, H = u.shape
    N = lam.shape[1]
    du = np.empty((B, L, H), np.float32)
    dBc = np.empty((B, L, N), np.complex64)
    dCc = np.empty((B, L, N), np.complex64)
    dt = np.empty((B, L), np.float32)
    dlam = np.empty((H, N), np.complex64)
    dlog = np.empty((H,), np.float32)
    dD = np.empty((H,), np.float32)
    lib().eacs_oracle_ssm_bwd(_ptr(lam), _ptr(log_dt), _ptr(t), _ptr(Bc), _ptr(Cc), _ptr(u), _ptr(D),
                              _ptr(gy), _ptr(du), _ptr(dBc), _ptr(dCc), _ptr(dt), _ptr(dlam),
                              _ptr(dlog), _ptr(dD), B, L, H, N, dt_min, dt_max)
    return du, dBc, dCc, dt, dlam, dlog, dD


def cell_fwd(lam, log_dt, u, Bc, Cc, t, D, mean, var, eps, eta, var_eps=1e-5,
             dt_init=1.0, dt_min=1e-3, dt_max=1e3, robust=None, gate_mode=0, T=0.1,
             train_exp=False):
    """Gated EACS cell over L (cst_ssm/modules/eacs.py:78-173, scan_range).

    robust: None or (k, spike_ratio, eps_factor) (eacs.py:67-71).
    gate_mode 0: hard gate; 1: soft gate blended into the state
    (cst_ssm/ops/eacs_cell_train.py:47-63).  train_exp selects the training
    cell's dA = exp(z) (eacs_cell_train.py:33) instead of zoh_kernels' form.
    Returns (y (B,L,H), gate (B,L), resid (B,L)).
    """
    lam = _c(lam, np.complex64)
    u = _c(u, np.float32)
    Bc = _c(Bc, np.complex64)
    Cc = _c(Cc, np.complex64)
    t = _c(t, np.float32)
    log_dt = _c(log_dt, np.float32)
    D = _c(D, np.float32)
    mean = _c(mean, np.float32)
    var = _c(var, np.float32)
    B, L, H = u.shape
    N = lam.shape[1]
    y = np.empty((B, L, H), np.float32)
    g = np.empty((B, L), np.float32)
    r = np.empty((B, L), np.float32)
    rk, rr, rf = (0, 2.0, 0.3) if robust is None else robust
    lib().eacs_oracle_cell_fwd(_ptr(lam), _ptr(log_dt), _ptr(u), _ptr(Bc), _ptr(Cc), _ptr(t),
                               _ptr(D), _ptr(mean), _ptr(var), eps, eta, var_eps, dt_init,
                               dt_min, dt_max, 0 if robust is None else 1, int(rk), rr, rf,
                               int(gate_mode), T, 1 if train_exp else 0,
                               _ptr(y), _ptr(g), _ptr(r), B, L, H, N)
    return y, g, r


def cell_bwd(lam, log_dt, u, Bc, Cc, t, D, mean, var, eps, eta, var_eps, dt_init, dt_max,
             T, gate_mode, gs, gy=None, ggs=None, grs=None, gns=None):
    """Backward of GatedEACSCellFunction (cst_ssm/ops/eacs_cell_train.py:117-175).

    Returns (du, dBc, dCc, dt, dlam, dlog_dt, dD, deps).
    """
    lam = _c(lam, np.complex64)
    u = _c(u, np.float32)
    Bc = _c(Bc, np.complex64)
    Cc = _c(Cc, np.complex64)
    t = _c(t, np.float32)
    log_dt = _c(log_dt, np.float32)
    D = _c(D, np.float32)
    mean = _c(mean, np.float32)
    var = _c(var, np.float32)
    gs = _c(gs, np.float32)
    gy = None if gy is None else _c(gy, np.float32)
    ggs = None if ggs is None else _c(ggs, np.float32)
    grs = None if grs is None else _c(grs, np.float32)
    gns = None if gns is None else _c(gns, np.float32)
    B, L, H = u.shape
    N = lam.shape[1]
    du = np.empty((B, L, H), np.float32)
    dBc = np.empty((B, L, N), np.complex64)
    dCc = np.empty((B, L, N), np.complex64)
    dt = np.empty((B, L), np.float32)
    dlam = np.empty((H, N), np.complex64)
    dlog = np.empty((H,), np.float32)
    dD = np.empty((H,), np.float32)
    deps = np.empty((1,), np.float32)
    lib().eacs_oracle_cell_bwd(_ptr(lam), _ptr(log_dt), _ptr(u), _ptr(Bc), _ptr(Cc), _ptr(t),
                               _ptr(D), _ptr(mean), _ptr(var), eps, eta, var_eps, dt_init,
                               dt_max, T, int(gate_mode), _ptr(gs), _ptr(gy), _ptr(ggs),
                               _ptr(grs), _ptr(gns), _ptr(du), _ptr(dBc), _ptr(dCc), _ptr(dt),
                               _ptr(dlam), _ptr(dlog), _ptr(dD), _ptr(deps), B, L, H, N)
    return du, dBc, dCc, dt, dlam, dlog, dD, deps


def cell_train_commits(lam, log_dt, u, Bc, Cc, t, D, mean, var, eps, eta, var_eps, dt_init,
                       dt_max, T, gate_mode, gs=None, gy=None, ggs=None, grs=None, gc=None):
    """Training through per-frame commits: EACSLayer._commit_range
    (cst_ssm/modules/eacs.py:386-401) under autograd with the training gate
    (gate_mode 0: STE, hard forward; 1: soft).

    gs: forward gates to pin (None: decided here, r > eps); gc: upstream
    adjoints of the commits, a dict with any of h, t, u, B, C.
    Returns (forward, grads): forward = (y, gate, resid, h, t_pi, u_pi, B_pi,
    C_pi), grads = (du, dBc, dCc, dt, dlam, dlog_dt, dD, deps).
    """
    lam = _c(lam, np.complex64)
    u = _c(u, np.float32)
    Bc = _c(Bc, np.complex64)
    Cc = _c(Cc, np.complex64)
    t = _c(t, np.float32)
    log_dt = _c(log_dt, np.float32)
    D = _c(D, np.float32)
    mean = _c(mean, np.float32)
    var = _c(var, np.float32)
    B, L, H = u.shape
    N = lam.shape[1]
    gs = None if gs is None else _c(gs, np.float32)
    opt = [None if g is None else _c(g, np.float32) for g in (gy, ggs, grs)]
    gc = gc or {}
    kinds = {"h": np.complex64, "t": np.float32, "u": np.float32, "B": np.complex64, "C": np.complex64}
    gcs = [None if gc.get(k) is None else _c(gc[k], kinds[k]) for k in ("h", "t", "u", "B", "C")]
    fwd = (np.empty((B, L, H), np.float32), np.empty((B, L), np.float32), np.empty((B, L), np.float32),
           np.empty((B, L, H, N), np.complex64), np.empty((B, L), np.float32),
           np.empty((B, L, H), np.float32), np.empty((B, L, N), np.complex64),
           np.empty((B, L, N), np.complex64))
    grads = (np.empty((B, L, H), np.float32), np.empty((B, L, N), np.complex64),
             np.empty((B, L, N), np.complex64), np.empty((B, L), np.float32),
             np.empty((H, N), np.complex64), np.empty((H,), np.float32), np.empty((H,), np.float32),
             np.empty((1,), np.float32))
    lib().eacs_oracle_cell_bwd_commits(
        _ptr(lam), _ptr(log_dt), _ptr(u), _ptr(Bc), _ptr(Cc), _ptr(t), _ptr(D), _ptr(mean),
        _ptr(var), eps, eta, var_eps, dt_init, dt_max, T, int(gate_mode), _ptr(gs),
        *[_ptr(g) for g in opt], *[_ptr(g) for g in gcs], *[_ptr(g) for g in grads],
        *[_ptr(f) for f in fwd], B, L, H, N)
    return fwd, grads


def query_readout_bwd(lam, log_dt, D, ch, ct, cu, cB, cC, frame_t, t_query, gy, idx=None,
                      dt_min=1e-3, dt_max=1e3):
    """Adjoint of readout_from_commits before proj_out
    (cst_ssm/modules/continuous_query.py:20-54).

    Returns (gc, gtq, dlam, dlog_dt, dD) with gc a dict h, t, u, B, C of the
    commits' adjoints."""
    lam = _c(lam, np.complex64)
    log_dt = _c(log_dt, np.float32)
    D = _c(D, np.float32)
    ch = _c(ch, np.complex64)
    ct = _c(ct, np.float32)
    cu = _c(cu, np.float32)
    cB = _c(cB, np.complex64)
    cC = _c(cC, np.complex64)
    frame_t = _c(frame_t, np.float32)
    t_query = _c(t_query, np.float32)
    gy = _c(gy, np.float32)
    idx = None if idx is None else _c(idx, np.int32)
    B, L, H, N = ch.shape
    Q = t_query.shape[1]
    gc = dict(h=np.empty((B, L, H, N), np.complex64), t=np.empty((B, L), np.float32),
              u=np.empty((B, L, H), np.float32), B=np.empty((B, L, N), np.complex64),
              C=np.empty((B, L, N), np.complex64))
    gtq = np.empty((B, Q), np.float32)
    dlam = np.empty((H, N), np.complex64)
    dlog = np.empty((H,), np.float32)
    dD = np.empty((H,), np.float32)
    lib().eacs_oracle_query_readout_bwd(
        _ptr(lam), _ptr(log_dt), _ptr(D), _ptr(ch), _ptr(ct), _ptr(cu), _ptr(cB), _ptr(cC),
        _ptr(frame_t), _ptr(t_query), _ptr(idx), _ptr(gy), _ptr(gc["h"]), _ptr(gc["t"]),
        _ptr(gc["u"]), _ptr(gc["B"]), _ptr(gc["C"]), _ptr(gtq), _ptr(dlam), _ptr(dlog), _ptr(dD),
        B, L, Q, H, N, dt_min, dt_max)
    return gc, gtq, dlam, dlog, dD


def stream_step_bwd(lam, log_dt, D, mean, var, u, Bc, Cc, t, valid, cpi, state, up, eps, eta,
                    var_eps=1e-5, dt_init=1.0, dt_min=1e-3, dt_max=1e3, cpi_mod=0.0, gate_mode=0,
                    T=0.1, gs=None):
    """Backward of one streaming step of one branch (the per-branch body of
    temporal_step, cst_ssm/modules/streaming.py:55-80, over eacs_step).

    u (B,H), Bc/Cc (B,N), t (B), valid (B) bool or None, cpi (B) or None;
    state = (h (B,H,N), t (B), u (B,H), B (B,N), C (B,N), initialized (B));
    up: dict of upstream gradients with any of y (B,H), gate, resid, innov
    (B), h, t, u, B, C (the state out).  gate_mode 0 STE, 1 soft, 2 hard
    (no gradient through the gate).  Returns dict du, dBc, dCc, dt, dcpi,
    dh, dt_in, du_in, dB_in, dC_in, dlam, dlog_dt, dD, deps."""
    lam = _c(lam, np.complex64)
    B, H = np.asarray(u).shape
    N = lam.shape[1]
    f = lambda x: None if x is None else _c(x, np.float32)  # noqa: E731
    c = lambda x: None if x is None else _c(x, np.complex64)  # noqa: E731
    h0, t0, u0, B0, C0, i0 = state
    valid = None if valid is None else _c(valid, np.uint8)
    ins = [lam, f(log_dt), f(D), f(mean), f(var), f(u), c(Bc), c(Cc), f(t)]
    st = [c(h0), f(t0), f(u0), c(B0), c(C0), _c(i0, np.uint8)]
    ups = [f(up.get("y")), f(up.get("gate")), f(up.get("resid")), f(up.get("innov")), c(up.get("h")),
           f(up.get("t")), f(up.get("u")), c(up.get("B")), c(up.get("C"))]
    out = dict(du=np.empty((B, H), np.float32), dBc=np.empty((B, N), np.complex64),
               dCc=np.empty((B, N), np.complex64), dt=np.empty(B, np.float32), dcpi=np.empty(B, np.float32),
               dh=np.empty((B, H, N), np.complex64), dt_in=np.empty(B, np.float32),
               du_in=np.empty((B, H), np.float32), dB_in=np.empty((B, N), np.complex64),
               dC_in=np.empty((B, N), np.complex64), dlam=np.empty((H, N), np.complex64),
               dlog_dt=np.empty(H, np.float32), dD=np.empty(H, np.float32), deps=np.empty(1, np.float32))
    lib().eacs_oracle_stream_step_bwd(
        *[_ptr(x) for x in ins], _ptr(valid), _ptr(f(cpi)), *[_ptr(x) for x in st], _ptr(f(gs)),
        *[_ptr(x) for x in ups], *[_ptr(out[k]) for k in out], eps, eta, var_eps, dt_init, dt_min,
        dt_max, cpi_mod, int(gate_mode), T, B, H, N)
    return out


def cell_commits(lam, log_dt, u, Bc, Cc, t, D, mean, var, eps, eta, var_eps=1e-5,
                 dt_init=1.0, dt_min=1e-3, dt_max=1e3, robust=None):
    """Hard-gate cell recording per-frame commits (cst_ssm/modules/eacs.py:386-439).

    Returns (y, gate, resid, h (B,L,H,N), t_pi (B,L), u_pi (B,L,H), B_pi, C_pi (B,L,N))."""
    lam = _c(lam, np.complex64)
    u = _c(u, np.float32)
    Bc = _c(Bc, np.complex64)
    Cc = _c(Cc, np.complex64)
    t = _c(t, np.float32)
    log_dt = _c(log_dt, np.float32)
    D = _c(D, np.float32)
    mean = _c(mean, np.float32)
    var = _c(var, np.float32)
    B, L, H = u.shape
    N = lam.shape[1]
    y = np.empty((B, L, H), np.float32)
    g = np.empty((B, L), np.float32)
    r = np.empty((B, L), np.float32)
    ch = np.empty((B, L, H, N), np.complex64)
    ct = np.empty((B, L), np.float32)
    cu = np.empty((B, L, H), np.float32)
    cB = np.empty((B, L, N), np.complex64)
    cC = np.empty((B, L, N), np.complex64)
    rk, rr, rf = (0, 2.0, 0.3) if robust is None else robust
    lib().eacs_oracle_cell_commits(_ptr(lam), _ptr(log_dt), _ptr(u), _ptr(Bc), _ptr(Cc), _ptr(t),
                                   _ptr(D), _ptr(mean), _ptr(var), eps, eta, var_eps, dt_init,
                                   dt_min, dt_max, 0 if robust is None else 1, int(rk), rr, rf,
                                   _ptr(y), _ptr(g), _ptr(r), _ptr(ch), _ptr(ct), _ptr(cu),
                                   _ptr(cB), _ptr(cC), B, L, H, N)
    return y, g, r, ch, ct, cu, cB, cC


def query_readout(lam, log_dt, D, ch, ct, cu, cB, cC, frame_t, t_query, idx=None,
                  dt_min=1e-3, dt_max=1e3):
    """readout_from_commits before proj_out (cst_ssm/modules/continuous_query.py:20-61)."""
    lam = _c(lam, np.complex64)
    log_dt = _c(log_dt, np.float32)
    D = _c(D, np.float32)
    ch = _c(ch, np.complex64)
    ct = _c(ct, np.float32)
    cu = _c(cu, np.float32)
    cB = _c(cB, np.complex64)
    cC = _c(cC, np.complex64)
    frame_t = _c(frame_t, np.float32)
    t_query = _c(t_query, np.float32)
    idx = None if idx is None else _c(idx, np.int32)
    B, L, H, N = ch.shape
    Q = t_query.shape[1]
    y = np.empty((B, Q, H), np.float32)
    lib().eacs_oracle_query_readout(_ptr(lam), _ptr(log_dt), _ptr(D), _ptr(ch), _ptr(ct), _ptr(cu),
                                    _ptr(cB), _ptr(cC), _ptr(frame_t), _ptr(t_query), _ptr(idx),
                                    _ptr(y), B, L, Q, H, N, dt_min, dt_max)
    return y


def stream_chunk(lam, log_dt, D, mean, var, u, Bc, Cc, t, valid, cpi, state, eps, eta,
                 var_eps=1e-5, dt_init=1.0, dt_min=1e-3, dt_max=1e3, cpi_mod=0.0,
                 gate_mode=0, T=0.1):
    """K streaming steps of one branch with explicit state
    (cst_ssm/modules/streaming.py:45-85).  state = (h (B,H,N), t (B), u (B,H),
    B (B,N), C (B,N), initialized (B)).  Returns (y, gate, resid, innov, state')."""
    lam = _c(lam, np.complex64)
    log_dt = _c(log_dt, np.float32)
    D = _c(D, np.float32)
    mean = _c(mean, np.float32)
    var = _c(var, np.float32)
    u = _c(u, np.float32)
    Bc = _c(Bc, np.complex64)
    Cc = _c(Cc, np.complex64)
    t = _c(t, np.float32)
    valid = None if valid is None else _c(valid, np.uint8)
    cpi = None if cpi is None else _c(cpi, np.float32)
    h0, t0, u0, B0, C0, i0 = state
    h0, t0, u0 = _c(h0, np.complex64), _c(t0, np.float32), _c(u0, np.float32)
    B0, C0, i0 = _c(B0, np.complex64), _c(C0, np.complex64), _c(i0, np.uint8)
    B, K, H = u.shape
    N = lam.shape[1]
    h1, t1, u1 = np.empty_like(h0), np.empty_like(t0), np.empty_like(u0)
    B1, C1, i1 = np.empty_like(B0), np.empty_like(C0), np.empty_like(i0)
    y = np.empty((B, K, H), np.float32)
    g, r, n = (np.empty((B, K), np.float32) for _ in range(3))
    lib().eacs_oracle_stream_chunk(_ptr(lam), _ptr(log_dt), _ptr(D), _ptr(mean), _ptr(var), _ptr(u),
                                   _ptr(Bc), _ptr(Cc), _ptr(t), _ptr(valid), _ptr(cpi), _ptr(h0),
                                   _ptr(t0), _ptr(u0), _ptr(B0), _ptr(C0), _ptr(i0), _ptr(h1),
                                   _ptr(t1), _ptr(u1), _ptr(B1), _ptr(C1), _ptr(i1), _ptr(y),
                                   _ptr(g), _ptr(r), _ptr(n), eps, eta, var_eps, dt_init, dt_min,
                                   dt_max, cpi_mod, int(gate_mode), T, B, K, H, N)
    return y, g, r, n, (h1, t1, u1, B1, C1, i1)
