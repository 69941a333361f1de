"""Generate golden vectors for the EACS hot path by running the reference.

Runs the reference's own PyTorch implementation (CST-SSM, imported from a
checkout given by --reference, default /root/reference) on small seeded inputs
and writes the op-boundary inputs and outputs to tests/golden/*.npz.  The
fixtures pin the CPU oracle (oracle/eacs_oracle.c) and the CUDA kernels; the
tests that read them never import the reference.

    python tests/golden/make_golden.py [--reference PATH]

Reference functions exercised (paths inside the CST-SSM project):
  ops/scan.py:36-44            sequential_scan_diag (+ autograd for the adjoint)
  ops/discretization.py:20-82  zoh_kernels / zoh_discretize / effective_dt
  modules/continuous_ssm.py:44-55  ungated layer core
  modules/eacs.py:78-173       eacs_step / scan_range (+ RobustCfg)
  ops/eacs_cell_train.py:81-199  GatedEACSCellFunction forward/backward
  modules/eacs.py:386-439      run_with_commits (per-frame commits)
  modules/continuous_query.py:12-61  segment_index / readout_from_commits
  modules/streaming.py:45-85   temporal_step (explicit branch state)
  modules/eacs.py:386-401 + continuous_query.py:20-54  _commit_range and
                               readout_from_commits under autograd (training)
  modules/streaming.py:45-85   temporal_step under autograd (training)

    python tests/golden/make_golden.py --groups query   # rewrite one group only
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(x):
    x = x.detach().cpu()
    if x.is_complex():
        return x.to(torch.complex64).numpy()
    return x.to(torch.float32).numpy()


def timestamps_exp(gen, B, L, mean=0.25, lo=1 / 30, hi=2.0):
    """Cumulative dt with dt ~ Exponential(mean) clipped to [lo, hi]."""
    dt = torch.empty(B, L).exponential_(1.0 / mean, generator=gen).clamp(lo, hi)
    return torch.cumsum(dt, 1)


def scan_cases(gen):
    from cst_ssm.ops.scan import sequential_scan_diag, associative_scan_diag
    out = {}
    for name, (B, L, H, N) in {"scan_small": (2, 33, 5, 4), "scan_odd": (1, 7, 3, 3)}.items():
        mag = torch.rand(B, L, H, N, generator=gen) * 0.3 + 0.69
        ph = torch.rand(B, L, H, N, generator=gen) * 2 * math.pi
        a = torch.polar(mag, ph).to(torch.complex64)
        b = torch.complex(torch.randn(B, L, H, N, generator=gen),
                          torch.randn(B, L, H, N, generator=gen))
        gh = torch.complex(torch.randn(B, L, H, N, generator=gen),
                           torch.randn(B, L, H, N, generator=gen))
        a_ = a.clone().requires_grad_(True)
        b_ = b.clone().requires_grad_(True)
        h = sequential_scan_diag(a_, b_)
        ga, gb = torch.autograd.grad(h, [a_, b_], gh)
        h_assoc = associative_scan_diag(a, b)
        out[name] = dict(a=_np(a), b=_np(b), h=_np(h), gh=_np(gh), ga=_np(ga), gb=_np(gb),
                         h_assoc=_np(h_assoc))
    return out


def ssm_core(lam, log_dt, t, Bc, Cc, u, D):
    """continuous_ssm.py:44-55 with the reference's own discretisation and scan."""
    from cst_ssm.ops.discretization import effective_dt, zoh_discretize
    from cst_ssm.ops.scan import sequential_scan_diag
    dt = torch.zeros_like(t)
    dt[:, 1:] = (t[:, 1:] - t[:, :-1]).clamp_min(0)
    if t.shape[1] > 1:
        dt[:, 0] = dt[:, 1]
    dt_eff = effective_dt(dt.unsqueeze(-1), log_dt)
    dA, dB = zoh_discretize(lam, dt_eff, Bc, inv_lam=torch.reciprocal(lam))
    dBu = dB * u.unsqueeze(-1)
    h = sequential_scan_diag(dA, dBu)
    return torch.einsum("bln,blhn->blh", Cc, h).real + D * u


def ssm_cases(gen):
    from cst_ssm.ops.discretization import make_lambda
    from cst_ssm.ops.spectral_init import BranchSpec, init_branch_lambda
    out = {}
    cases = {
        # the CPU scan case: B=2, L=256, D=64 channels, N=16, tau log-uniform [0.5, 64] s.
        "ssm_c0": (2, 256, 64, 16, 0.5, 64.0, False),
        "ssm_odd": (3, 9, 7, 5, 0.1, 4.0, True),
        "ssm_l1": (2, 1, 4, 4, 0.5, 4.0, False),
    }
    for name, (B, L, H, N, tmin, tmax, dup) in cases.items():
        a_lnr, a_im = init_branch_lambda(BranchSpec(name, N, tmin, tmax), H, generator=gen)
        lam = make_lambda(a_lnr, a_im).to(torch.complex64)
        log_dt = torch.randn(H, generator=gen) * 0.3
        t = timestamps_exp(gen, B, L)
        if dup and L > 3:
            t[:, 3] = t[:, 2]           # duplicate timestamp: dt = 0 -> dt_min clamp
            t[0, 5] = t[0, 4] - 0.5     # decreasing timestamp: clamp_min(0)
        s = 1.0 / math.sqrt(N)
        Bc = torch.complex(torch.randn(B, L, N, generator=gen) * s,
                           torch.randn(B, L, N, generator=gen) * s)
        Cc = torch.complex(torch.randn(B, L, N, generator=gen) * s,
                           torch.randn(B, L, N, generator=gen) * s)
        u = torch.randn(B, L, H, generator=gen)
        D = torch.randn(H, generator=gen)
        gy = torch.randn(B, L, H, generator=gen)
        leaves = [x.clone().requires_grad_(True) for x in (lam, log_dt, t, Bc, Cc, u, D)]
        y = ssm_core(*leaves)
        grads = torch.autograd.grad(y, leaves, gy)
        gl = dict(zip(["dlam", "dlog_dt", "dt", "dBc", "dCc", "du", "dD"], grads))
        out[name] = dict(lam=_np(lam), log_dt=_np(log_dt), t=_np(t), Bc=_np(Bc), Cc=_np(Cc),
                         u=_np(u), D=_np(D), y=_np(y), gy=_np(gy), **{k: _np(v) for k, v in gl.items()})
    return out


def _layer_inputs(H, N, tmin, tmax, B, L, seed, dup_frames=False, ramp=False):
    """Op-boundary tensors from the reference EACSLayer constructor (seeded)."""
    from cst_ssm.modules.eacs import EACSLayer
    from cst_ssm.modules.event_gate import EventGate
    from cst_ssm.ops.spectral_init import BranchSpec
    torch.manual_seed(seed)
    layer = EACSLayer(H, BranchSpec("b", N, tmin, tmax), gate=EventGate(init_eps=0.12)).eval()
    with torch.no_grad():
        layer.log_dt_scale.normal_(0.0, 0.2)
        layer.D.normal_(0.0, 1.0)
        layer.obs_norm.running_mean.normal_(0.0, 0.1)
        layer.obs_norm.running_var.uniform_(0.5, 1.5)
    x = torch.randn(B, L, H)
    if dup_frames:
        # ablation_pareto.py-style duplicated frames: runs of identical features
        for l in range(1, L):
            if (l // 3) % 2 == 1:
                x[:, l] = x[:, l - 1]
    t = timestamps_exp(torch.Generator().manual_seed(seed + 1), B, L)
    with torch.no_grad():
        u, Bc, Cc = layer._project(layer.norm(x))
        if ramp:
            # Residual spikes for robust_guard: with a large running mean the
            # residual scales with |u - y_hat|, so observations that grow
            # geometrically over runs of 6 frames make r double step after step.
            layer.obs_norm.running_mean.fill_(20.0)
            v = torch.randn(B, 1, H)
            k = (torch.arange(L) % 6).view(1, L, 1).float()
            u = v * 0.05 * (2.6 ** k) + 0.01 * torch.randn(B, L, H)
    return layer, u, Bc, Cc, t


def _run_scan_range(layer, u, Bc, Cc, t, eps=None, robust=None):
    from cst_ssm.modules.eacs import scan_range
    lam = layer.lam().to(torch.complex64)
    p = layer.step_params(lam)
    if eps is not None:
        p.eps = torch.tensor(float(eps))
    state = (torch.zeros(u.shape[0], layer.H, layer.N, dtype=torch.complex64),
             t[:, 0] - layer.dt_init, u[:, 0], Bc[:, 0], Cc[:, 0])
    with torch.no_grad():
        ys, gs, rs, ns, _ = scan_range(p, state, u, Bc, Cc, t, 0, u.shape[1],
                                       robust=robust, skip_compute=robust is None)
    return ys, gs, rs


def _spike_hits(rs, robust):
    """Number of steps whose threshold robust_guard lowered (eacs.py:155-170)."""
    if robust is None:
        return 0
    hits = 0
    for row in rs:
        spike, prev = 0.0, None
        for r in row.tolist():
            if spike >= robust.k:
                hits += 1
            if prev is not None:
                spike = spike + 1.0 if r > prev * robust.spike_ratio else 0.0
            prev = r
    return hits


def _calibrate(layer, u, Bc, Cc, t, rate, robust=None, margin=2e-4):
    """Bisect eps for a target update rate, then nudge it so no residual sits
    within margin of the threshold (the gate comparison stays unambiguous)."""
    _, _, rs = _run_scan_range(layer, u, Bc, Cc, t, eps=0.0, robust=robust)
    lo, hi = 0.0, float(rs.max()) * 4
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        _, gs, _ = _run_scan_range(layer, u, Bc, Cc, t, eps=mid, robust=robust)
        if float(gs.mean()) > rate:
            lo = mid
        else:
            hi = mid
    eps = 0.5 * (lo + hi)
    for _ in range(200):
        ys, gs, rs = _run_scan_range(layer, u, Bc, Cc, t, eps=eps, robust=robust)
        gap = (rs - eps).abs()
        if robust is not None:
            gap = torch.minimum(gap, (rs - eps * robust.eps_factor).abs())
        if float(gap.min()) > margin:
            return eps, ys, gs, rs
        eps *= 1.0 + 3 * margin
    raise RuntimeError("could not calibrate eps away from residuals")


def cell_cases():
    from cst_ssm.modules.eacs import RobustCfg
    out = {}
    specs = {
        # name: (H, N, tau_min, tau_max, B, L, seed, target update rate, robust, dup, ramp)
        "cell_commit": (48, 16, 0.5, 4.0, 2, 64, 0, None, None, False, False),
        "cell_wide": (256, 16, 0.5, 64.0, 2, 40, 1, None, None, False, False),
        "cell_skip50": (48, 16, 0.5, 4.0, 2, 64, 2, 0.5, None, True, False),
        "cell_skip30": (40, 8, 4.0, 32.0, 3, 48, 3, 0.3, None, True, False),
        "cell_skip70": (33, 5, 32.0, 256.0, 2, 40, 4, 0.7, None, False, False),
        "cell_n32": (24, 32, 0.5, 64.0, 2, 36, 5, 0.4, None, True, False),
        "cell_robust": (32, 16, 0.5, 4.0, 2, 64, 6, 0.6, (3, 2.0, 0.3), False, True),
        "cell_robust_k1": (32, 8, 0.5, 4.0, 2, 64, 7, 0.55, (1, 1.05, 0.5), True, False),
        "cell_l1": (16, 4, 0.5, 4.0, 2, 1, 8, None, None, False, False),
    }
    for name, (H, N, tmin, tmax, B, L, seed, q, rb, dup, ramp) in specs.items():
        layer, u, Bc, Cc, t = _layer_inputs(H, N, tmin, tmax, B, L, seed, dup, ramp)
        robust = None if rb is None else RobustCfg(*rb)
        if q is None:
            eps = float(layer.gate.eps.detach())
            ys, gs, rs = _run_scan_range(layer, u, Bc, Cc, t, robust=robust)
        else:
            eps, ys, gs, rs = _calibrate(layer, u, Bc, Cc, t, q, robust=robust)
        d = dict(lam=_np(layer.lam()), log_dt=_np(layer.log_dt_scale), u=_np(u), Bc=_np(Bc),
                 Cc=_np(Cc), t=_np(t), D=_np(layer.D), mean=_np(layer.obs_norm.running_mean),
                 var=_np(layer.obs_norm.running_var),
                 scalars=np.array([eps, layer.gate.norm_eta, layer.obs_norm.eps, layer.dt_init,
                                   1e-3, layer.dt_max], np.float64),
                 robust=np.array([-1, 0, 0] if rb is None else rb, np.float64),
                 y=_np(ys), gate=_np(gs), resid=_np(rs))
        out[name] = d
        print(f"{name}: update rate {float(gs.mean()):.3f}, "
              f"min|r-eps| {float((rs - eps).abs().min()):.2e}, "
              f"robust-lowered steps {_spike_hits(rs, robust)}")
    return out


def train_cases():
    from cst_ssm.ops.eacs_cell_train import GatedEACSCellFunction
    out = {}
    specs = {
        # name: (H, N, B, L, seed, gate_mode, T, target update rate)
        "train_ste": (6, 4, 2, 12, 10, "ste", 0.5, 0.5),
        "train_ste_commit": (8, 4, 2, 10, 11, "ste", 0.3, None),
        "train_soft": (5, 3, 2, 9, 12, "soft", 0.4, 0.5),
    }
    for name, (H, N, B, L, seed, mode, T, q) in specs.items():
        layer, u, Bc, Cc, t = _layer_inputs(H, N, 0.5, 4.0, B, L, seed, dup_frames=True)
        if q is None:
            eps_v = float(layer.gate.eps.detach())
        else:
            eps_v, _, _, _ = _calibrate(layer, u, Bc, Cc, t, q)
        g = torch.Generator().manual_seed(seed + 100)
        lam = layer.lam().detach().to(torch.complex64).requires_grad_(True)
        log_dt = layer.log_dt_scale.detach().clone().requires_grad_(True)
        D = layer.D.detach().clone().requires_grad_(True)
        eps = torch.tensor(eps_v).requires_grad_(True)
        u_ = u.clone().requires_grad_(True)
        Bc_ = Bc.clone().requires_grad_(True)
        Cc_ = Cc.clone().requires_grad_(True)
        t_ = t.clone().requires_grad_(True)
        mean = layer.obs_norm.running_mean.detach()
        var = layer.obs_norm.running_var.detach()
        ys, gs, rs, ns = GatedEACSCellFunction.apply(
            u_, Bc_, Cc_, t_, lam, log_dt, D, eps, mean, var, T, layer.gate.norm_eta,
            layer.obs_norm.eps, layer.dt_init, mode, False, layer.dt_max)
        gy = torch.randn(ys.shape, generator=g)
        ggs = torch.randn(gs.shape, generator=g)
        grs = torch.randn(rs.shape, generator=g)
        gns = torch.randn(ns.shape, generator=g)
        grads = torch.autograd.grad([ys, gs, rs, ns], [u_, Bc_, Cc_, t_, lam, log_dt, D, eps],
                                    [gy, ggs, grs, gns])
        names = ["du", "dBc", "dCc", "dt", "dlam", "dlog_dt", "dD", "deps"]
        d = dict(lam=_np(lam), log_dt=_np(log_dt), u=_np(u), Bc=_np(Bc), Cc=_np(Cc), t=_np(t),
                 D=_np(D), mean=_np(mean), var=_np(var),
                 scalars=np.array([eps_v, layer.gate.norm_eta, layer.obs_norm.eps,
                                   layer.dt_init, 1e-3, layer.dt_max, T], np.float64),
                 gate_mode=np.array([0 if mode == "ste" else 1]),
                 y=_np(ys), gate=_np(gs), resid=_np(rs), innov=_np(ns),
                 gy=_np(gy), ggs=_np(ggs), grs=_np(grs), gns=_np(gns))
        for k, v in zip(names, grads):
            d[k] = _np(v)
        out[name] = d
        print(f"{name}: update rate {float(gs.mean()):.3f}")
    return out


def query_cases():
    """EACSLayer.run_with_commits (eacs.py:404-439) and readout_from_commits
    (continuous_query.py:20-61) on seeded layers, eval mode.  The layer's
    proj_out is set to the identity so the readout is the core's value."""
    from cst_ssm.modules.continuous_query import readout_from_commits
    out = {}
    specs = {
        # name: (H, N, tau_min, tau_max, B, L, Q, seed, target update rate)
        "query_skip": (24, 8, 0.5, 4.0, 2, 40, 29, 20, 0.5),
        "query_commit": (16, 16, 0.5, 64.0, 2, 24, 17, 21, None),
        "query_n5": (12, 5, 4.0, 32.0, 3, 19, 11, 22, 0.3),
    }
    for name, (H, N, tmin, tmax, B, L, Q, seed, q) in specs.items():
        layer, u, Bc, Cc, t = _layer_inputs(H, N, tmin, tmax, B, L, seed, dup_frames=True)
        torch.manual_seed(seed + 7)
        x = torch.randn(B, L, H)
        for l in range(1, L):
            if (l // 3) % 2 == 1:
                x[:, l] = x[:, l - 1]
        with torch.no_grad():
            u, Bc, Cc = layer._project(layer.norm(x))
            layer.proj_out.weight.copy_(torch.eye(H))
            layer.proj_out.bias.zero_()
        eps = float(layer.gate.eps.detach()) if q is None else _calibrate(layer, u, Bc, Cc, t, q)[0]
        orig = layer.step_params

        def step_params(lam, _orig=orig, _eps=eps):
            p = _orig(lam)
            p.eps = torch.tensor(_eps)
            return p

        layer.step_params = step_params
        g = torch.Generator().manual_seed(seed + 50)
        # queries: inside segments, on frames, before the first and after the last frame
        tq = t[:, :1] - 0.3 + (t[:, -1:] - t[:, :1] + 0.8) * torch.rand(B, Q, generator=g)
        tq[:, 0] = t[:, 0] - 0.2
        tq[:, 1] = t[:, 5]
        tq[:, 2] = t[:, -1] + 0.4
        tq = tq.sort(dim=1).values
        with torch.no_grad():
            res, commits = layer.run_with_commits(x, t)
            yq = readout_from_commits(layer, commits, tq)
            yf = readout_from_commits(layer, commits, commits["frame_t"])
        d = dict(lam=_np(layer.lam()), log_dt=_np(layer.log_dt_scale), u=_np(u), Bc=_np(Bc),
                 Cc=_np(Cc), t=_np(t), D=_np(layer.D), mean=_np(layer.obs_norm.running_mean),
                 var=_np(layer.obs_norm.running_var),
                 scalars=np.array([eps, layer.gate.norm_eta, layer.obs_norm.eps, layer.dt_init,
                                   1e-3, layer.dt_max], np.float64),
                 y=_np(res.y - x), gate=_np(res.gates), resid=_np(res.residual),
                 ch=_np(commits["h"]), ct=_np(commits["t"]), cu=_np(commits["u"]),
                 cB=_np(commits["B"]), cC=_np(commits["C"]), t_query=_np(tq), yq=_np(yq),
                 yf=_np(yf))
        out[name] = d
        print(f"{name}: update rate {float(res.gates.mean()):.3f}, "
              f"min|r-eps| {float((res.residual - eps).abs().min()):.2e}")
    return out


def qtrain_cases():
    """Training through per-frame commits: EACSLayer._commit_range
    (eacs.py:386-401) in training mode (STE or soft gate, event_gate.py:84-105)
    followed by readout_from_commits (continuous_query.py:20-54) at query
    times and at the frame times, differentiated by autograd with respect to
    the op-boundary tensors (u, B, C, t, lam, log_dt_scale, D, eps, the query
    times).  proj_out is the identity, so the readouts are the core's values."""
    from cst_ssm.modules.continuous_query import readout_from_commits
    out = {}
    specs = {
        # name: (H, N, B, L, Q, seed, use_ste, temperature, target update rate)
        "qtrain_ste": (6, 4, 2, 12, 9, 30, True, 0.5, 0.5),
        "qtrain_soft": (5, 3, 2, 10, 7, 31, False, 0.4, 0.5),
        "qtrain_commit": (8, 4, 2, 9, 6, 32, True, 0.3, None),
    }
    for name, (H, N, B, L, Q, seed, ste, T, q) in specs.items():
        layer, u, Bc, Cc, t = _layer_inputs(H, N, 0.5, 4.0, B, L, seed, dup_frames=True)
        eps_v = float(layer.gate.eps.detach()) if q is None else _calibrate(layer, u, Bc, Cc, t, q)[0]
        with torch.no_grad():
            layer.proj_out.weight.copy_(torch.eye(H))
            layer.proj_out.bias.zero_()
        layer.train()
        layer.gate.use_ste = ste
        layer.gate.set_temperature(T)
        eps = torch.tensor(eps_v).requires_grad_(True)
        orig = layer.step_params

        def step_params(lam, _orig=orig, _eps=eps):
            p = _orig(lam)
            p.eps = _eps
            return p

        layer.step_params = step_params
        g = torch.Generator().manual_seed(seed + 100)
        tq = t[:, :1] - 0.3 + (t[:, -1:] - t[:, :1] + 0.8) * torch.rand(B, Q, generator=g)
        tq[:, 0] = t[:, 0] - 0.2
        tq[:, 1] = t[:, 4]
        tq[:, 2] = t[:, -1] + 0.4
        tq = tq.sort(dim=1).values
        lam = layer.lam().detach().to(torch.complex64).requires_grad_(True)
        u_, Bc_, Cc_, t_, tq_ = (x.clone().requires_grad_(True) for x in (u, Bc, Cc, t, tq))
        state = (torch.zeros(B, H, N, dtype=torch.complex64), t_[:, 0] - layer.dt_init,
                 u_[:, 0], Bc_[:, 0], Cc_[:, 0])
        ys, gs, rs, Hc, Tc, Uc, Bs, Cs = layer._commit_range(lam, state, u_, Bc_, Cc_, t_, 0, L)
        commits = dict(h=Hc, t=Tc, u=Uc, B=Bs, C=Cs, lam=lam, frame_t=t_,
                       log_dt_scale=layer.log_dt_scale, dt_max=layer.dt_max)
        yq = readout_from_commits(layer, commits, tq_)
        yf = readout_from_commits(layer, commits, commits["frame_t"])
        up = [torch.randn(x.shape, generator=g) for x in (ys, gs, rs, yq, yf)]
        leaves = [u_, Bc_, Cc_, t_, lam, layer.log_dt_scale, layer.D, eps, tq_]
        grads = torch.autograd.grad([ys, gs, rs, yq, yf], leaves, up)
        names = ["du", "dBc", "dCc", "dt", "dlam", "dlog_dt", "dD", "deps", "dtq"]
        d = dict(lam=_np(lam), log_dt=_np(layer.log_dt_scale), u=_np(u), Bc=_np(Bc), Cc=_np(Cc),
                 t=_np(t), D=_np(layer.D), mean=_np(layer.obs_norm.running_mean),
                 var=_np(layer.obs_norm.running_var),
                 scalars=np.array([eps_v, layer.gate.norm_eta, layer.obs_norm.eps, layer.dt_init,
                                   1e-3, layer.dt_max, T], np.float64),
                 gate_mode=np.array([0 if ste else 1]),
                 y=_np(ys), gate=_np(gs), resid=_np(rs), ch=_np(Hc), ct=_np(Tc), cu=_np(Uc),
                 cB=_np(Bs), cC=_np(Cs), t_query=_np(tq), yq=_np(yq), yf=_np(yf),
                 gy=_np(up[0]), ggs=_np(up[1]), grs=_np(up[2]), gq=_np(up[3]), gf=_np(up[4]))
        for k, v in zip(names, grads):
            d[k] = _np(v)
        out[name] = d
        print(f"{name}: update rate {float(gs.detach().round().mean()):.3f}, "
              f"min|r-eps| {float((rs.detach() - eps_v).abs().min()):.2e}")
    return out


def stream_cases():
    """temporal_step (streaming.py:45-85) on a one-branch MultiScaleEACS with
    proj_out = identity and out_norm removed, so each step's output is
    x + y_core on valid rows; the per-step projections are recomputed with
    the same calls temporal_step makes."""
    from torch import nn
    from cst_ssm.modules.multiscale import MultiScaleEACS
    from cst_ssm.modules.streaming import initial_states, temporal_step
    from cst_ssm.ops.spectral_init import BranchSpec
    out = {}
    specs = {
        # name: (H, N, B, K, seed, init_eps, cpi_modulation, soft gate (train, no STE), T)
        "stream_hard": (24, 8, 3, 14, 30, 0.6, 0.0, False, 0.1),
        "stream_cpi": (16, 16, 2, 12, 31, 0.6, 0.5, False, 0.1),
        "stream_soft": (12, 5, 2, 10, 32, 0.6, 0.0, True, 0.3),
    }
    for name, (H, N, B, K, seed, e0, m, soft, T) in specs.items():
        torch.manual_seed(seed)
        temporal = MultiScaleEACS(H, branches=[BranchSpec("s", N, 0.5, 4.0)],
                                  gate_kwargs=dict(init_eps=e0, eps_max=3.0, cpi_modulation=m,
                                                   use_ste=not soft, temperature=T))
        br = temporal.branches[0]
        with torch.no_grad():
            br.log_dt_scale.normal_(0.0, 0.2)
            br.D.normal_(0.0, 1.0)
            br.obs_norm.running_mean.normal_(0.0, 0.1)
            br.obs_norm.running_var.uniform_(0.5, 1.5)
            br.proj_out.weight.copy_(torch.eye(H))
            br.proj_out.bias.zero_()
        temporal.out_norm = nn.Identity()
        temporal.train(soft)
        x = torch.randn(B, K, H)
        for k in range(1, K):
            if k % 4 == 2:  # repeated frames: small residuals, skipped steps
                x[:, k] = x[:, k - 1]
        t = timestamps_exp(torch.Generator().manual_seed(seed + 1), B, K)
        t[:, 5] = t[:, 4]
        valid = torch.ones(B, K, dtype=torch.bool)
        valid[1, :3] = False   # row 1 starts late: its first valid step commits
        valid[0, 6] = False
        valid[-1, K - 2] = False
        cpi = torch.rand(B, K) * 1.4 - 0.2 if m > 0 else None
        states = initial_states(temporal, B, "cpu")
        mid = K // 2
        ys, gs, rs, ns, us, Bs, Cs, st_mid = [], [], [], [], [], [], [], None
        with torch.no_grad():
            for k in range(K):
                xk = x[:, k]
                u_k, B_k, C_k = br._project(br.norm(xk))
                us.append(u_k); Bs.append(B_k); Cs.append(C_k)
                y, g, r, n, w, states = temporal_step(temporal, xk, t[:, k], states, valid[:, k],
                                                      None if cpi is None else cpi[:, k])
                ys.append(torch.where(valid[:, k, None], y - xk, torch.zeros_like(y)))
                gs.append(g[:, 0]); rs.append(r[:, 0]); ns.append(n[:, 0])
                if k == mid - 1:
                    st_mid = states[0]
        st = states[0]
        eps = float(br.gate.eps.detach())
        rr = torch.stack(rs, 1)
        print(f"{name}: eps {eps:.4f}, gate mean {float(torch.stack(gs, 1).mean()):.3f}, "
              f"min|r-eps| {float((rr[torch.stack(gs, 1) < 2] - eps).abs().min()):.2e}")
        d = dict(lam=_np(br.lam()), log_dt=_np(br.log_dt_scale), D=_np(br.D),
                 mean=_np(br.obs_norm.running_mean), var=_np(br.obs_norm.running_var),
                 u=_np(torch.stack(us, 1)), Bc=_np(torch.stack(Bs, 1)), Cc=_np(torch.stack(Cs, 1)),
                 t=_np(t), valid=valid.numpy().astype(np.uint8),
                 scalars=np.array([eps, br.gate.norm_eta, br.obs_norm.eps, br.dt_init, 1e-3,
                                   br.dt_max, m, T, 1.0 if soft else 0.0, mid], np.float64),
                 y=_np(torch.stack(ys, 1)), gate=_np(torch.stack(gs, 1)), resid=_np(rr),
                 innov=_np(torch.stack(ns, 1)),
                 h=_np(st.h), st_t=_np(st.t), st_u=_np(st.u), st_B=_np(st.B), st_C=_np(st.C),
                 st_init=st.initialized.numpy().astype(np.uint8),
                 mid_h=_np(st_mid.h), mid_t=_np(st_mid.t), mid_u=_np(st_mid.u),
                 mid_B=_np(st_mid.B), mid_C=_np(st_mid.C),
                 mid_init=st_mid.initialized.numpy().astype(np.uint8))
        if cpi is not None:
            d["cpi"] = _np(cpi)
        out[name] = d
    return out


def sgrad_cases():
    """temporal_step (streaming.py:45-85) over K steps under autograd, on a
    one-branch MultiScaleEACS whose projections return op-boundary leaves
    (u, B, C per step), whose lam() returns a leaf and whose gate threshold is
    a leaf, with proj_out = identity, out_norm removed and x = 0, so each
    step's output is the core's y on valid rows.  Gradients of a weighted sum
    of every step's outputs (y, gate, resid, innov) and the final state with
    respect to the per-step inputs (u, B, C, t, cpi), the initial state (h, t,
    u, B, C; rows 0 and 2 start initialised, row 1 does not) and lam,
    log_dt_scale, D, eps."""
    from torch import nn
    from cst_ssm.modules.event_gate import EventGate
    from cst_ssm.modules.multiscale import MultiScaleEACS
    from cst_ssm.modules.streaming import BranchState, temporal_step
    from cst_ssm.ops.spectral_init import BranchSpec
    out = {}
    specs = {
        # name: (H, N, B, K, seed, init_eps, cpi_modulation, mode, T)
        "sgrad_ste": (12, 8, 3, 6, 40, 0.7, 0.0, "ste", 0.2),
        "sgrad_cpi": (10, 4, 3, 5, 41, 0.7, 0.5, "ste", 0.2),
        "sgrad_soft": (8, 5, 3, 5, 42, 0.7, 0.0, "soft", 0.3),
        "sgrad_eval": (12, 8, 3, 6, 43, 0.7, 0.0, "eval", 0.2),
    }
    for name, (H, N, B, K, seed, e0, m, mode, T) in specs.items():
        torch.manual_seed(seed)
        temporal = MultiScaleEACS(H, branches=[BranchSpec("s", N, 0.5, 4.0)],
                                  gate_kwargs=dict(init_eps=e0, eps_max=3.0, cpi_modulation=m,
                                                   use_ste=mode != "soft", temperature=T))
        br = temporal.branches[0]
        with torch.no_grad():
            br.log_dt_scale.normal_(0.0, 0.2)
            br.D.normal_(0.0, 1.0)
            br.obs_norm.running_mean.normal_(0.0, 0.1)
            br.obs_norm.running_var.uniform_(0.5, 1.5)
            br.proj_out.weight.copy_(torch.eye(H))
            br.proj_out.bias.zero_()
        temporal.out_norm = nn.Identity()
        br.norm = nn.Identity()
        temporal.train(mode != "eval")
        g = torch.Generator().manual_seed(seed + 1)
        lam = br.lam().detach().to(torch.complex64).requires_grad_(True)
        br.lam = lambda _l=lam: _l
        eps = torch.tensor(float(br.gate.eps.detach())).requires_grad_(True)

        eps_leaf = eps

        class Gate(EventGate):
            @property
            def eps(self):
                return eps_leaf
        br.gate.__class__ = Gate
        s = 1 / math.sqrt(2 * N)
        u = torch.randn(B, K, H, generator=g)
        for k in range(1, K):
            if k % 3 == 2:  # repeated frames: small residuals, skipped steps
                u[:, k] = u[:, k - 1] + 0.02 * torch.randn(B, H, generator=g)
        Bc = torch.complex(torch.randn(B, K, N, generator=g), torch.randn(B, K, N, generator=g)) * s
        Cc = torch.complex(torch.randn(B, K, N, generator=g), torch.randn(B, K, N, generator=g)) * s
        t = 1.0 + timestamps_exp(g, B, K)
        cpi = (torch.rand(B, K, generator=g) * 1.4 - 0.2) if m > 0 else None
        valid = torch.ones(B, K, dtype=torch.bool)
        valid[1, :2] = False   # row 1 starts late
        valid[0, 3] = False
        valid[2, K - 1] = False
        init = torch.tensor([True, False, True])
        h0 = torch.complex(torch.randn(B, H, N, generator=g), torch.randn(B, H, N, generator=g)) * 0.3
        st0 = [h0, torch.rand(B, generator=g) * 0.5, torch.randn(B, H, generator=g),
               torch.complex(torch.randn(B, N, generator=g), torch.randn(B, N, generator=g)) * s,
               torch.complex(torch.randn(B, N, generator=g), torch.randn(B, N, generator=g)) * s]
        leaves = [x.clone().requires_grad_(True) for x in [u, Bc, Cc, t] + ([cpi] if cpi is not None else [])
                  + st0]
        u_, Bc_, Cc_, t_ = leaves[:4]
        cpi_ = leaves[4] if cpi is not None else None
        sl = leaves[-5:]
        states = [BranchState(*sl, init.clone())]
        outs, ups = [], []
        x0 = torch.zeros(B, H)
        rec = dict(gate=[], resid=[], innov=[], y=[])
        for k in range(K):
            br._project = lambda xn, _k=k: (u_[:, _k], Bc_[:, _k], Cc_[:, _k])
            y, gk, rk, nk, w, states = temporal_step(temporal, x0, t_[:, k], states, valid[:, k],
                                                     None if cpi_ is None else cpi_[:, k])
            for key, val in (("y", y), ("gate", gk[:, 0]), ("resid", rk[:, 0]), ("innov", nk[:, 0])):
                rec[key].append(val)
        for key in ("y", "gate", "resid", "innov"):
            v = torch.stack(rec[key], 1)
            outs.append(v)
            ups.append(torch.randn(v.shape, generator=g))
        fin = states[0]
        for v in (fin.h, fin.t, fin.u, fin.B, fin.C):
            outs.append(v)
            ups.append(torch.complex(torch.randn(v.shape, generator=g), torch.randn(v.shape, generator=g))
                       if v.is_complex() else torch.randn(v.shape, generator=g))
        wrt = leaves + [lam, br.log_dt_scale, br.D, eps]
        live = [(o, w) for o, w in zip(outs, ups) if o.requires_grad]  # eval: the gate is a constant
        grads = torch.autograd.grad([o for o, _ in live], wrt, [w for _, w in live], allow_unused=True)
        names = ["du", "dBc", "dCc", "dt"] + (["dcpi"] if cpi is not None else []) + \
            ["dh0", "dt0", "du0", "dB0", "dC0", "dlam", "dlog_dt", "dD", "deps"]
        gates = torch.stack(rec["gate"], 1).detach()
        rr = torch.stack(rec["resid"], 1).detach()
        print(f"{name}: gate mean {float(gates.mean()):.3f}, min|r-eps| "
              f"{float((rr - float(eps))[valid].abs().min()):.2e}")
        d = dict(lam=_np(lam), log_dt=_np(br.log_dt_scale), D=_np(br.D),
                 mean=_np(br.obs_norm.running_mean), var=_np(br.obs_norm.running_var),
                 u=_np(u), Bc=_np(Bc), Cc=_np(Cc), t=_np(t), valid=valid.numpy().astype(np.uint8),
                 h0=_np(st0[0]), t0=_np(st0[1]), u0=_np(st0[2]), B0=_np(st0[3]), C0=_np(st0[4]),
                 init0=init.numpy().astype(np.uint8),
                 scalars=np.array([float(eps), br.gate.norm_eta, br.obs_norm.eps, br.dt_init, 1e-3,
                                   br.dt_max, m, T], np.float64),
                 gate_mode=np.array([{"ste": 0, "soft": 1, "eval": 2}[mode]]),
                 y=_np(outs[0]), gate=_np(outs[1]), resid=_np(outs[2]), innov=_np(outs[3]),
                 fh=_np(fin.h), ft=_np(fin.t), fu=_np(fin.u), fB=_np(fin.B), fC=_np(fin.C),
                 gy=_np(ups[0]), gg=_np(ups[1]), gr=_np(ups[2]), gn=_np(ups[3]), gh=_np(ups[4]),
                 gt=_np(ups[5]), gu=_np(ups[6]), gB=_np(ups[7]), gC=_np(ups[8]))
        if cpi is not None:
            d["cpi"] = _np(cpi)
        for k, v in zip(names, grads):
            d[k] = np.zeros(1, np.float32) if v is None else _np(v)
        out[name] = d
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--groups", default="scan,ssm,cell,train,query,stream,qtrain,sgrad",
                    help="comma-separated groups to (re)write")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gen = torch.Generator().manual_seed(1234)
    makers = {"scan": lambda: scan_cases(gen), "ssm": lambda: ssm_cases(gen),
              "cell": cell_cases, "train": train_cases, "query": query_cases,
              "stream": stream_cases, "qtrain": qtrain_cases, "sgrad": sgrad_cases}
    want = args.groups.split(",")
    groups = {}
    for name in ("scan", "ssm", "cell", "train", "query", "stream", "qtrain", "sgrad"):  # fixed order: gen is shared
        cases = makers[name]()
        if name in want:
            groups[name] = cases
    for group, cases in groups.items():
        flat = {f"{case}/{k}": v for case, d in cases.items() for k, v in d.items()}
        path = os.path.join(HERE, f"{group}.npz")
        np.savez_compressed(path, **flat)
        print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
