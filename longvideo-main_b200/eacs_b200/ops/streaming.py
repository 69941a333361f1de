"""Streaming EACS steps with explicit branch state on B200.

Mirrors cst_ssm/modules/streaming.py:45-85 (temporal_step).  Per branch the
projections, proj_out, fusion and out_norm stay in torch (GEMMs and small
elementwise work); the cell step itself -- first-observation commit, valid
masks, CPI-modulated threshold, prediction, residual over H, gate, update,
readout and the new state -- is one kernel launch (eacs_stream_chunk) instead
of the reference's ~40 tensor operations.  `stream_chunk` runs K known steps
of one branch in one launch with the same semantics.

Inference path: no autograd through the state.  install(..., streaming=True)
binds `temporal_step` with a dispatcher that keeps the reference's own code
where gradients are needed or the tensors are on the CPU.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require


def _f32(x):
    return x.float().contiguous()


def _c64(x):
    return x.to(torch.complex64).contiguous()


@torch.no_grad()
def stream_chunk(lam, log_dt_scale, D, mean, var, u, Bc, Cc, t, valid, cpi, state, eps, eta,
                 var_eps=1e-5, dt_init=1.0, dt_min=1e-3, dt_max=1e3, cpi_modulation=0.0,
                 gate_mode="hard", temperature=0.1):
    """K steps of one branch from an explicit state.

    u (B,K,H), Bc/Cc (B,K,N), t (B,K), valid (B,K) bool or None, cpi (B,K) or
    None; state = (h (B,H,N), t (B), u (B,H), B (B,N), C (B,N), initialized (B)).
    Returns (y (B,K,H) before proj_out, gate, resid, innov (B,K), new state)."""
    h0, t0, u0, B0, C0, i0 = state
    dev = cuda_tensors("stream_chunk", lam, log_dt_scale, D, mean, var, u, Bc, Cc, t, h0, t0, u0,
                       B0, C0, i0)
    require(gate_mode in ("hard", "soft"), "stream_chunk: gate_mode must be 'hard' or 'soft'")
    B, K, H = u.shape
    N = lam.shape[1]
    require(Bc.shape == (B, K, N) and Cc.shape == (B, K, N) and t.shape == (B, K)
            and h0.shape == (B, H, N), "stream_chunk: shape mismatch")
    if u.dtype not in _lib.DTYPE_CODES:
        u = u.float()
    # every converted copy stays bound to a name until the launch is enqueued:
    # a temporary freed earlier could hand its memory to the next conversion
    u_c = u.contiguous()
    B_c, C_c, t_c = _c64(Bc), _c64(Cc), _f32(t)
    valid_c = None if valid is None else valid.to(torch.uint8).contiguous()
    cpi_c = None if cpi is None else _f32(cpi)
    ins = [_c64(lam), _f32(log_dt_scale), _f32(D), _f32(mean), _f32(var)]
    st_in = [_c64(h0), _f32(t0), _f32(u0), _c64(B0), _c64(C0), i0.to(torch.uint8).contiguous()]
    st_out = [torch.empty_like(x) for x in st_in]
    y = torch.empty(B, K, H, dtype=torch.float32, device=dev)
    g, r, n = (torch.empty(B, K, dtype=torch.float32, device=dev) for _ in range(3))
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().eacs_stream_chunk(
            *[x.data_ptr() for x in ins], u_c.data_ptr(), _lib.DTYPE_CODES[u_c.dtype],
            B_c.data_ptr(), C_c.data_ptr(), t_c.data_ptr(), _lib.ptr(valid_c),
            _lib.ptr(cpi_c), *[x.data_ptr() for x in st_in], *[x.data_ptr() for x in st_out],
            y.data_ptr(), g.data_ptr(), r.data_ptr(), n.data_ptr(), float(eps), float(eta),
            float(var_eps), float(dt_init), float(dt_min), float(dt_max), float(cpi_modulation),
            1 if gate_mode == "soft" else 0, float(temperature), B, K, H, N,
            _lib.stream_ptr(dev)), "eacs_stream_chunk")
    h1, t1, u1, B1, C1, i1 = st_out
    return y, g, r, n, (h1, t1, u1, B1, C1, i1.bool())


def _gate_mode(br) -> str:
    return "soft" if (br.training and not br.gate.use_ste) else "hard"


@torch.no_grad()
def temporal_step(temporal, x: Tensor, t: Tensor, states: list, valid: Tensor,
                  cpi: Tensor | None = None):
    """streaming.py:45-85: one observation for every branch; returns
    (y, gates (B,S), resid, innov, fusion weights, new states)."""
    ys, gs, rs, ns, new = [], [], [], [], []
    vb = valid.bool()
    for br, state in zip(temporal.branches, states):
        if br.robust_guard:
            raise ValueError("streaming CPIB does not support robust_guard; disable it explicitly")
        u, Bc, Cc = br._project(br.norm(x))
        if bool((vb & state.initialized & (t < state.t)).any()):
            raise ValueError("timestamps must not precede the last committed observation")
        st = (state.h, state.t, state.u, state.B, state.C, state.initialized)
        y, g, r, n, st1 = stream_chunk(
            br.lam(), br.log_dt_scale, br.D, br.obs_norm.running_mean, br.obs_norm.running_var,
            u[:, None], Bc[:, None], Cc[:, None], t.float()[:, None], vb[:, None],
            None if cpi is None else cpi.float()[:, None], st, float(br.gate.eps.item()),
            br.gate.norm_eta, br.obs_norm.eps, br.dt_init, 1e-3, float(br.dt_max),
            float(br.gate.cpi_modulation) if cpi is not None else 0.0, _gate_mode(br),
            float(br.gate.temperature))
        new.append(type(state)(*st1))
        delta = br.proj_out(y[:, 0].to(x.dtype))
        ys.append(delta * vb[:, None])
        gs.append(g[:, 0])
        rs.append(r[:, 0])
        ns.append(n[:, 0])
    weights = temporal.fusion(x).softmax(-1)
    fused = (torch.stack(ys, -1) * weights[:, None, :]).sum(-1)
    y = temporal.out_norm(x + fused) * vb[:, None]
    return y, torch.stack(gs, 1), torch.stack(rs, 1), torch.stack(ns, 1), weights, new


def streaming_fusable(temporal, x: Tensor, states) -> bool:
    if not x.is_cuda:
        return False
    for br in temporal.branches:
        if br.disc_mode != "continuous" or getattr(br.gate, "gate_kind", "event") != "event":
            return False
    if torch.is_grad_enabled():
        if x.requires_grad or any(p.requires_grad for p in temporal.parameters()):
            return False
        if any(s.h.requires_grad or s.u.requires_grad for s in states):
            return False
    return True


def make_temporal_step(original):
    def dispatch(temporal, x, t, states, valid, cpi=None):
        if streaming_fusable(temporal, x, states):
            return temporal_step(temporal, x, t, states, valid, cpi)
        return original(temporal, x, t, states, valid, cpi)
    dispatch.__wrapped__ = original
    return dispatch
