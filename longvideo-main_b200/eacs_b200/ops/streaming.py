"""Streaming EACS steps with explicit branch state on B200.

Mirrors cst_ssm/modules/streaming.py:45-85 (temporal_step).  Per branch the
projections, proj_out, fusion and out_norm stay in torch (GEMMs and small
elementwise work); the cell step itself -- first-observation commit, valid
masks, CPI-modulated threshold, prediction, residual over H, gate, update,
readout and the new state -- is one kernel launch (eacs_stream_chunk) instead
of the reference's ~40 tensor operations.  `stream_chunk` runs K known steps
of one branch in one launch with the same semantics.

Under autograd each branch's step is `StreamStepFunction` (forward: the
same kernel with K = 1; backward: eacs_stream_step_bwd, one launch per row
and branch plus a parameter sum), so gradients flow through the state from
step to step as in the reference's per-step autograd graph.
install(..., streaming=True) binds `temporal_step` with a dispatcher that
keeps the reference's own code only for CPU tensors, non-event gates and
non-continuous discretisation.
"""
from __future__ import annotations

import ctypes

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
    """The branch gate's forward kind: "soft" (training without STE) or "hard"."""
    return "soft" if (br.training and not br.gate.use_ste) else "hard"


def _grad_mode(br) -> str:
    """Its backward kind: "ste" / "soft" in training, "hard" (no gradient
    through r > eps) in eval (event_gate.py:98-105)."""
    if not br.training:
        return "hard"
    return "ste" if br.gate.use_ste else "soft"


_GRAD_MODES = {"ste": 0, "soft": 1, "hard": 2}


class StreamStepFunction(torch.autograd.Function):
    """One streaming step of one branch under autograd (the per-branch body of
    temporal_step, streaming.py:55-80): (y before proj_out, gate, resid,
    innov, h', t', u', B', C', initialized') from the frame (u, B, C, t, cpi),
    the state and the parameters.  The backward is eacs_stream_step_bwd."""

    @staticmethod
    def forward(ctx, u, Bc, Cc, t, cpi, h, st_t, st_u, st_B, st_C, lam, log_dt, D, eps, init, valid,
                mean, var, hp):
        ctx.set_materialize_grads(False)
        eta, var_eps, dt_init, dt_min, dt_max, cpi_mod, mode, T = hp[:8]
        eps_v = hp[8] if len(hp) > 8 else float(eps)  # the threshold's value, when the caller has it
        st = (h, st_t, st_u, st_B, st_C, init)
        y, g, r, n, st1 = stream_chunk(
            lam, log_dt, D, mean, var, u.float()[:, None], Bc[:, None], Cc[:, None], t.float()[:, None],
            None if valid is None else valid[:, None], None if cpi is None else cpi.float()[:, None], st,
            eps_v, eta, var_eps, dt_init, dt_min, dt_max, cpi_mod, "soft" if mode == "soft" else "hard", T)
        h1, t1, u1, B1, C1, i1 = st1
        ctx.mark_non_differentiable(i1)
        keep = [u.float().contiguous(), _c64(Bc), _c64(Cc), _f32(t), None if cpi is None else _f32(cpi),
                _c64(h), _f32(st_t), _f32(st_u), _c64(st_B), _c64(st_C), _c64(lam), _f32(log_dt), _f32(D),
                _f32(mean), _f32(var), init.to(torch.uint8).contiguous(),
                None if valid is None else valid.to(torch.uint8).contiguous(), g[:, 0].contiguous()]
        ctx.keep = keep
        ctx.hp = (eps_v, float(eta), float(var_eps), float(dt_init), float(dt_min), float(dt_max),
                  float(cpi_mod), _GRAD_MODES[mode], float(T))
        ctx.dtypes = (u.dtype, Bc.dtype, Cc.dtype, t.dtype, None if cpi is None else cpi.dtype, h.dtype,
                      st_t.dtype, st_u.dtype, st_B.dtype, st_C.dtype, lam.dtype, log_dt.dtype, D.dtype,
                      eps.dtype if torch.is_tensor(eps) else None, eps.shape if torch.is_tensor(eps) else None)
        return y[:, 0], g[:, 0], r[:, 0], n[:, 0], h1, t1, u1, B1, C1, i1

    @staticmethod
    def backward(ctx, gy, gg, gr, gn, gh, gt, gu, gB, gC, _gi):
        (u, Bc, Cc, t, cpi, h, st_t, st_u, st_B, st_C, lam, log_dt, D, mean, var, init, valid,
         gate) = ctx.keep
        eps, eta, var_eps, dt_init, dt_min, dt_max, cpi_mod, mode, T = ctx.hp
        dev = u.device
        B, H = u.shape
        N = lam.shape[1]
        f = lambda x: None if x is None else x.float().contiguous()  # noqa: E731
        c = lambda x: None if x is None else x.to(torch.complex64).contiguous()  # noqa: E731
        ups = [f(gy), f(gg), f(gr), f(gn), c(gh), f(gt), f(gu), c(gB), c(gC)]
        f32 = dict(dtype=torch.float32, device=dev)
        c64 = dict(dtype=torch.complex64, device=dev)
        out = [torch.empty(B, H, **f32), torch.empty(B, N, **c64), torch.empty(B, N, **c64),
               torch.empty(B, **f32), None if cpi is None else torch.empty(B, **f32),
               torch.empty(B, H, N, **c64), torch.empty(B, **f32), torch.empty(B, H, **f32),
               torch.empty(B, N, **c64), torch.empty(B, N, **c64), torch.empty(H, N, **c64),
               torch.empty(H, **f32), torch.empty(H, **f32), torch.empty(1, **f32)]
        L_ = _lib.lib()
        ws = torch.empty(int(L_.eacs_stream_step_bwd_workspace_size(B, H, N)), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            _lib.check(L_.eacs_stream_step_bwd(
                lam.data_ptr(), log_dt.data_ptr(), D.data_ptr(), mean.data_ptr(), var.data_ptr(), u.data_ptr(),
                Bc.data_ptr(), Cc.data_ptr(), t.data_ptr(), _lib.ptr(valid), _lib.ptr(cpi), h.data_ptr(),
                st_t.data_ptr(), st_u.data_ptr(), st_B.data_ptr(), st_C.data_ptr(), init.data_ptr(),
                gate.data_ptr(), *[_lib.ptr(x) for x in ups], *[_lib.ptr(x) for x in out],
                ws.data_ptr(), ws.numel(), eps, eta, var_eps, dt_init, dt_min, dt_max, cpi_mod, mode, T,
                B, H, N, _lib.stream_ptr(dev)), "eacs_stream_step_bwd")
        dt_ = ctx.dtypes
        du, dBc, dCc, dt, dcpi, dh, dt_in, du_in, dB_in, dC_in, dlam, dlog, dD, deps = out
        grads = [du.to(dt_[0]), dBc.to(dt_[1]), dCc.to(dt_[2]), dt.to(dt_[3]),
                 None if dcpi is None else dcpi.to(dt_[4]), dh.to(dt_[5]), dt_in.to(dt_[6]),
                 du_in.to(dt_[7]), dB_in.to(dt_[8]), dC_in.to(dt_[9]), dlam.to(dt_[10]), dlog.to(dt_[11]),
                 dD.to(dt_[12]), None if dt_[13] is None else deps.to(dt_[13]).reshape(dt_[14])]
        return (*grads, None, None, None, None, None)


_EPS_CACHE: dict = {}
_SCALAR_CACHE: dict = {}


def host_float(x) -> float:
    """float(x) for a number; for a one-element tensor (a buffer such as the
    gate temperature) its value, read from the device only when the tensor
    changed since the last read (its version counter or storage)."""
    if not torch.is_tensor(x):
        return float(x)
    key = (x.data_ptr(), x._version)
    hit = _SCALAR_CACHE.get(id(x))
    if hit is None or hit[0] != key:
        hit = (key, float(x.detach()))
        _SCALAR_CACHE[id(x)] = hit
    return hit[1]


def eps_value(gate) -> float:
    """The gate threshold as a Python float, read from the device only when
    its parameters changed since the last read (EventGate.eps is
    eps_min + (eps_max - eps_min) sigmoid(eps_raw), times eps_anneal): a
    stream of frames then takes no host synchronisation for it."""
    raw, anneal = getattr(gate, "eps_raw", None), getattr(gate, "eps_anneal", None)
    if not (torch.is_tensor(raw) and torch.is_tensor(anneal)):
        return float(gate.eps)
    key = (raw._version, anneal._version, raw.data_ptr(), anneal.data_ptr(), gate.eps_min, gate.eps_max)
    hit = _EPS_CACHE.get(id(gate))
    if hit is None or hit[0] != key:
        hit = (key, float(gate.eps.detach()))
        _EPS_CACHE[id(gate)] = hit
    return hit[1]


def stream_step(br, u, Bc, Cc, t, valid, cpi, state, eps=None):
    """One step of branch `br` (an EACSLayer) from `state` (h, t, u, B, C,
    initialized): (y (B,H) before proj_out, gate, resid, innov, state').
    eps: the threshold (default: the branch gate's).  Differentiable where
    any input needs a gradient."""
    mode = _grad_mode(br)
    if eps is None:
        eps, eps_v = br.gate.eps, eps_value(br.gate)
    else:
        eps_v = float(eps)
    hp = (br.gate.norm_eta, br.obs_norm.eps, br.dt_init, 1e-3, host_float(br.dt_max),
          float(br.gate.cpi_modulation) if cpi is not None else 0.0, mode, host_float(br.gate.temperature), eps_v)
    lam = br.lam()
    h, st_t, st_u, st_B, st_C, init = state
    ins = (u, Bc, Cc, t, cpi, h, st_t, st_u, st_B, st_C, lam, br.log_dt_scale, br.D, eps)
    if torch.is_grad_enabled() and any(torch.is_tensor(x) and x.requires_grad for x in ins):
        y, g, r, n, h1, t1, u1, B1, C1, i1 = StreamStepFunction.apply(
            u, Bc, Cc, t, cpi, h, st_t, st_u, st_B, st_C, lam, br.log_dt_scale, br.D, eps, init, valid,
            br.obs_norm.running_mean, br.obs_norm.running_var, hp)
        return y, g, r, n, (h1, t1, u1, B1, C1, i1.bool())
    with torch.no_grad():
        y, g, r, n, st1 = stream_chunk(
            lam, br.log_dt_scale, br.D, br.obs_norm.running_mean, br.obs_norm.running_var, u[:, None],
            Bc[:, None], Cc[:, None], t.float()[:, None], None if valid is None else valid[:, None],
            None if cpi is None else cpi.float()[:, None], state, hp[8], *hp[:6], _gate_mode(br), hp[7])
    return y[:, 0], g[:, 0], r[:, 0], n[:, 0], st1


def _needs_grad_frame(temporal, x, t, states, cpi) -> bool:
    if not torch.is_grad_enabled():
        return False
    if any(torch.is_tensor(z) and z.requires_grad for z in (x, t, cpi)):
        return True
    if any(p.requires_grad for p in temporal.parameters()):
        return True
    return any(z.requires_grad for st in states for z in (st.h, st.t, st.u, st.B, st.C))


def temporal_step(temporal, x: Tensor, t: Tensor, states: list, valid: Tensor,
                  cpi: Tensor | None = None):
    """streaming.py:45-85: one observation for every branch; returns
    (y, gates (B,S), resid, innov, fusion weights, new states).  Without
    autograd a frame the fused path takes runs as eacs_stream_frame."""
    for br in temporal.branches:
        if br.robust_guard:
            raise ValueError("streaming CPIB does not support robust_guard; disable it explicitly")
    if not _needs_grad_frame(temporal, x, t, states, cpi) and frame_fusable(temporal, x, states):
        return temporal_step_frame(temporal, x, t, states, valid, cpi)
    ys, gs, rs, ns, new = [], [], [], [], []
    vb = valid.bool()
    # the reference checks each branch's state in turn; one check over all
    # branches (one host synchronisation) raises the same error
    bad = None
    for state in states:
        b = vb & state.initialized & (t < state.t)
        bad = b if bad is None else bad | b
    if bad is not None and bool(bad.any()):
        raise ValueError("timestamps must not precede the last committed observation")
    for br, state in zip(temporal.branches, states):
        u, Bc, Cc = br._project(br.norm(x))
        st = (state.h, state.t, state.u, state.B, state.C, state.initialized)
        y, g, r, n, st1 = stream_step(br, u, Bc, Cc, t.float(), vb, None if cpi is None else cpi.float(), st)
        new.append(type(state)(*st1))
        delta = br.proj_out(y.to(x.dtype))
        ys.append(delta * vb[:, None])
        gs.append(g)
        rs.append(r)
        ns.append(n)
    weights = temporal.fusion(x).softmax(-1)
    fused = (torch.stack(ys, -1) * weights[:, None, :]).sum(-1)
    y = temporal.out_norm(x + fused) * vb[:, None]
    return y, torch.stack(gs, 1), torch.stack(rs, 1), torch.stack(ns, 1), weights, new


_CP, _CF = ctypes.c_void_p, ctypes.c_float


class FrameBranch(ctypes.Structure):
    """EacsFrameBranch (include/eacs_b200.h): one branch's weights, cell
    parameters and state buffers for eacs_stream_frame."""
    _fields_ = ([("ln_w", _CP), ("ln_b", _CP), ("ln_eps", _CF)]
                + [(k, _CP) for k in ("wu", "bu", "wB", "bB", "wC", "bC", "wo", "bo",
                                      "lam", "log_dt", "D", "mean", "var")]
                + [(k, _CF) for k in ("eps", "eta", "var_eps", "dt_init", "dt_min", "dt_max",
                                      "cpi_modulation", "temperature")]
                + [("gate_mode", ctypes.c_int), ("H", ctypes.c_int), ("N", ctypes.c_int)]
                + [(k, _CP) for k in ("h_in", "t_in", "u_in", "B_in", "C_in", "init_in",
                                      "h_out", "t_out", "u_out", "B_out", "C_out", "init_out")])


def _f32_param(t) -> bool:
    return t is not None and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()


def frame_fusable(temporal, x: Tensor, states) -> bool:
    """Whether one frame can run as eacs_stream_frame: float32 CUDA rows
    (at most 8) of width d (B*d <= 51200), 1-4 continuous event-gate branches
    without robust_guard, float32 contiguous weights with LayerNorm affines."""
    if not (x.is_cuda and x.dim() == 2 and x.dtype == torch.float32 and 1 <= x.shape[0] <= 8
            and x.shape[0] * x.shape[1] <= 51200):
        return False
    if not 1 <= len(temporal.branches) <= 4:
        return False
    mods = [temporal.fusion, temporal.out_norm]
    if not isinstance(temporal.out_norm, torch.nn.LayerNorm):
        return False
    for br in temporal.branches:
        if (br.robust_guard or br.disc_mode != "continuous" or getattr(br.gate, "gate_kind", "event") != "event"
                or not isinstance(br.norm, torch.nn.LayerNorm) or br.N > 64):
            return False
        mods += [br.norm, br.proj_u, br.proj_B, br.proj_C, br.proj_out]
    return all(_f32_param(m.weight) and _f32_param(m.bias) for m in mods)


_LAM_CACHE: dict = {}


def _frame_lam(br) -> Tensor:
    """br.lam() as contiguous complex64, recomputed only when one of the
    layer's own parameters changed (without autograd the value is all that
    is needed)."""
    key = tuple((p.data_ptr(), p._version) for p in br.parameters(recurse=False))
    hit = _LAM_CACHE.get(id(br))
    if hit is None or hit[0] != key:
        hit = (key, br.lam().detach().to(torch.complex64).contiguous())
        _LAM_CACHE[id(br)] = hit
    return hit[1]


def temporal_step_frame(temporal, x: Tensor, t: Tensor, states: list, valid: Tensor,
                        cpi: Tensor | None = None):
    """temporal_step (streaming.py:45-85) for one frame without autograd, as
    eacs_stream_frame: S + 3 launches for the whole module (norms, projections,
    cell steps, proj_out, fusion, out_norm).  Same returns as temporal_step."""
    vb = valid.bool()
    B, d = x.shape
    S = len(temporal.branches)
    dev = x.device
    keep = [x.contiguous(), t.float().contiguous(), vb.contiguous().view(torch.uint8),
            None if cpi is None else cpi.float().contiguous()]
    arr = (FrameBranch * S)()
    new = []
    ptr = lambda z: None if z is None else z.data_ptr()  # noqa: E731
    for s, (br, st) in enumerate(zip(temporal.branches, states)):
        ins = [_frame_lam(br), _f32(br.log_dt_scale), _f32(br.D),
               _f32(br.obs_norm.running_mean), _f32(br.obs_norm.running_var),
               _c64(st.h), _f32(st.t), _f32(st.u), _c64(st.B), _c64(st.C),
               st.initialized.bool().contiguous().view(torch.uint8)]
        outs = [torch.empty_like(z) for z in ins[5:]]
        keep += ins + outs
        f = arr[s]
        f.ln_w, f.ln_b, f.ln_eps = br.norm.weight.data_ptr(), br.norm.bias.data_ptr(), float(br.norm.eps)
        f.wu, f.bu = br.proj_u.weight.data_ptr(), br.proj_u.bias.data_ptr()
        f.wB, f.bB = br.proj_B.weight.data_ptr(), br.proj_B.bias.data_ptr()
        f.wC, f.bC = br.proj_C.weight.data_ptr(), br.proj_C.bias.data_ptr()
        f.wo, f.bo = br.proj_out.weight.data_ptr(), br.proj_out.bias.data_ptr()
        f.lam, f.log_dt, f.D, f.mean, f.var = [z.data_ptr() for z in ins[:5]]
        f.eps, f.eta, f.var_eps = eps_value(br.gate), br.gate.norm_eta, br.obs_norm.eps
        f.dt_init, f.dt_min, f.dt_max = br.dt_init, 1e-3, host_float(br.dt_max)
        f.cpi_modulation = float(br.gate.cpi_modulation) if cpi is not None else 0.0
        f.temperature = host_float(br.gate.temperature)
        f.gate_mode = 1 if _gate_mode(br) == "soft" else 0
        f.H, f.N = br.H, br.N
        f.h_in, f.t_in, f.u_in, f.B_in, f.C_in, f.init_in = [z.data_ptr() for z in ins[5:]]
        f.h_out, f.t_out, f.u_out, f.B_out, f.C_out, f.init_out = [z.data_ptr() for z in outs]
        new.append((type(st), outs))
    y = torch.empty(B, d, dtype=torch.float32, device=dev)
    weights = torch.empty(B, S, dtype=torch.float32, device=dev)
    gate, resid, innov = (torch.empty(S, B, dtype=torch.float32, device=dev) for _ in range(3))
    L_ = _lib.lib()
    nbytes = int(L_.eacs_stream_frame_workspace_size(ctypes.byref(arr), S, B, d))
    require(nbytes > 0, "eacs_stream_frame: unsupported sizes")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    # the timestamp check (streaming.py:60-61) reads the previous frame's state, so
    # its host synchronisation comes last: the frame above was prepared while the
    # previous one still ran on the GPU
    bad = None
    for state in states:
        b = vb & state.initialized & (t < state.t)
        bad = b if bad is None else bad | b
    if bad is not None and bool(bad.any()):
        raise ValueError("timestamps must not precede the last committed observation")
    with torch.cuda.device(dev):
        _lib.check(L_.eacs_stream_frame(
            keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), ptr(keep[3]), ctypes.byref(arr), S,
            temporal.fusion.weight.data_ptr(), temporal.fusion.bias.data_ptr(), temporal.out_norm.weight.data_ptr(),
            temporal.out_norm.bias.data_ptr(), float(temporal.out_norm.eps), y.data_ptr(), weights.data_ptr(),
            gate.data_ptr(), resid.data_ptr(), innov.data_ptr(), ws.data_ptr(), ws.numel(), B, d,
            _lib.stream_ptr(dev)), "eacs_stream_frame")
    new = [cls(*outs[:5], outs[5].view(torch.bool)) for cls, outs in new]  # the kernel wrote 0 / 1
    return y, gate.t(), resid.t(), innov.t(), weights, new


def streaming_fusable(temporal, x: Tensor, states) -> bool:
    if not x.is_cuda:
        return False
    for br in temporal.branches:
        if br.disc_mode != "continuous" or getattr(br.gate, "gate_kind", "event") != "event":
            return False
    return True


def make_temporal_step(original):
    def dispatch(temporal, x, t, states, valid, cpi=None):
        if streaming_fusable(temporal, x, states):
            return temporal_step(temporal, x, t, states, valid, cpi)
        return original(temporal, x, t, states, valid, cpi)
    dispatch.__wrapped__ = original
    return dispatch
