"""Per-frame commits and continuous-time queries on B200.

Mirrors cst_ssm/modules/eacs.py:386-439 (EACSLayer.run_with_commits) and
cst_ssm/modules/continuous_query.py:12-65 (segment_index,
readout_from_commits, continuous_query):

* `cell_commits` runs the gated cell (hard gate) and records, after every
  frame, the committed state h_pi (B,L,H,N) and t_pi, u_pi, B_pi, C_pi, in one
  pass of the cell kernels instead of the reference's Python step loop;
* `segment_index` and `readout_from_commits` evolve a frame's commits to query
  times in one kernel (8 B of h_pi read per (query, h, n)).

* `CellCommitsFunction` and `QueryReadoutFunction` are the same two steps
  under autograd (training through continuous queries): the training forward
  (STE or soft gate) with a replay that records the commits, and backwards
  that carry the commits' adjoints into the cell's reverse scan
  (eacs_cell_train_commits_fwd/_bwd, eacs_query_readout_bwd).

`install(..., queries=True)` binds these to the reference with a dispatcher;
the reference's own implementation runs only where the gate is
CPI-modulated or not an event gate, or the discretisation is not continuous.
"""
from __future__ import annotations

import sys

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require
from .eacs_gated_scan import prepare, workspace_bytes


@torch.no_grad()
def cell_commits(lam, log_dt_scale, u, Bc, Cc, t, D, mean, var, eps, eta, var_eps=1e-5,
                 dt_init=1.0, dt_min=1e-3, dt_max=1e3, robust=None):
    """Hard-gate cell with per-frame commits.

    Returns (ys (B,L,H) fp32, gates, resid (B,L), commits) with commits a dict
    h (B,L,H,N) complex64, t (B,L), u (B,L,H) fp32, B, C (B,L,N) complex64."""
    dev, (lam_c, log_c, u_c, B_c, C_c, t_c, D_c, m_c, v_c) = prepare(
        lam, log_dt_scale, u, Bc, Cc, t, D, mean, var)
    B, L, H = u_c.shape
    N = lam_c.shape[1]
    f32 = dict(dtype=torch.float32, device=dev)
    c64 = dict(dtype=torch.complex64, device=dev)
    ys = torch.empty(B, L, H, **f32)
    gates = torch.empty(B, L, **f32)
    resid = torch.empty(B, L, **f32)
    commits = dict(h=torch.empty(B, L, H, N, **c64), t=torch.empty(B, L, **f32),
                   u=torch.empty(B, L, H, **f32), B=torch.empty(B, L, N, **c64),
                   C=torch.empty(B, L, N, **c64))
    if ys.numel() == 0:
        return ys, gates, resid, commits
    if robust is None:
        rb = (0, 3, 2.0, 0.3)
    else:
        k, ratio, factor = (robust.k, robust.spike_ratio, robust.eps_factor) if hasattr(robust, "k") \
            else robust
        rb = (1, int(k), float(ratio), float(factor))
    L_ = _lib.lib()
    nbytes = int(L_.eacs_cell_commits_workspace_size(B, L, H, N))
    require(nbytes > 0, f"eacs_cell_commits: unsupported sizes B={B} L={L} H={H} N={N}")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L_.eacs_cell_commits(
            lam_c.data_ptr(), log_c.data_ptr(), u_c.data_ptr(), _lib.DTYPE_CODES[u_c.dtype],
            B_c.data_ptr(), C_c.data_ptr(), t_c.data_ptr(), D_c.data_ptr(), m_c.data_ptr(),
            v_c.data_ptr(), float(eps), float(eta), float(var_eps), float(dt_init), float(dt_min),
            float(dt_max), *rb, ys.data_ptr(), gates.data_ptr(), resid.data_ptr(),
            commits["h"].data_ptr(), commits["t"].data_ptr(), commits["u"].data_ptr(),
            commits["B"].data_ptr(), commits["C"].data_ptr(), ws.data_ptr(), ws.numel(),
            B, L, H, N, _lib.stream_ptr(dev)), "eacs_cell_commits")
    return ys, gates, resid, commits


@torch.no_grad()
def segment_index(frame_t: Tensor, t_query: Tensor) -> Tensor:
    """Last k with frame_t[k] <= t* per query, clamped to [0, L-1]; (B,Q) int64
    (continuous_query.py:12-17)."""
    dev = cuda_tensors("segment_index", frame_t, t_query)
    ft = frame_t.float().contiguous()
    tq = t_query.float().contiguous()
    B, L = ft.shape
    Q = tq.shape[1]
    require(tq.shape[0] == B, "segment_index: batch mismatch")
    idx = torch.empty(B, Q, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().eacs_query_index(ft.data_ptr(), tq.data_ptr(), idx.data_ptr(), B, L, Q,
                                               _lib.stream_ptr(dev)), "eacs_query_index")
    return idx.long()


@torch.no_grad()
def query_readout(lam, log_dt_scale, D, commits: dict, t_query: Tensor, idx: Tensor | None = None,
                  dt_min: float = 1e-3, dt_max: float = 1e3) -> Tensor:
    """readout_from_commits before proj_out: (B,Q,H) fp32."""
    h = commits["h"]
    dev = cuda_tensors("query_readout", lam, log_dt_scale, D, h, commits["t"], commits["u"],
                       commits["B"], commits["C"], t_query)
    B, L, H, N = h.shape
    tq = t_query.float().contiguous()
    Q = tq.shape[1]
    require(tq.shape[0] == B and lam.shape == (H, N), "query_readout: shape mismatch")
    if idx is None:
        idx = segment_index(commits["frame_t"], tq)
    idx32 = idx.to(torch.int32).contiguous()
    parts = [lam.to(torch.complex64).contiguous(), log_dt_scale.float().contiguous(),
             D.float().contiguous(), h.to(torch.complex64).contiguous(),
             commits["t"].float().contiguous(), commits["u"].float().contiguous(),
             commits["B"].to(torch.complex64).contiguous(),
             commits["C"].to(torch.complex64).contiguous()]
    y = torch.empty(B, Q, H, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().eacs_query_readout(*[p.data_ptr() for p in parts], tq.data_ptr(),
                                                 idx32.data_ptr(), y.data_ptr(), B, L, Q, H, N,
                                                 float(dt_min), float(dt_max), _lib.stream_ptr(dev)),
                   "eacs_query_readout")
    return y


_GATE_MODES = {"ste": 0, "soft": 1, "hard": 2}


class CellCommitsFunction(torch.autograd.Function):
    """EACSLayer._commit_range (eacs.py:386-401) under autograd, after the
    projections: (ys, gates, resid, h, t_pi, u_pi, B_pi, C_pi) per frame with
    the training gate (gate_mode "ste": hard forward, soft backward; "soft")
    or the eval gate ("hard": r > eps, no gradient through it).  The backward is one reverse scan over the checkpoints the forward's replay
    wrote, with the commits' upstream adjoints joining at their steps."""

    @staticmethod
    def forward(ctx, u, Bc, Cc, t, lam, log_dt, D, eps, mean, var, T, eta, var_eps, dt_init,
                gate_mode, dt_max):
        ctx.set_materialize_grads(False)
        cuda_tensors("CellCommitsFunction", u, Bc, Cc, t, lam, log_dt, D, mean, var)
        dev, prep = prepare(lam, log_dt, u, Bc, Cc, t, D, mean, var)
        lam_c, log_c, u_c, B_c, C_c, t_c, D_c, m_c, v_c = prep
        B, L, H = u_c.shape
        N = lam_c.shape[1]
        f32 = dict(dtype=torch.float32, device=dev)
        c64 = dict(dtype=torch.complex64, device=dev)
        ys, gs, rs = torch.empty(B, L, H, **f32), torch.empty(B, L, **f32), torch.empty(B, L, **f32)
        stats = torch.empty(B, L, 2, **f32)
        ch, ct = torch.empty(B, L, H, N, **c64), torch.empty(B, L, **f32)
        cu, cB, cC = torch.empty(B, L, H, **f32), torch.empty(B, L, N, **c64), torch.empty(B, L, N, **c64)
        eps_v = float(eps)
        bwd_ws = None
        if ys.numel():
            L_ = _lib.lib()
            nbytes = int(L_.eacs_cell_train_commits_workspace_size(B, L, H, N))
            require(nbytes > 0, f"eacs_cell_train_commits_fwd: unsupported sizes B={B} L={L} H={H} N={N}")
            bwd_ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            ws = torch.empty(workspace_bytes(B, L, H, N), dtype=torch.uint8, device=dev)
            with torch.cuda.device(dev):
                _lib.check(L_.eacs_cell_train_commits_fwd(
                    lam_c.data_ptr(), log_c.data_ptr(), u_c.data_ptr(), _lib.DTYPE_CODES[u_c.dtype],
                    B_c.data_ptr(), C_c.data_ptr(), t_c.data_ptr(), D_c.data_ptr(), m_c.data_ptr(),
                    v_c.data_ptr(), eps_v, float(eta), float(var_eps), float(dt_init), 1e-3,
                    float(dt_max), _GATE_MODES[gate_mode], float(T), ys.data_ptr(),
                    gs.data_ptr(), rs.data_ptr(), stats.data_ptr(), ch.data_ptr(), ct.data_ptr(),
                    cu.data_ptr(), cB.data_ptr(), cC.data_ptr(), ws.data_ptr(), ws.numel(),
                    bwd_ws.data_ptr(), bwd_ws.numel(), B, L, H, N, _lib.stream_ptr(dev)),
                    "eacs_cell_train_commits_fwd")
        ctx.prep, ctx.bwd_ws, ctx.gate_mode = prep, bwd_ws, _GATE_MODES[gate_mode]
        ctx.save_for_backward(gs, rs, stats)
        ctx.hp = (eps_v, float(T), float(eta), float(var_eps), float(dt_init), float(dt_max))
        ctx.dtypes = (u.dtype, Bc.dtype, Cc.dtype, t.dtype, lam.dtype, log_dt.dtype, D.dtype,
                      eps.dtype if torch.is_tensor(eps) else None,
                      eps.shape if torch.is_tensor(eps) else None)
        return ys, gs, rs, ch, ct, cu, cB, cC

    @staticmethod
    def backward(ctx, g_ys, g_gs, g_rs, g_ch, g_ct, g_cu, g_cB, g_cC):
        gs, rs, stats = ctx.saved_tensors
        lam_c, log_c, u_c, B_c, C_c, t_c, D_c, m_c, v_c = ctx.prep
        eps_v, T, eta, var_eps, dt_init, dt_max = ctx.hp
        dev = u_c.device
        B, L, H = u_c.shape
        N = lam_c.shape[1]
        gy = torch.zeros(B, L, H, dtype=torch.float32, device=dev) if g_ys is None else g_ys.float().contiguous()
        ggs, grs = (None if g is None else g.float().contiguous() for g in (g_gs, g_rs))
        gch = None if g_ch is None else g_ch.to(torch.complex64).contiguous()
        gct, gcu = (None if g is None else g.float().contiguous() for g in (g_ct, g_cu))
        gcB, gcC = (None if g is None else g.to(torch.complex64).contiguous() for g in (g_cB, g_cC))
        du = torch.empty(B, L, H, dtype=torch.float32, device=dev)
        dBc = torch.empty(B, L, N, dtype=torch.complex64, device=dev)
        dCc = torch.empty_like(dBc)
        dt = torch.empty(B, L, dtype=torch.float32, device=dev)
        dlam = torch.empty(H, N, dtype=torch.complex64, device=dev)
        dlog = torch.empty(H, dtype=torch.float32, device=dev)
        dD = torch.empty(H, dtype=torch.float32, device=dev)
        deps = torch.empty(1, dtype=torch.float32, device=dev)
        if du.numel():
            ws = ctx.bwd_ws
            with torch.cuda.device(dev):
                _lib.check(_lib.lib().eacs_cell_train_commits_bwd(
                    lam_c.data_ptr(), log_c.data_ptr(), u_c.data_ptr(), _lib.DTYPE_CODES[u_c.dtype],
                    B_c.data_ptr(), C_c.data_ptr(), t_c.data_ptr(), D_c.data_ptr(), m_c.data_ptr(),
                    v_c.data_ptr(), eps_v, eta, var_eps, dt_init, 1e-3, dt_max, ctx.gate_mode, T,
                    gs.data_ptr(),
                    rs.data_ptr(), stats.data_ptr(), gy.data_ptr(), _lib.ptr(ggs), _lib.ptr(grs),
                    _lib.ptr(gch), _lib.ptr(gct), _lib.ptr(gcu), _lib.ptr(gcB), _lib.ptr(gcC),
                    du.data_ptr(), dBc.data_ptr(), dCc.data_ptr(), dt.data_ptr(), dlam.data_ptr(),
                    dlog.data_ptr(), dD.data_ptr(), deps.data_ptr(), ws.data_ptr(), ws.numel(),
                    B, L, H, N, _lib.stream_ptr(dev)), "eacs_cell_train_commits_bwd")
        else:
            for x in (du, dBc, dCc, dt, dlam, dlog, dD, deps):
                x.zero_()
        u_t, B_t, C_t, t_t, lam_t, log_t, D_t, eps_t, eps_shape = ctx.dtypes
        deps_out = None if eps_t is None else deps.to(eps_t).reshape(eps_shape)
        return (du.to(u_t), dBc.to(B_t), dCc.to(C_t), dt.to(t_t), dlam.to(lam_t), dlog.to(log_t),
                dD.to(D_t), deps_out, None, None, None, None, None, None, None, None)


def cell_commits_train(lam, log_dt_scale, u, Bc, Cc, t, D, mean, var, eps, eta, T, gate_mode,
                       var_eps=1e-5, dt_init=1.0, dt_max=1e3):
    """The differentiable counterpart of cell_commits: (ys, gates, resid,
    commits) with the training gate ("ste" or "soft")."""
    ys, gs, rs, ch, ct, cu, cB, cC = CellCommitsFunction.apply(
        u, Bc, Cc, t, lam, log_dt_scale, D, eps, mean, var, T, eta, var_eps, dt_init, gate_mode, dt_max)
    return ys, gs, rs, dict(h=ch, t=ct, u=cu, B=cB, C=cC)


class QueryReadoutFunction(torch.autograd.Function):
    """readout_from_commits before proj_out (continuous_query.py:20-54) under
    autograd: y (B,Q,H) from the commits at idx, and the adjoints of the
    commits, lam, log_dt_scale, D and the query times."""

    @staticmethod
    def forward(ctx, lam, log_dt, D, h, ct, cu, cB, cC, t_query, idx, dt_min, dt_max):
        ctx.set_materialize_grads(False)
        dev = cuda_tensors("QueryReadoutFunction", lam, log_dt, D, h, ct, cu, cB, cC, t_query, idx)
        B, L, H, N = h.shape
        parts = [lam.to(torch.complex64).contiguous(), log_dt.float().contiguous(), D.float().contiguous(),
                 h.to(torch.complex64).contiguous(), ct.float().contiguous(), cu.float().contiguous(),
                 cB.to(torch.complex64).contiguous(), cC.to(torch.complex64).contiguous()]
        tq = t_query.float().contiguous()
        Q = tq.shape[1]
        require(tq.shape[0] == B and lam.shape == (H, N), "QueryReadoutFunction: shape mismatch")
        idx32 = idx.to(torch.int32).contiguous()
        y = torch.empty(B, Q, H, dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().eacs_query_readout(*[p.data_ptr() for p in parts], tq.data_ptr(),
                                                     idx32.data_ptr(), y.data_ptr(), B, L, Q, H, N,
                                                     float(dt_min), float(dt_max), _lib.stream_ptr(dev)),
                       "eacs_query_readout")
        ctx.parts, ctx.tq, ctx.idx = parts, tq, idx32
        ctx.lim = (float(dt_min), float(dt_max))
        ctx.dtypes = (lam.dtype, log_dt.dtype, D.dtype, h.dtype, ct.dtype, cu.dtype, cB.dtype, cC.dtype,
                      t_query.dtype)
        return y

    @staticmethod
    def backward(ctx, gy):
        parts, tq, idx = ctx.parts, ctx.tq, ctx.idx
        dev = tq.device
        B, L, H, N = parts[3].shape
        Q = tq.shape[1]
        f32 = dict(dtype=torch.float32, device=dev)
        c64 = dict(dtype=torch.complex64, device=dev)
        gc = [torch.empty(B, L, H, N, **c64), torch.empty(B, L, **f32), torch.empty(B, L, H, **f32),
              torch.empty(B, L, N, **c64), torch.empty(B, L, N, **c64)]
        dlam, dlog, dD = torch.empty(H, N, **c64), torch.empty(H, **f32), torch.empty(H, **f32)
        gy = (torch.zeros(B, Q, H, **f32) if gy is None else gy.float()).contiguous()
        # the kernel takes each frame's queries contiguous: sort by frame
        # (stable), and scatter the query times' adjoints back
        order = None
        if Q > 1 and not bool((idx[:, 1:] >= idx[:, :-1]).all()):
            idx, order = torch.sort(idx, dim=1, stable=True)
            tq = torch.gather(tq, 1, order)
            gy = torch.gather(gy, 1, order[..., None].expand(B, Q, H)).contiguous()
            idx = idx.contiguous()
        want_tq = ctx.needs_input_grad[8]
        gtq = torch.empty(B, Q, **f32) if want_tq else None
        L_ = _lib.lib()
        ws = torch.empty(int(L_.eacs_query_readout_bwd_workspace_size(B, L, Q, H, N)), dtype=torch.uint8,
                         device=dev)
        with torch.cuda.device(dev):
            _lib.check(L_.eacs_query_readout_bwd(
                *[p.data_ptr() for p in parts], tq.data_ptr(), idx.data_ptr(), gy.data_ptr(),
                *[g.data_ptr() for g in gc], _lib.ptr(gtq), dlam.data_ptr(), dlog.data_ptr(),
                dD.data_ptr(), ws.data_ptr(), ws.numel(), B, L, Q, H, N, *ctx.lim,
                _lib.stream_ptr(dev)), "eacs_query_readout_bwd")
        if gtq is not None and order is not None:
            gtq = torch.empty_like(gtq).scatter_(1, order, gtq)
        dt = ctx.dtypes
        out = [dlam.to(dt[0]), dlog.to(dt[1]), dD.to(dt[2])] + [g.to(d) for g, d in zip(gc, dt[3:8])]
        out.append(None if gtq is None else gtq.to(dt[8]))
        return (*out, None, None, None)


def _needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(isinstance(t, Tensor) and t.requires_grad for t in ts)


def run_with_commits(layer, x: Tensor, timestamps: Tensor, cpi: Tensor | None = None,
                     use_chunk: bool | None = None):
    """EACSLayer.run_with_commits (eacs.py:404-439): (EACSOutput, commits).

    In eval mode (hard gate) without gradients, the commit kernels; in
    training mode or where gradients flow, CellCommitsFunction with the gate
    the reference's EventGate uses (STE or soft, its temperature).  As in the
    reference's _commit_range, robust_guard is not applied here; use_chunk
    (the reference's activation checkpointing) changes nothing here: the
    backward recomputes from its own checkpoints."""
    x_in = x
    xn = layer.norm(x)
    u, Bc, Cc = layer._project(xn)
    lam = layer.lam().to(torch.complex64)
    t = timestamps.float()
    train_gate = layer.training
    if train_gate or _needs_grad(x, u, Bc, Cc, t, lam, layer.log_dt_scale, layer.D,
                                 getattr(layer.gate, "eps_raw", None)):
        gate = layer.gate
        mode = ("ste" if gate.use_ste else "soft") if train_gate else "hard"
        eps = gate.eps
        T = float(gate.temperature)
        ys, gates, resid, commits = cell_commits_train(
            lam, layer.log_dt_scale, u, Bc, Cc, t, layer.D, layer.obs_norm.running_mean,
            layer.obs_norm.running_var, eps, gate.norm_eta, T, mode, layer.obs_norm.eps, layer.dt_init,
            layer.dt_max)
        if not train_gate:
            gates = gates.detach()  # eval: (r > eps) is a constant
    else:
        with torch.no_grad():
            ys, gates, resid, commits = cell_commits(
                lam, layer.log_dt_scale, u, Bc, Cc, t, layer.D, layer.obs_norm.running_mean,
                layer.obs_norm.running_var, float(layer.gate.eps.item()), layer.gate.norm_eta,
                layer.obs_norm.eps, layer.dt_init, 1e-3, layer.dt_max)
    delta = layer.proj_out(ys.to(x_in.dtype))
    y = x_in + delta if layer.add_residual else delta
    commits.update(lam=lam, frame_t=t, log_dt_scale=layer.log_dt_scale, dt_max=layer.dt_max)
    EACSOutput = sys.modules[type(layer).__module__].EACSOutput
    return EACSOutput(y=y, gates=gates, update_rate=gates.mean(), residual=resid), commits


def readout_from_commits(layer, commits: dict, t_query: Tensor, idx: Tensor | None = None) -> Tensor:
    """continuous_query.py:20-61: (B,Q,d) readouts at t_query."""
    frame_t = commits["frame_t"]
    if t_query is frame_t:
        B, L = frame_t.shape
        idx = torch.arange(L, device=frame_t.device).expand(B, L)
    dt_max = float(commits.get("dt_max", 1e3))
    ins = (commits["lam"], commits["log_dt_scale"], layer.D, commits["h"], commits["t"], commits["u"],
           commits["B"], commits["C"], t_query)
    if _needs_grad(*ins):
        if idx is None:
            idx = segment_index(frame_t, t_query)
        y = QueryReadoutFunction.apply(*ins, idx, 1e-3, dt_max)
    else:
        y = query_readout(commits["lam"], commits["log_dt_scale"], layer.D, commits, t_query, idx,
                          dt_max=dt_max)
    return layer.proj_out(y)


def continuous_query(layer, x: Tensor, timestamps: Tensor, t_query: Tensor,
                     cpi: Tensor | None = None, use_chunk: bool | None = None) -> Tensor:
    """continuous_query.py:56-61: x (B,L,d), timestamps (B,L), t_query (B,Q) -> (B,Q,d)."""
    _, commits = run_with_commits(layer, x, timestamps, cpi=cpi, use_chunk=use_chunk)
    return readout_from_commits(layer, commits, t_query)


# ---------------------------------------------------------------------------
# dispatch used by install(): ours where it applies, the reference's otherwise
# ---------------------------------------------------------------------------
def commits_fusable(layer, x: Tensor, cpi: Tensor | None) -> bool:
    if not x.is_cuda or layer.disc_mode != "continuous":
        return False
    if getattr(layer.gate, "gate_kind", "event") != "event":
        return False
    return cpi is None or getattr(layer.gate, "cpi_modulation", 0.0) == 0


def make_run_with_commits(original):
    def dispatch(self, x, timestamps, cpi=None, use_chunk=None):
        if commits_fusable(self, x, cpi):
            return run_with_commits(self, x, timestamps, cpi=cpi, use_chunk=use_chunk)
        return original(self, x, timestamps, cpi=cpi, use_chunk=use_chunk)
    dispatch.__wrapped__ = original
    return dispatch


def make_readout_from_commits(original):
    def dispatch(layer, commits, t_query, idx=None):
        if commits["h"].is_cuda and t_query.is_cuda:
            return readout_from_commits(layer, commits, t_query, idx)
        return original(layer, commits, t_query, idx)
    dispatch.__wrapped__ = original
    return dispatch


def make_segment_index(original):
    def dispatch(frame_t, t_query):
        if frame_t.is_cuda and t_query.is_cuda:
            return segment_index(frame_t, t_query)
        return original(frame_t, t_query)
    dispatch.__wrapped__ = original
    return dispatch
