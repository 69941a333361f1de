"""Per-frame commits and continuous-time queries on B200.

Mirrors cst_ssm/modules/eacs.py:386-439 (EACSLayer.run_with_commits) and
cst_ssm/modules/continuous_query.py:12-65 (segment_index,
readout_from_commits, continuous_query):

* `cell_commits` runs the gated cell (hard gate) and records, after every
  frame, the committed state h_pi (B,L,H,N) and t_pi, u_pi, B_pi, C_pi, in one
  pass of the cell kernels instead of the reference's Python step loop;
* `segment_index` and `readout_from_commits` evolve a frame's commits to query
  times in one kernel (8 B of h_pi read per (query, h, n)).

These are inference paths: their outputs carry no autograd history.
`install(..., queries=True)` binds them to the reference with a dispatcher
that keeps the reference's own implementation where gradients must flow
through the commits or the gate is CPI-modulated.
"""
from __future__ import annotations

import sys

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require
from .eacs_gated_scan import prepare


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


@torch.no_grad()
def run_with_commits(layer, x: Tensor, timestamps: Tensor, cpi: Tensor | None = None,
                     use_chunk: bool | None = None):
    """EACSLayer.run_with_commits (eacs.py:404-439): (EACSOutput, commits).

    As in the reference's _commit_range, robust_guard is not applied here."""
    x_in = x
    xn = layer.norm(x)
    u, Bc, Cc = layer._project(xn)
    lam = layer.lam().to(torch.complex64)
    t = timestamps.float()
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
    y = query_readout(commits["lam"], commits["log_dt_scale"], layer.D, commits, t_query, idx,
                      dt_max=float(commits.get("dt_max", 1e3)))
    return layer.proj_out(y)


def continuous_query(layer, x: Tensor, timestamps: Tensor, t_query: Tensor,
                     cpi: Tensor | None = None, use_chunk: bool | None = None) -> Tensor:
    """continuous_query.py:56-61: x (B,L,d), timestamps (B,L), t_query (B,Q) -> (B,Q,d)."""
    _, commits = run_with_commits(layer, x, timestamps, cpi=cpi, use_chunk=use_chunk)
    return readout_from_commits(layer, commits, t_query)


# ---------------------------------------------------------------------------
# dispatch used by install(): ours where it applies, the reference's otherwise
# ---------------------------------------------------------------------------
def _needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(isinstance(t, Tensor) and t.requires_grad for t in ts)


def commits_fusable(layer, x: Tensor, cpi: Tensor | None) -> bool:
    if not x.is_cuda or layer.disc_mode != "continuous":
        return False
    if getattr(layer.gate, "gate_kind", "event") != "event":
        return False
    if cpi is not None and getattr(layer.gate, "cpi_modulation", 0.0) != 0:
        return False
    return not _needs_grad(x, *layer.parameters())


def make_run_with_commits(original):
    def dispatch(self, x, timestamps, cpi=None, use_chunk=None):
        if commits_fusable(self, x, cpi):
            return run_with_commits(self, x, timestamps, cpi=cpi, use_chunk=use_chunk)
        return original(self, x, timestamps, cpi=cpi, use_chunk=use_chunk)
    dispatch.__wrapped__ = original
    return dispatch


def make_readout_from_commits(original):
    def dispatch(layer, commits, t_query, idx=None):
        h = commits["h"]
        if h.is_cuda and not _needs_grad(h, commits["u"], commits["B"], commits["C"], commits["t"],
                                         commits["lam"], commits["log_dt_scale"], layer.D):
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
