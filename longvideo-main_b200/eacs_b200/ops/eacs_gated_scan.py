"""Gated EACS cell forward on B200 (mirrors cst_ssm/ops/eacs_gated_scan.py).

`eacs_cell_forward` keeps the reference signature (eacs_gated_scan.py:35-49)
and adds the two behaviours the reference only has in Python
(modules/eacs.py:145-173 scan_range): `robust` (a RobustCfg-like object or a
(k, spike_ratio, eps_factor) tuple) and `gate_mode="soft"`.  `EXT` is a
drop-in for the reference's JIT extension object (`eacs_cell_fwd`, bound at
cst_ssm/ops/csrc/eacs_cell_cuda.cu:225-227).

u may be float32, float16 or bfloat16: the kernel reads it in place (the
reference casts it to float32 first; the values are the same).  y is float32.
"""
from __future__ import annotations

import contextlib
import contextvars

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require


def _robust_tuple(robust):
    if robust is None:
        return 0, 0, 2.0, 0.3
    if isinstance(robust, (tuple, list)):
        k, ratio, factor = robust
    else:
        k, ratio, factor = robust.k, robust.spike_ratio, robust.eps_factor
    return 1, int(k), float(ratio), float(factor)


def workspace_bytes(B: int, L: int, H: int, N: int) -> int:
    return int(_lib.lib().eacs_cell_fwd_workspace_size(B, L, H, N))


# Cells the caller is launching side by side on separate streams (the
# branches of a MultiScaleEACS forward); set by side_by_side().
_SIDE_BY_SIDE = contextvars.ContextVar("eacs_cells_side_by_side", default=1)


@contextlib.contextmanager
def side_by_side(n: int):
    """Cells launched inside this block run n at a time on separate streams:
    eacs_cell_forward then lays out the speculative pass so that the n cells
    together fit the GPU in one wave (eacs_cell_fwd_side_by_side)."""
    tok = _SIDE_BY_SIDE.set(max(1, int(n)))
    try:
        yield
    finally:
        _SIDE_BY_SIDE.reset(tok)


def cell_forward_into(lam, log_dt_scale, u, Bc, Cc, t, D, mean, var, eps, eta, var_eps,
                      dt_init, dt_min, dt_max, robust, gate_mode, temperature,
                      y, gates, resid, workspace):
    """Launch the kernel on prepared (contiguous, correctly typed) tensors."""
    B, L, H = u.shape
    N = lam.shape[1]
    rb, rk, rr, rf = _robust_tuple(robust)
    args = (lam.data_ptr(), log_dt_scale.data_ptr(), u.data_ptr(), _lib.DTYPE_CODES[u.dtype],
            Bc.data_ptr(), Cc.data_ptr(), t.data_ptr(), D.data_ptr(), mean.data_ptr(), var.data_ptr(),
            float(eps), float(eta), float(var_eps), float(dt_init), float(dt_min), float(dt_max),
            rb, rk, rr, rf, 1 if gate_mode == "soft" else 0, float(temperature),
            y.data_ptr(), gates.data_ptr(), resid.data_ptr(),
            workspace.data_ptr() if workspace is not None else None,
            workspace.numel() if workspace is not None else 0,
            B, L, H, N)
    k = _SIDE_BY_SIDE.get()
    if k > 1:
        _lib.check(_lib.lib().eacs_cell_fwd_side_by_side(*args, k, _lib.stream_ptr(u.device)),
                   "eacs_cell_fwd_side_by_side")
    else:
        _lib.check(_lib.lib().eacs_cell_fwd(*args, _lib.stream_ptr(u.device)), "eacs_cell_fwd")


def prepare(lam, log_dt_scale, u, Bc, Cc, t, D, mean, var):
    dev = cuda_tensors("eacs_cell_forward", lam, log_dt_scale, u, Bc, Cc, t, D, mean, var)
    require(u.dim() == 3 and lam.dim() == 2, "u:(B,L,H), lam:(H,N)")
    require(lam.size(0) == u.size(2), "lam's H must match u's H")
    B, L, H = u.shape
    N = lam.shape[1]
    require(Bc.shape == (B, L, N) and Cc.shape == (B, L, N), "Bc, Cc: (B,L,N)")
    require(t.shape == (B, L), "t: (B,L)")
    if u.dtype not in _lib.DTYPE_CODES:
        u = u.float()
    return dev, (lam.to(torch.complex64).contiguous(), log_dt_scale.float().contiguous(),
                 u.contiguous(), Bc.to(torch.complex64).contiguous(),
                 Cc.to(torch.complex64).contiguous(), t.float().contiguous(),
                 D.float().contiguous(), mean.float().contiguous(), var.float().contiguous())


def gated_kernel_available() -> bool:
    if not torch.cuda.is_available():
        return False
    _lib.lib()
    return True


@torch.no_grad()
def eacs_cell_forward(lam: Tensor, log_dt_scale: Tensor, u: Tensor, Bc: Tensor,
                      Cc: Tensor, t: Tensor, D: Tensor, mean: Tensor, var: Tensor,
                      eps: float, eta: float, var_eps: float = 1e-5,
                      dt_init: float = 1.0, dt_min: float = 1e-3, dt_max: float = 1e3,
                      robust=None, gate_mode: str = "hard", temperature: float = 0.1):
    """Fused forward; returns (ys[B,L,H] fp32, gates[B,L], resid[B,L])."""
    require(gate_mode in ("hard", "soft"), "gate_mode must be 'hard' or 'soft'")
    dev, (lam_c, log_c, u_c, B_c, C_c, t_c, D_c, m_c, v_c) = prepare(
        lam, log_dt_scale, u, Bc, Cc, t, D, mean, var)
    B, L, H = u_c.shape
    N = lam_c.shape[1]
    y = torch.empty(B, L, H, dtype=torch.float32, device=dev)
    gates = torch.empty(B, L, dtype=torch.float32, device=dev)
    resid = torch.empty(B, L, dtype=torch.float32, device=dev)
    if y.numel() == 0:
        return y, gates, resid
    ws = torch.empty(workspace_bytes(B, L, H, N), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        cell_forward_into(lam_c, log_c, u_c, B_c, C_c, t_c, D_c, m_c, v_c, eps, eta, var_eps,
                          dt_init, dt_min, dt_max, robust, gate_mode, temperature,
                          y, gates, resid, ws)
    return y, gates, resid


def _host_tensor(name, x, dtype):
    require(isinstance(x, Tensor) and not x.is_cuda, f"eacs_cell_forward_host: {name} must be a host tensor")
    x = x if x.dtype == dtype else x.to(dtype)
    return x.contiguous()


@torch.no_grad()
def eacs_cell_forward_host(lam: Tensor, log_dt_scale: Tensor, u: Tensor, Bc: Tensor, Cc: Tensor,
                           t: Tensor, D: Tensor, mean: Tensor, var: Tensor, eps: float,
                           eta: float, var_eps: float = 1e-5, dt_init: float = 1.0,
                           dt_min: float = 1e-3, dt_max: float = 1e3, robust=None,
                           chunk: int = 512, out=None):
    """eacs_cell_forward (hard gate) with u, Bc, Cc, t and the outputs in host
    memory: the time chunks' copies overlap the cell of neighbouring chunks
    (eacs_cell_fwd_host).  Parameters stay on the device.  Host inputs should
    be pinned (Tensor.pin_memory()); `out` = (y, gates, resid) pinned host
    tensors to write into, else they are allocated pinned.  Returns them;
    they are complete once the current stream has synchronised."""
    dev = cuda_tensors("eacs_cell_forward_host", lam, log_dt_scale, D, mean, var)
    require(u.dim() == 3 and lam.dim() == 2 and lam.size(0) == u.size(2), "u:(B,L,H), lam:(H,N)")
    B, L, H = u.shape
    N = lam.shape[1]
    require(Bc.shape == (B, L, N) and Cc.shape == (B, L, N) and t.shape == (B, L),
            "Bc, Cc: (B,L,N), t: (B,L)")
    u_h = u.contiguous() if u.dtype in _lib.DTYPE_CODES else u.float().contiguous()
    require(not u_h.is_cuda, "eacs_cell_forward_host: u must be a host tensor")
    B_h = _host_tensor("Bc", Bc, torch.complex64)
    C_h = _host_tensor("Cc", Cc, torch.complex64)
    t_h = _host_tensor("t", t, torch.float32)
    params = (lam.to(torch.complex64).contiguous(), log_dt_scale.float().contiguous(),
              D.float().contiguous(), mean.float().contiguous(), var.float().contiguous())
    if out is None:
        out = (torch.empty(B, L, H, dtype=torch.float32, pin_memory=True),
               torch.empty(B, L, dtype=torch.float32, pin_memory=True),
               torch.empty(B, L, dtype=torch.float32, pin_memory=True))
    y, gates, resid = out
    require(y.shape == (B, L, H) and gates.shape == (B, L) and resid.shape == (B, L)
            and not y.is_cuda and y.dtype == torch.float32 and y.is_contiguous(),
            "eacs_cell_forward_host: out = (y (B,L,H), gates, resid (B,L)) float32 host tensors")
    if y.numel() == 0:
        return y, gates, resid
    rb, rk, rr, rf = _robust_tuple(robust)
    L_ = _lib.lib()
    nbytes = int(L_.eacs_cell_fwd_host_workspace_size(B, L, H, N, int(chunk)))
    require(nbytes > 0, f"eacs_cell_fwd_host: unsupported sizes B={B} L={L} H={H} N={N}")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L_.eacs_cell_fwd_host(
            *[p.data_ptr() for p in params], u_h.data_ptr(), _lib.DTYPE_CODES[u_h.dtype],
            B_h.data_ptr(), C_h.data_ptr(), t_h.data_ptr(), float(eps), float(eta),
            float(var_eps), float(dt_init), float(dt_min), float(dt_max), rb, rk, rr, rf,
            y.data_ptr(), gates.data_ptr(), resid.data_ptr(), ws.data_ptr(), ws.numel(),
            B, L, H, N, int(chunk), _lib.stream_ptr(dev)), "eacs_cell_fwd_host")
    # Lifetimes: the workspace and converted parameters are device memory of
    # this stream, which the call leaves waiting for all its copies; converted
    # host inputs are pageable, whose copies are staged before the call
    # returns; the caller's own pinned tensors must stay alive until the
    # stream has synchronised, as with any asynchronous copy.
    return y, gates, resid


class _CellExt:
    """Object with the reference extension's method (eacs_cell_cuda.cu:170-175)."""

    @staticmethod
    def eacs_cell_fwd(lam, log_dt, u, Bc, Cc, t, Dp, mean, var, eps, eta, var_eps, dt_init,
                      dt_min, dt_max):
        y, g, r = eacs_cell_forward(lam, log_dt, u, Bc, Cc, t, Dp, mean, var, eps, eta,
                                    var_eps, dt_init, dt_min, dt_max)
        return [y, g, r]


EXT = _CellExt()


def _load():
    _lib.lib()
    return EXT
